// GDN decode for sm_100a: one fused, single-pass HBM-streaming kernel.
//
// Replaces gdn_decode_kernel (reference gdn_decode/solution/triton/kernel.py:71-218).
// Per (batch b, v-head h) the state S[v, k] (k-last, 128 x 128 fp32 = 64 KiB) is
// read once and written once.  For every row v:
//   sk = S[v,:].k   sq = S[v,:].q            (one shuffle-reduction pass)
//   old = g * sk ;  delta = beta * (v_v - old)
//   S'[v,:] = g * S[v,:] + delta * k
//   o_v = scale * S'[v,:].q = scale * (g * sq + delta * (k.q))
// so the output needs no second pass over the state (the reference's two-pass
// K-tiled configurations re-read it, kernel.py:176-213).
//
// The state may also be stored as bf16 (gdn_decode_launch_bf16state, the bf16-state
// backend of FlashInfer's decode, flashinfer/gdn_decode.py:146-149): it is widened to
// fp32 on load, updated in fp32 and rounded to nearest bf16 on store, halving the
// state traffic.
//
// Thread mapping: 8 lanes own one state row, each lane 16 columns accessed 16 bytes
// at a time (fp32: 4 float4 at columns 4j + 32m; bf16: 2 x 8 values at 8j + 64m;
// j = lane % 8), so every 128-bit load instruction of a warp covers four fully used
// 128-byte segments.  A warp owns RPW rows, a CTA
// of 8 warps owns 8*RPW rows of one head; all of a thread's state loads are
// issued before any arithmetic so each SM keeps ~64-128 KiB in flight.
#include "gdn_common.cuh"

namespace gdn {
namespace {

template <int RPW, bool L2NORM, bool HAS_STATE, typename ST>
__global__ void __launch_bounds__(256)
    decode_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                  const __nv_bfloat16* __restrict__ v, const ST* state,
                  const float* __restrict__ A_log, const __nv_bfloat16* __restrict__ a,
                  const float* __restrict__ dt_bias, const __nv_bfloat16* __restrict__ b,
                  float scale, __nv_bfloat16* __restrict__ out, ST* new_state, int HQ,
                  int HV, int ratio) {
  constexpr int ROWS = 8 * RPW;            // state rows per CTA
  constexpr int VSPLIT = kHeadDim / ROWS;  // CTAs per (b, h)
  constexpr int NG = RPW / 4;              // 4-row groups per warp
  const int cta = blockIdx.x;
  const int bh = cta / VSPLIT;
  const int vs = cta - bh * VSPLIT;
  const int bidx = bh / HV;
  const int h = bh - bidx * HV;
  const int qh = h / ratio;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 3;
  const int j = lane & 7;
  const int row0 = vs * ROWS + warp * RPW + sub;  // rows row0 + 4r, r < NG
  const size_t head_base = (size_t)bh * kHeadDim * kHeadDim;

  // ---- issue the state loads first ----
  using RS = RowSlice<ST>;
  float S[NG][16];
  if constexpr (HAS_STATE) {
    const ST* sp = state + head_base + (size_t)row0 * kHeadDim;
#pragma unroll
    for (int r = 0; r < NG; ++r) RS::load(sp + r * 4 * kHeadDim, j, S[r]);
  } else {
#pragma unroll
    for (int r = 0; r < NG; ++r)
#pragma unroll
      for (int e = 0; e < 16; ++e) S[r][e] = 0.f;
  }

  // ---- q, k slices (the lane's 16 columns), v values, gates ----
  float kf[16], qf[16];
  RS::load_bf16(q + ((size_t)bidx * HQ + qh) * kHeadDim, j, qf);
  RS::load_bf16(k + ((size_t)bidx * HQ + qh) * kHeadDim, j, kf);
  float vv[NG];
  const __nv_bfloat16* vp = v + (size_t)bh * kHeadDim + row0;
#pragma unroll
  for (int r = 0; r < NG; ++r) vv[r] = bf2f(vp[4 * r]);
  const float g = expf(gate_log_g(__ldg(A_log + h), bf2f(a[bh]), __ldg(dt_bias + h)));
  const float beta = sigmoid_f(bf2f(b[bh]));

  if constexpr (L2NORM) {
    float ssk = 0.f, ssq = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      ssk = fmaf(kf[e], kf[e], ssk);
      ssq = fmaf(qf[e], qf[e], ssq);
    }
    ssk = xor_sum8(ssk);
    ssq = xor_sum8(ssq);
    const float rk = rsqrtf(ssk + kL2NormEps);
    const float rq = rsqrtf(ssq + kL2NormEps);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      kf[e] *= rk;
      qf[e] *= rq;
    }
  }
  float kq = 0.f;
#pragma unroll
  for (int e = 0; e < 16; ++e) kq = fmaf(kf[e], qf[e], kq);
  kq = xor_sum8(kq);

  scale = default_scale(scale);
  ST* nsp = new_state + head_base + (size_t)row0 * kHeadDim;
  __nv_bfloat16* op = out + (size_t)bh * kHeadDim + row0;
#pragma unroll
  for (int r = 0; r < NG; ++r) {
    float sk = 0.f, sq = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      sk = fmaf(S[r][e], kf[e], sk);
      sq = fmaf(S[r][e], qf[e], sq);
    }
    sk = xor_sum8(sk);
    sq = xor_sum8(sq);
    const float old = g * sk;
    const float delta = beta * (vv[r] - old);
#pragma unroll
    for (int e = 0; e < 16; ++e) S[r][e] = fmaf(g, S[r][e], delta * kf[e]);
    RS::store(nsp + r * 4 * kHeadDim, j, S[r]);
    if (j == 0) op[4 * r] = __float2bfloat16_rn(scale * fmaf(g, sq, delta * kq));
  }
}

template <int RPW, typename ST>
cudaError_t launch_rpw(const void* q, const void* k, const void* v, const ST* state,
                       const float* A_log, const void* a, const float* dt_bias, const void* b,
                       float scale, void* out, ST* new_state, int batch, int HQ, int HV,
                       bool l2norm, cudaStream_t stream) {
  constexpr int VSPLIT = kHeadDim / (8 * RPW);
  const long long ctas = (long long)batch * HV * VSPLIT;
  const dim3 grid((unsigned)ctas), block(256);
  const int ratio = HV / HQ;
  auto Q = static_cast<const __nv_bfloat16*>(q);
  auto K = static_cast<const __nv_bfloat16*>(k);
  auto V = static_cast<const __nv_bfloat16*>(v);
  auto A = static_cast<const __nv_bfloat16*>(a);
  auto Bt = static_cast<const __nv_bfloat16*>(b);
  auto O = static_cast<__nv_bfloat16*>(out);
  if (state != nullptr) {
    if (l2norm)
      decode_kernel<RPW, true, true, ST><<<grid, block, 0, stream>>>(Q, K, V, state, A_log, A, dt_bias, Bt, scale, O, new_state, HQ, HV, ratio);
    else
      decode_kernel<RPW, false, true, ST><<<grid, block, 0, stream>>>(Q, K, V, state, A_log, A, dt_bias, Bt, scale, O, new_state, HQ, HV, ratio);
  } else {
    if (l2norm)
      decode_kernel<RPW, true, false, ST><<<grid, block, 0, stream>>>(Q, K, V, state, A_log, A, dt_bias, Bt, scale, O, new_state, HQ, HV, ratio);
    else
      decode_kernel<RPW, false, false, ST><<<grid, block, 0, stream>>>(Q, K, V, state, A_log, A, dt_bias, Bt, scale, O, new_state, HQ, HV, ratio);
  }
  return cudaGetLastError();
}

inline bool misaligned(const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) != 0; }

}  // namespace
}  // namespace gdn

namespace gdn {
namespace {
template <typename ST>
int decode_entry(const void* q, const void* k, const void* v, const ST* state, const float* A_log,
                 const void* a, const float* dt_bias, const void* b, float scale, void* output,
                 ST* new_state, int batch, int num_q_heads, int num_k_heads, int num_v_heads,
                 int head_size, int use_qk_l2norm, void* stream) {
  if (batch < 0 || num_q_heads <= 0 || num_k_heads <= 0 || num_v_heads <= 0)
    return GDN_ERR_INVALID_ARGUMENT;
  if (head_size != kHeadDim || num_k_heads != num_q_heads || num_v_heads % num_q_heads != 0)
    return GDN_ERR_UNSUPPORTED;
  if (batch == 0) return GDN_OK;
  if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !output || !new_state)
    return GDN_ERR_INVALID_ARGUMENT;
  if (misaligned(q, 8) || misaligned(k, 8) || misaligned(v, 2) || misaligned(output, 2) ||
      misaligned(new_state, 16) || (state && misaligned(state, 16)))
    return GDN_ERR_INVALID_ARGUMENT;
  const long long heads = (long long)batch * num_v_heads;
  if (heads * 4 > 0x7fffffffLL) return GDN_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool l2 = use_qk_l2norm != 0;
  cudaError_t err;
  // Enough CTAs to fill 148 SMs several times over; bigger CTAs when there are.
  if (heads >= 4 * 148)
    err = launch_rpw<16, ST>(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, batch, num_q_heads, num_v_heads, l2, st);
  else if (heads >= 2 * 148)
    err = launch_rpw<8, ST>(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, batch, num_q_heads, num_v_heads, l2, st);
  else
    err = launch_rpw<4, ST>(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, batch, num_q_heads, num_v_heads, l2, st);
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
}  // namespace
}  // namespace gdn

extern "C" int gdn_decode_launch(const void* q, const void* k, const void* v, const float* state,
                                 const float* A_log, const void* a, const float* dt_bias,
                                 const void* b, float scale, void* output, float* new_state,
                                 int batch, int num_q_heads, int num_k_heads, int num_v_heads,
                                 int head_size, int use_qk_l2norm, void* stream) {
  return gdn::decode_entry<float>(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state,
                                  batch, num_q_heads, num_k_heads, num_v_heads, head_size,
                                  use_qk_l2norm, stream);
}

extern "C" int gdn_decode_launch_bf16state(const void* q, const void* k, const void* v,
                                           const void* state, const float* A_log, const void* a,
                                           const float* dt_bias, const void* b, float scale,
                                           void* output, void* new_state, int batch,
                                           int num_q_heads, int num_k_heads, int num_v_heads,
                                           int head_size, int use_qk_l2norm, void* stream) {
  return gdn::decode_entry<__nv_bfloat16>(
      q, k, v, static_cast<const __nv_bfloat16*>(state), A_log, a, dt_bias, b, scale, output,
      static_cast<__nv_bfloat16*>(new_state), batch, num_q_heads, num_k_heads, num_v_heads,
      head_size, use_qk_l2norm, stream);
}
