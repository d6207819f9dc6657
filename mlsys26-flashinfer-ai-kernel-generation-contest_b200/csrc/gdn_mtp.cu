// GDN multi-token decode (MTP / speculative-decoding verification) for sm_100a.
//
// Follows the definition reference _gdn_mtp_reference (flashinfer/trace/templates/
// gdn.py:379-466): for each batch row b the state of pool slot idx[b] (k-last
// [HV, V, K] fp32) is carried through T tokens, each one the decode update
//   old = g S k ;  delta = beta (v - old) ;  S' = g S + delta k ;  o = scale S' q
// with the per-token output written as bf16 and, optionally, the state after every
// token written to intermediate_states[idx[b], t] (rollback buffer).  The final
// state goes to final_state[idx[b]]; the pool may be updated in place.
//
// Same HBM-streaming structure as the decode kernel (gdn_decode.cu): 8 lanes own
// one 512-byte state row, the rows of one (b, v-head) are spread over 2-4 CTAs, and
// the state stays in registers across the T tokens, so the pool slot is read once
// and written once.  The next token's q/k/v/gates are loaded while the current
// token is applied.  A batch row whose index lies outside [0, pool_size) is a
// padding row: its outputs are zero and no state is read or written.  The pool and
// the rollback buffer may be bf16 (gdn_mtp_launch_bf16state): widened on load,
// carried in fp32 through the T tokens, rounded to nearest bf16 on every store.
#include "gdn_common.cuh"

namespace gdn {
namespace {

struct MtpToken {
  float kf[16], qf[16];
  float g, beta;
};

template <int NG, typename ST>
__device__ __forceinline__ void mtp_load_token(const __nv_bfloat16* __restrict__ q,
                                               const __nv_bfloat16* __restrict__ k,
                                               const __nv_bfloat16* __restrict__ v,
                                               const __nv_bfloat16* __restrict__ a,
                                               const __nv_bfloat16* __restrict__ b,
                                               size_t bt, int HQ, int HV, int qh, int h, int j,
                                               int row0, float nexpA, float dtb, MtpToken& tk,
                                               float (&vv)[NG]) {
  RowSlice<ST>::load_bf16(q + (bt * HQ + qh) * kHeadDim, j, tk.qf);
  RowSlice<ST>::load_bf16(k + (bt * HQ + qh) * kHeadDim, j, tk.kf);
  const __nv_bfloat16* vp = v + (bt * HV + h) * kHeadDim + row0;
#pragma unroll
  for (int r = 0; r < NG; ++r) vv[r] = bf2f(vp[4 * r]);
  // same expression as the decode kernel's gate_log_g, with exp(A_log) hoisted
  tk.g = expf(nexpA * softplus_f(bf2f(a[bt * HV + h]) + dtb));
  tk.beta = sigmoid_f(bf2f(b[bt * HV + h]));
}

template <int RPW, int MINB, bool L2NORM, bool INTER, typename IdxT, typename ST>
__global__ void __launch_bounds__(256, MINB)
    mtp_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
               const __nv_bfloat16* __restrict__ v, const ST* pool,
               const IdxT* __restrict__ indices, const float* __restrict__ A_log,
               const __nv_bfloat16* __restrict__ a, const float* __restrict__ dt_bias,
               const __nv_bfloat16* __restrict__ b, float scale, __nv_bfloat16* __restrict__ out,
               ST* new_pool, ST* __restrict__ inter, int T, long long pool_size, int HQ,
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
  const long long slot = (long long)indices[bidx];
  __nv_bfloat16* op0 = out + ((size_t)bidx * T * HV + h) * kHeadDim + row0;
  if (slot < 0 || slot >= pool_size) {  // padding row
    if (j == 0)
      for (int t = 0; t < T; ++t)
#pragma unroll
        for (int r = 0; r < NG; ++r) op0[(size_t)t * HV * kHeadDim + 4 * r] = __float2bfloat16_rn(0.f);
    return;
  }
  const size_t head_base = ((size_t)slot * HV + h) * kHeadDim * kHeadDim;

  using RS = RowSlice<ST>;
  float S[NG][16];
  {
    const ST* sp = pool + head_base + (size_t)row0 * kHeadDim;
#pragma unroll
    for (int r = 0; r < NG; ++r) RS::load(sp + r * 4 * kHeadDim, j, S[r]);
  }
  const float nexpA = -expf(__ldg(A_log + h));
  const float dtb = __ldg(dt_bias + h);
  scale = default_scale(scale);

  MtpToken cur;
  float vv[NG];
  mtp_load_token<NG, ST>(q, k, v, a, b, (size_t)bidx * T, HQ, HV, qh, h, j, row0, nexpA, dtb, cur, vv);
  for (int t = 0; t < T; ++t) {
    MtpToken nxt;
    float vn[NG];
    if (t + 1 < T)
      mtp_load_token<NG, ST>(q, k, v, a, b, (size_t)bidx * T + t + 1, HQ, HV, qh, h, j, row0, nexpA,
                         dtb, nxt, vn);
    if constexpr (L2NORM) {
      float ssk = 0.f, ssq = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        ssk = fmaf(cur.kf[e], cur.kf[e], ssk);
        ssq = fmaf(cur.qf[e], cur.qf[e], ssq);
      }
      ssk = xor_sum8(ssk);
      ssq = xor_sum8(ssq);
      const float rk = rsqrtf(ssk + kL2NormEps);
      const float rq = rsqrtf(ssq + kL2NormEps);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        cur.kf[e] *= rk;
        cur.qf[e] *= rq;
      }
    }
    float kq = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) kq = fmaf(cur.kf[e], cur.qf[e], kq);
    kq = xor_sum8(kq);
    const float g = cur.g, beta = cur.beta;
    __nv_bfloat16* op = op0 + (size_t)t * HV * kHeadDim;
    ST* ip = nullptr;
    if constexpr (INTER)
      ip = inter + (((size_t)slot * T + t) * HV + h) * kHeadDim * kHeadDim +
           (size_t)row0 * kHeadDim;
#pragma unroll
    for (int r = 0; r < NG; ++r) {
      float sk = 0.f, sq = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        sk = fmaf(S[r][e], cur.kf[e], sk);
        sq = fmaf(S[r][e], cur.qf[e], sq);
      }
      sk = xor_sum8(sk);
      sq = xor_sum8(sq);
      const float old = g * sk;
      const float delta = beta * (vv[r] - old);
#pragma unroll
      for (int e = 0; e < 16; ++e) S[r][e] = fmaf(g, S[r][e], delta * cur.kf[e]);
      if constexpr (INTER) RS::store(ip + r * 4 * kHeadDim, j, S[r]);
      if (j == 0) op[4 * r] = __float2bfloat16_rn(scale * fmaf(g, sq, delta * kq));
    }
    if (t + 1 < T) {
      cur = nxt;
#pragma unroll
      for (int r = 0; r < NG; ++r) vv[r] = vn[r];
    }
  }
  ST* nsp = new_pool + head_base + (size_t)row0 * kHeadDim;
#pragma unroll
  for (int r = 0; r < NG; ++r) RS::store(nsp + r * 4 * kHeadDim, j, S[r]);
}

template <int RPW, int MINB, typename IdxT, typename ST>
cudaError_t launch_mtp_rpw(const void* q, const void* k, const void* v, const ST* pool,
                           const void* indices, const float* A_log, const void* a,
                           const float* dt_bias, const void* b, float scale, void* out,
                           ST* new_pool, ST* inter, int batch, int T, long long pool_size,
                           int HQ, int HV, bool l2norm, cudaStream_t st) {
  constexpr int VSPLIT = kHeadDim / (8 * RPW);
  const dim3 grid((unsigned)((long long)batch * HV * VSPLIT)), block(256);
  auto Q = static_cast<const __nv_bfloat16*>(q);
  auto K = static_cast<const __nv_bfloat16*>(k);
  auto V = static_cast<const __nv_bfloat16*>(v);
  auto A = static_cast<const __nv_bfloat16*>(a);
  auto Bt = static_cast<const __nv_bfloat16*>(b);
  auto O = static_cast<__nv_bfloat16*>(out);
  auto I = static_cast<const IdxT*>(indices);
  const int ratio = HV / HQ;
#define GDN_MTP_LAUNCH(L2, IN)                                                                \
  mtp_kernel<RPW, MINB, L2, IN, IdxT, ST><<<grid, block, 0, st>>>(Q, K, V, pool, I, A_log, A, dt_bias, \
                                                        Bt, scale, O, new_pool, inter, T,    \
                                                        pool_size, HQ, HV, ratio)
  if (inter != nullptr) {
    if (l2norm) GDN_MTP_LAUNCH(true, true); else GDN_MTP_LAUNCH(false, true);
  } else {
    if (l2norm) GDN_MTP_LAUNCH(true, false); else GDN_MTP_LAUNCH(false, false);
  }
#undef GDN_MTP_LAUNCH
  return cudaGetLastError();
}

template <typename IdxT, typename ST>
cudaError_t launch_mtp(const void* q, const void* k, const void* v, const ST* pool,
                       const void* indices, const float* A_log, const void* a,
                       const float* dt_bias, const void* b, float scale, void* out,
                       ST* new_pool, ST* inter, int batch, int T, long long pool_size,
                       int HQ, int HV, bool l2norm, cudaStream_t st) {
  // Write-heavy (with the rollback buffer, T + 1 state writes per read): what matters is
  // how many stores each SM keeps in flight.  64 rows per CTA at two CTAs per SM (registers
  // capped at 128, no spills) overlaps one CTA's state loads with the other's stores; at
  // B = 128, T = 4 that is 259 us against 279 us for 128 rows at one CTA per SM, the rate of
  // a plain stream with the same 1 : 5 read / write mix.  Small batches: 32 rows per CTA.
  const long long heads = (long long)batch * HV;
  if (heads >= 2 * 148)
    return launch_mtp_rpw<8, 2, IdxT, ST>(q, k, v, pool, indices, A_log, a, dt_bias, b, scale, out,
                                          new_pool, inter, batch, T, pool_size, HQ, HV, l2norm, st);
  return launch_mtp_rpw<4, 1, IdxT, ST>(q, k, v, pool, indices, A_log, a, dt_bias, b, scale, out,
                                        new_pool, inter, batch, T, pool_size, HQ, HV, l2norm, st);
}

inline bool misaligned(const void* p, uintptr_t n) {
  return (reinterpret_cast<uintptr_t>(p) % n) != 0;
}

}  // namespace
}  // namespace gdn

namespace gdn {
namespace {
template <typename ST>
int mtp_entry(const void* q, const void* k, const void* v, const ST* initial_state,
              const void* state_indices, int state_indices_int64, const float* A_log,
              const void* a, const float* dt_bias, const void* b, float scale, void* output,
              ST* final_state, ST* intermediate_states, int batch, int seq_len, int pool_size,
              int num_q_heads, int num_k_heads, int num_v_heads, int head_size,
              int use_qk_l2norm, void* stream) {
  if (batch < 0 || seq_len < 0 || pool_size < 0 || num_q_heads <= 0 || num_k_heads <= 0 ||
      num_v_heads <= 0)
    return GDN_ERR_INVALID_ARGUMENT;
  if (head_size != kHeadDim || num_k_heads != num_q_heads || num_v_heads % num_q_heads != 0)
    return GDN_ERR_UNSUPPORTED;
  if (batch == 0 || seq_len == 0) return GDN_OK;
  if (!q || !k || !v || !initial_state || !state_indices || !A_log || !a || !dt_bias || !b ||
      !output || !final_state)
    return GDN_ERR_INVALID_ARGUMENT;
  constexpr uintptr_t sa = 16;  // 16-byte state accesses
  if (misaligned(q, 8) || misaligned(k, 8) || misaligned(v, 2) || misaligned(output, 2) ||
      misaligned(initial_state, sa) || misaligned(final_state, sa) ||
      (intermediate_states && misaligned(intermediate_states, sa)) ||
      misaligned(state_indices, state_indices_int64 ? 8 : 4))
    return GDN_ERR_INVALID_ARGUMENT;
  if ((long long)batch * num_v_heads * 4 > 0x7fffffffLL) return GDN_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool l2 = use_qk_l2norm != 0;
  const cudaError_t err =
      state_indices_int64
          ? launch_mtp<long long, ST>(q, k, v, initial_state, state_indices, A_log, a, dt_bias,
                                      b, scale, output, final_state, intermediate_states, batch,
                                      seq_len, pool_size, num_q_heads, num_v_heads, l2, st)
          : launch_mtp<int, ST>(q, k, v, initial_state, state_indices, A_log, a, dt_bias, b,
                                scale, output, final_state, intermediate_states, batch, seq_len,
                                pool_size, num_q_heads, num_v_heads, l2, st);
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
}  // namespace
}  // namespace gdn

extern "C" int gdn_mtp_launch(const void* q, const void* k, const void* v,
                              const float* initial_state, const void* state_indices,
                              int state_indices_int64, const float* A_log, const void* a,
                              const float* dt_bias, const void* b, float scale, void* output,
                              float* final_state, float* intermediate_states, int batch,
                              int seq_len, int pool_size, int num_q_heads, int num_k_heads,
                              int num_v_heads, int head_size, int use_qk_l2norm, void* stream) {
  return gdn::mtp_entry<float>(q, k, v, initial_state, state_indices, state_indices_int64, A_log,
                               a, dt_bias, b, scale, output, final_state, intermediate_states,
                               batch, seq_len, pool_size, num_q_heads, num_k_heads, num_v_heads,
                               head_size, use_qk_l2norm, stream);
}

extern "C" int gdn_mtp_launch_bf16state(const void* q, const void* k, const void* v,
                                        const void* initial_state, const void* state_indices,
                                        int state_indices_int64, const float* A_log,
                                        const void* a, const float* dt_bias, const void* b,
                                        float scale, void* output, void* final_state,
                                        void* intermediate_states, int batch, int seq_len,
                                        int pool_size, int num_q_heads, int num_k_heads,
                                        int num_v_heads, int head_size, int use_qk_l2norm,
                                        void* stream) {
  using B16 = __nv_bfloat16;
  return gdn::mtp_entry<B16>(q, k, v, static_cast<const B16*>(initial_state), state_indices,
                             state_indices_int64, A_log, a, dt_bias, b, scale, output,
                             static_cast<B16*>(final_state), static_cast<B16*>(intermediate_states),
                             batch, seq_len, pool_size, num_q_heads, num_k_heads, num_v_heads,
                             head_size, use_qk_l2norm, stream);
}
