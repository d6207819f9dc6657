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
#include "gdn_stream.cuh"
#include "sm100.cuh"

namespace gdn {
namespace {

template <int RPW, int MINB, bool L2NORM, bool HAS_STATE, typename ST>
__global__ void __launch_bounds__(256, MINB)
    decode_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                  const __nv_bfloat16* __restrict__ v, const ST* state,
                  const float* __restrict__ A_log, const __nv_bfloat16* __restrict__ a,
                  const float* __restrict__ dt_bias, const __nv_bfloat16* __restrict__ b,
                  float scale, __nv_bfloat16* __restrict__ out, ST* new_state,
                  const RowStrides rs, int HV, int ratio) {
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
  RS::load_bf16(q + (size_t)bidx * rs.q + qh * kHeadDim, j, qf);
  RS::load_bf16(k + (size_t)bidx * rs.k + qh * kHeadDim, j, kf);
  float vv[NG];
  const __nv_bfloat16* vp = v + (size_t)bidx * rs.v + h * kHeadDim + row0;
#pragma unroll
  for (int r = 0; r < NG; ++r) vv[r] = bf2f(vp[4 * r]);
  const float g =
      expf(gate_log_g(__ldg(A_log + h), bf2f(a[(size_t)bidx * rs.a + h]), __ldg(dt_bias + h)));
  const float beta = sigmoid_f(bf2f(b[(size_t)bidx * rs.b + h]));

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
  __nv_bfloat16* op = out + (size_t)bidx * rs.o + h * kHeadDim + row0;
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

template <int RPW, int MINB, typename ST>
cudaError_t launch_rpw(const void* q, const void* k, const void* v, const ST* state,
                       const float* A_log, const void* a, const float* dt_bias, const void* b,
                       float scale, void* out, ST* new_state, int batch, int HQ, int HV,
                       const RowStrides& rs, bool l2norm, cudaStream_t stream) {
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
      decode_kernel<RPW, MINB, true, true, ST><<<grid, block, 0, stream>>>(Q, K, V, state, A_log, A, dt_bias, Bt, scale, O, new_state, rs, HV, ratio);
    else
      decode_kernel<RPW, MINB, false, true, ST><<<grid, block, 0, stream>>>(Q, K, V, state, A_log, A, dt_bias, Bt, scale, O, new_state, rs, HV, ratio);
  } else {
    if (l2norm)
      decode_kernel<RPW, MINB, true, false, ST><<<grid, block, 0, stream>>>(Q, K, V, state, A_log, A, dt_bias, Bt, scale, O, new_state, rs, HV, ratio);
    else
      decode_kernel<RPW, MINB, false, false, ST><<<grid, block, 0, stream>>>(Q, K, V, state, A_log, A, dt_bias, Bt, scale, O, new_state, rs, HV, ratio);
  }
  return cudaGetLastError();
}

inline bool misaligned(const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) != 0; }

}  // namespace
}  // namespace gdn

namespace gdn {
namespace {
// ------------------------------------------------------------ streaming variant
// For batches that fill the GPU: a persistent kernel (one or two CTAs per SM) whose
// copy warp streams each head's state, q, k and v rows into a ring of shared-memory
// stages with plain bulk copies (cp.async.bulk, mbarrier completion), while 8 compute
// warps work on the stage before it.  Up to (stages - 1) heads of state are in flight
// per CTA at any time, independent of how long the compute warps take, so HBM sees a
// steady stream instead of the load-all / compute / store waves of decode_kernel.
// Rows are read from the stage one at a time (few registers per thread).  Per row the
// arithmetic is decode_kernel's, in the same order (identical results).
__device__ unsigned int g_decode_device_error = 0;
constexpr unsigned kDecodeErrCopyTimeout = 1u;  // a stage's copies never landed
constexpr unsigned kDecodeErrFreeTimeout = 8u;  // a stage was never released

template <typename ST>
struct StreamCfg {
  static constexpr uint32_t kStateBytes = kHeadDim * kHeadDim * sizeof(ST);
  static constexpr uint32_t kStage = kStateBytes + 1024;  // state | q | k | v (256 B each)
  static constexpr int kStages = 3;
  static constexpr int kCtasPerSm = sizeof(ST) == 2 ? 2 : 1;
  static constexpr uint32_t kBars = kStages * kStage;
  static constexpr uint32_t kSmem = kBars + 64;
  static constexpr int kThreads = 288;  // 8 compute warps + the copy warp
};

__device__ __forceinline__ bool stream_wait(uint64_t* bar, uint32_t parity,
                                            volatile int* abort_flag, unsigned code) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (sm100::mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort_flag) return false;
  }
  atomicOr(&g_decode_device_error, code);
  *abort_flag = 1;
  return false;
}

template <bool L2NORM, typename ST>
__global__ void __launch_bounds__(StreamCfg<ST>::kThreads, StreamCfg<ST>::kCtasPerSm)
    decode_stream_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                         const __nv_bfloat16* __restrict__ v, const ST* state,
                         const float* __restrict__ A_log, const __nv_bfloat16* __restrict__ a,
                         const float* __restrict__ dt_bias, const __nv_bfloat16* __restrict__ b,
                         float scale, __nv_bfloat16* __restrict__ out, ST* new_state,
                         const RowStrides rs, int HV, int ratio, int heads) {
  using C = StreamCfg<ST>;
  using RS = RowSlice<ST>;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sb = sm100::smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBars);
  uint64_t* empty = full + C::kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + C::kStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int nmine = heads > (int)blockIdx.x ? (heads - 1 - (int)blockIdx.x) / G + 1 : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 8);
    }
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();

  if (warp == 8) {
    // ============================== copy warp
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nmine; ++i) {
        const int slot = i % C::kStages;
        if (i >= C::kStages &&
            !stream_wait(&empty[slot], ((i / C::kStages) - 1) & 1, abort_flag, kDecodeErrFreeTimeout))
          break;
        const int bh = (int)blockIdx.x + i * G;
        const int bidx = bh / HV, h = bh - bidx * HV, qh = h / ratio;
        uint8_t* st = smem + (size_t)slot * C::kStage;
        sm100::mbar_arrive_expect_tx(&full[slot], C::kStateBytes + 768u);
        sm100::bulk_load(st, state + (size_t)bh * kHeadDim * kHeadDim, C::kStateBytes, &full[slot]);
        sm100::bulk_load(st + C::kStateBytes, q + (size_t)bidx * rs.q + qh * kHeadDim, 256u, &full[slot]);
        sm100::bulk_load(st + C::kStateBytes + 256, k + (size_t)bidx * rs.k + qh * kHeadDim, 256u, &full[slot]);
        sm100::bulk_load(st + C::kStateBytes + 512, v + (size_t)bidx * rs.v + h * kHeadDim, 256u, &full[slot]);
        issued = i + 1;
      }
      if (*abort_flag) {  // let copies still in flight land before the CTA exits (bounded)
        for (int i = issued - C::kStages > 0 ? issued - C::kStages : 0; i < issued; ++i)
          sm100::mbar_wait(&full[i % C::kStages], (i / C::kStages) & 1, 1u << 20);
      }
    }
    return;
  }
  // ============================== compute warps: 16 rows each (rows row0 + 4r)
  const int sub = lane >> 3, j = lane & 7;
  const int row0 = warp * 16 + sub;
  scale = default_scale(scale);
  // gate inputs of the next head, loaded one head ahead
  auto load_gate_inputs = [&](int i, float& al, float& av, float& db, float& bv) {
    const int bh = (int)blockIdx.x + i * G;
    const int bidx = bh / HV, h = bh - bidx * HV;
    al = __ldg(A_log + h);
    db = __ldg(dt_bias + h);
    av = bf2f(a[(size_t)bidx * rs.a + h]);
    bv = bf2f(b[(size_t)bidx * rs.b + h]);
  };
  float nal = 0.f, nav = 0.f, ndb = 0.f, nbv = 0.f;
  if (nmine > 0) load_gate_inputs(0, nal, nav, ndb, nbv);
  for (int i = 0; i < nmine; ++i) {
    const float al = nal, av = nav, db = ndb, bv = nbv;
    if (i + 1 < nmine) load_gate_inputs(i + 1, nal, nav, ndb, nbv);
    const int slot = i % C::kStages;
    if (!stream_wait(&full[slot], (i / C::kStages) & 1, abort_flag, kDecodeErrCopyTimeout)) break;
    const int bh = (int)blockIdx.x + i * G;
    const uint32_t st = sb + (uint32_t)slot * C::kStage;
    float kf[16], qf[16], vv[4];
    load_vec_smem<ST>(st + C::kStateBytes, j, qf);
    load_vec_smem<ST>(st + C::kStateBytes + 256u, j, kf);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      uint16_t bits;
      asm volatile("ld.shared.u16 %0, [%1];" : "=h"(bits)
                   : "r"(st + C::kStateBytes + 512u + 2u * (uint32_t)(row0 + 4 * r)));
      vv[r] = __uint_as_float((uint32_t)bits << 16);
    }
    const float g = expf(gate_log_g(al, av, db));
    const float beta = sigmoid_f(bv);
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
    ST* nsp = new_state + (size_t)bh * kHeadDim * kHeadDim + (size_t)row0 * kHeadDim;
    __nv_bfloat16* op = out + (size_t)(bh / HV) * rs.o + (bh % HV) * kHeadDim + row0;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float Sr[16];
      load_row_smem<ST>(st + (uint32_t)((row0 + 4 * r) * kHeadDim * sizeof(ST)), j, Sr);
      if (r == 3) {  // this warp's last read of the stage: release it
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&empty[slot]);
      }
      float sk = 0.f, sq = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        sk = fmaf(Sr[e], kf[e], sk);
        sq = fmaf(Sr[e], qf[e], sq);
      }
      sk = xor_sum8(sk);
      sq = xor_sum8(sq);
      const float old = g * sk;
      const float delta = beta * (vv[r] - old);
#pragma unroll
      for (int e = 0; e < 16; ++e) Sr[e] = fmaf(g, Sr[e], delta * kf[e]);
      RS::store(nsp + r * 4 * kHeadDim, j, Sr);
      if (j == 0) op[4 * r] = __float2bfloat16_rn(scale * fmaf(g, sq, delta * kq));
    }
  }
}

template <typename ST>
cudaError_t launch_stream(const void* q, const void* k, const void* v, const ST* state,
                          const float* A_log, const void* a, const float* dt_bias, const void* b,
                          float scale, void* out, ST* new_state, int batch, int HQ, int HV,
                          const RowStrides& rs, bool l2norm, cudaStream_t stream) {
  using C = StreamCfg<ST>;
  static int sms[64] = {};
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    if (cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return cudaErrorInvalidValue;
    cudaError_t e1 = cudaFuncSetAttribute(decode_stream_kernel<true, ST>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    cudaError_t e2 = cudaFuncSetAttribute(decode_stream_kernel<false, ST>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e1 != cudaSuccess || e2 != cudaSuccess) return cudaErrorInvalidValue;
    configured[dev] = true;
  }
  const int heads = batch * HV;
  const int grid = heads < sms[dev] * C::kCtasPerSm ? heads : sms[dev] * C::kCtasPerSm;
  auto Q = static_cast<const __nv_bfloat16*>(q);
  auto K = static_cast<const __nv_bfloat16*>(k);
  auto V = static_cast<const __nv_bfloat16*>(v);
  auto A = static_cast<const __nv_bfloat16*>(a);
  auto Bt = static_cast<const __nv_bfloat16*>(b);
  auto O = static_cast<__nv_bfloat16*>(out);
  if (l2norm)
    decode_stream_kernel<true, ST><<<grid, C::kThreads, C::kSmem, stream>>>(
        Q, K, V, state, A_log, A, dt_bias, Bt, scale, O, new_state, rs, HV, HV / HQ, heads);
  else
    decode_stream_kernel<false, ST><<<grid, C::kThreads, C::kSmem, stream>>>(
        Q, K, V, state, A_log, A, dt_bias, Bt, scale, O, new_state, rs, HV, HV / HQ, heads);
  return cudaGetLastError();
}
}  // namespace

// Device error bits of the streaming decode kernel (bounded waits that ran out).
unsigned read_decode_device_error(bool clear) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_decode_device_error, sizeof(v)) != cudaSuccess) return ~0u;
  if (clear && v != 0) {
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_decode_device_error, &zero, sizeof(zero)) != cudaSuccess) return ~0u;
  }
  return v;
}
}  // namespace gdn

namespace gdn {
namespace {
// Where the streaming kernel is the faster one (measured on B200): bf16 state from a
// few waves of heads on.
template <typename ST>
bool stream_pays(long long heads) {
  return sizeof(ST) == 2 && heads >= 4 * 148;
}

template <typename ST>
int decode_entry(const void* q, const void* k, const void* v, const ST* state, const float* A_log,
                 const void* a, const float* dt_bias, const void* b, float scale, void* output,
                 ST* new_state, int batch, int num_q_heads, int num_k_heads, int num_v_heads,
                 int head_size, int use_qk_l2norm, void* stream,
                 const RowStrides* strides = nullptr) {
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
  const RowStrides rs = strides ? *strides : dense_rows(num_q_heads, num_v_heads);
  const long long qk_row = (long long)num_q_heads * kHeadDim, v_row = (long long)num_v_heads * kHeadDim;
  // rows of one tensor never overlap; q/k rows keep their 8-byte alignment
  if (rs.q < qk_row || rs.k < qk_row || rs.v < v_row || rs.o < v_row || rs.a < num_v_heads ||
      rs.b < num_v_heads || rs.q % 4 != 0 || rs.k % 4 != 0)
    return GDN_ERR_INVALID_ARGUMENT;
  const long long heads = (long long)batch * num_v_heads;
  if (heads * 4 > 0x7fffffffLL) return GDN_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool l2 = use_qk_l2norm != 0;
  cudaError_t err;
  // Batches that fill the GPU several times over: the streaming kernel (bulk copies
  // need 16-byte aligned q, k, v rows); otherwise one-shot CTAs, bigger when there are
  // enough heads to fill 148 SMs several times over.
  const bool rows16 = !misaligned(q, 16) && !misaligned(k, 16) && !misaligned(v, 16) &&
                      rs.q % 8 == 0 && rs.k % 8 == 0 && rs.v % 8 == 0;
  if (state != nullptr && stream_pays<ST>(heads) && rows16)
    err = launch_stream<ST>(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, batch,
                            num_q_heads, num_v_heads, rs, l2, st);
  // CTA sizing, measured on B200 with L2 cold (ncu launch times, 32 v-heads): from 256
  // heads on, 128 rows per CTA at two CTAs per SM (B = 8: 7.7 us against 8.9 us with 32
  // rows; B = 16: 11.5 against 13.0 us with 64); below that 32 rows per CTA, four CTAs per
  // SM (registers capped at 64) once three per SM would need a second wave (B = 4: 5.8
  // against 6.4 us), else three per SM (B = 1: 4.0 us; the cap costs 0.6 us there).
  else if (heads >= 256)
    err = launch_rpw<16, 2, ST>(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, batch, num_q_heads, num_v_heads, rs, l2, st);
  else if (heads * 4 > 3 * 148 && sizeof(ST) == 4)  // (the bf16 variant would spill)
    err = launch_rpw<4, 4, ST>(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, batch, num_q_heads, num_v_heads, rs, l2, st);
  else
    err = launch_rpw<4, 1, ST>(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, batch, num_q_heads, num_v_heads, rs, l2, st);
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

extern "C" int gdn_decode_launch_strided(const void* q, const void* k, const void* v,
                                         const float* state, const float* A_log, const void* a,
                                         const float* dt_bias, const void* b, float scale,
                                         void* output, float* new_state, int batch,
                                         int num_q_heads, int num_k_heads, int num_v_heads,
                                         int head_size, int use_qk_l2norm, long long q_stride,
                                         long long k_stride, long long v_stride,
                                         long long a_stride, long long b_stride,
                                         long long output_stride, void* stream) {
  const gdn::RowStrides rs{q_stride, k_stride, v_stride, a_stride, b_stride, output_stride};
  return gdn::decode_entry<float>(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state,
                                  batch, num_q_heads, num_k_heads, num_v_heads, head_size,
                                  use_qk_l2norm, stream, &rs);
}
