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
// one 512-byte state row, the rows of one (b, v-head) are spread over 1-4 CTAs, and
// the state stays in registers across the T tokens, so the pool slot is read once
// and written once.  The next token's q/k/v/gates are loaded while the current
// token is applied.  A batch row whose index lies outside [0, pool_size) is a
// padding row: its outputs are zero and no state is read or written.  The pool and
// the rollback buffer may be bf16 (gdn_mtp_launch_bf16state): widened on load,
// carried in fp32 through the T tokens, rounded to nearest bf16 on every store.
#include "gdn_common.cuh"
#include "gdn_stream.cuh"
#include "sm100.cuh"

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

template <int RPW, bool L2NORM, bool INTER, typename IdxT, typename ST>
__global__ void __launch_bounds__(256)
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

// ------------------------------------------------------------ streaming variant
// With the rollback buffer a call writes T + 1 states per slot for every one it reads.
// mtp_kernel (one CTA per (row, v-head)) then stalls on every token: the next token's q,
// k, v and gates come from global memory while the token's own work is only a few hundred
// cycles, so each SM issues its stores in bursts and HBM idles between them.  This
// persistent variant (one CTA per SM) streams, a few items ahead, each item's slot state
// and the q, k, v rows of all its T tokens into a ring of shared-memory stages (plain bulk
// copies, mbarrier transaction counts); the gates of all T tokens are computed once per
// item, one token per lane.  The token loop then touches global memory only to store.
// Each of the 8 warps takes 16 rows of an item exactly as mtp_kernel<16> does (rows
// warp * 16 + sub + 4 r, the same columns per lane) and runs the T tokens with
// mtp_kernel's arithmetic in the same order (identical results).  Lane 0 of warp 0
// refills a stage once every warp has finished with it (a ninth copy warp would cap the
// registers at 168 and make the compute warps spill).  Every wait is bounded: one that
// runs out sets a bit of g_mtp_device_error and the CTA gives up (after letting its
// copies in flight land).
__device__ unsigned int g_mtp_device_error = 0;
constexpr unsigned kMtpErrCopyTimeout = 1u;  // a stage's copy never landed
constexpr unsigned kMtpErrFreeTimeout = 8u;  // a stage was never released
constexpr int kMtpStreamMaxT = 8;           // tokens whose q, k, v rows fit a stage

template <typename ST>
struct MtpStreamCfg {
  static constexpr uint32_t kStateBytes = kHeadDim * kHeadDim * sizeof(ST);
  static constexpr uint32_t kTokBytes = 3 * kHeadDim * 2;  // q | k | v rows, bf16
  static constexpr uint32_t kStage = kStateBytes + kMtpStreamMaxT * kTokBytes;
  static constexpr int kStages = sizeof(ST) == 4 ? 3 : 5;  // 210 / 190 KB
  static constexpr uint32_t kBars = kStages * kStage;
  static constexpr uint32_t kSmem = kBars + 128;
  static constexpr int kThreads = 256;
  static_assert(kSmem <= 232448, "shared memory budget");
};

__device__ __forceinline__ bool mtp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                         unsigned code) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (sm100::mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort_flag) return false;
  }
  atomicOr(&g_mtp_device_error, code);
  *abort_flag = 1;
  return false;
}

template <bool L2NORM, bool INTER, typename IdxT, typename ST>
__global__ void __launch_bounds__(MtpStreamCfg<ST>::kThreads, 1)
    mtp_stream_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                      const __nv_bfloat16* __restrict__ v, const ST* pool,
                      const IdxT* __restrict__ indices, const float* __restrict__ A_log,
                      const __nv_bfloat16* __restrict__ a, const float* __restrict__ dt_bias,
                      const __nv_bfloat16* __restrict__ b, float scale,
                      __nv_bfloat16* __restrict__ out, ST* new_pool, ST* __restrict__ inter,
                      int T, long long pool_size, int HQ, int HV, int ratio, int items) {
  using C = MtpStreamCfg<ST>;
  using RS = RowSlice<ST>;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sb = sm100::smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBars);
  uint64_t* empty = full + C::kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + C::kStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int nmine = items > (int)blockIdx.x ? (items - 1 - (int)blockIdx.x) / G + 1 : 0;
  const bool issuer = threadIdx.x == 0;
  // item i -> stage i % kStages: its slot state (state | q_0 k_0 v_0 | q_1 k_1 v_1 | ..);
  // a padding row has nothing to read
  auto issue = [&](int i) {
    const int stage = i % C::kStages;
    const int bh = (int)blockIdx.x + i * G;
    const int bidx = bh / HV, h = bh - bidx * HV, qh = h / ratio;
    const long long slot = (long long)indices[bidx];
    if (slot < 0 || slot >= pool_size) {
      sm100::mbar_arrive(&full[stage]);
      return;
    }
    uint8_t* dst = smem + (size_t)stage * C::kStage;
    sm100::mbar_arrive_expect_tx(&full[stage], C::kStateBytes + (uint32_t)T * C::kTokBytes);
    sm100::bulk_load(dst, pool + ((size_t)slot * HV + h) * kHeadDim * kHeadDim, C::kStateBytes,
                     &full[stage]);
    for (int t = 0; t < T; ++t) {
      const size_t bt = (size_t)bidx * T + t;
      uint8_t* tok = dst + C::kStateBytes + (size_t)t * C::kTokBytes;
      sm100::bulk_load(tok, q + (bt * HQ + qh) * kHeadDim, 256u, &full[stage]);
      sm100::bulk_load(tok + 256, k + (bt * HQ + qh) * kHeadDim, 256u, &full[stage]);
      sm100::bulk_load(tok + 512, v + (bt * HV + h) * kHeadDim, 256u, &full[stage]);
    }
  };
  int issued = 0;  // items whose copies were issued (thread 0)
  if (issuer) {
    for (int s = 0; s < C::kStages; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 8);
    }
    *abort_flag = 0;
    sm100::fence_mbar_init();
    for (; issued < C::kStages && issued < nmine; ++issued) issue(issued);
  }
  __syncthreads();

  constexpr int NG = 4;
  const int sub = lane >> 3, j = lane & 7;
  const int row0 = warp * 16 + sub;
  scale = default_scale(scale);
  for (int i = 0; i < nmine; ++i) {
    const int stage = i % C::kStages;
    const int bh = (int)blockIdx.x + i * G;
    const int bidx = bh / HV, h = bh - bidx * HV;
    // gates of token `lane` (lanes < T), the same expression as mtp_load_token
    float gl = 0.f, bl = 0.f;
    if (lane < T) {
      const size_t ti = ((size_t)bidx * T + lane) * HV + h;
      gl = expf(-expf(__ldg(A_log + h)) * softplus_f(bf2f(a[ti]) + __ldg(dt_bias + h)));
      bl = sigmoid_f(bf2f(b[ti]));
    }
    if (!mtp_wait(&full[stage], (i / C::kStages) & 1, abort_flag, kMtpErrCopyTimeout)) break;
    const long long slot = (long long)indices[bidx];
    __nv_bfloat16* op0 = out + ((size_t)bidx * T * HV + h) * kHeadDim + row0;
    if (slot >= 0 && slot < pool_size) {
      const uint32_t st = sb + (uint32_t)stage * C::kStage;
      float S[NG][16];
#pragma unroll
      for (int r = 0; r < NG; ++r)
        load_row_smem<ST>(st + (uint32_t)((row0 + 4 * r) * kHeadDim * sizeof(ST)), j, S[r]);
      for (int t = 0; t < T; ++t) {
        const uint32_t tok = st + C::kStateBytes + (uint32_t)t * C::kTokBytes;
        float kf[16], qf[16], vv[NG];
        load_vec_smem<ST>(tok, j, qf);
        load_vec_smem<ST>(tok + 256u, j, kf);
#pragma unroll
        for (int r = 0; r < NG; ++r) {
          uint16_t bits;
          asm volatile("ld.shared.u16 %0, [%1];" : "=h"(bits)
                       : "r"(tok + 512u + 2u * (uint32_t)(row0 + 4 * r)));
          vv[r] = __uint_as_float((uint32_t)bits << 16);
        }
        const float g = __shfl_sync(0xffffffffu, gl, t);
        const float beta = __shfl_sync(0xffffffffu, bl, t);
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
            sk = fmaf(S[r][e], kf[e], sk);
            sq = fmaf(S[r][e], qf[e], sq);
          }
          sk = xor_sum8(sk);
          sq = xor_sum8(sq);
          const float old = g * sk;
          const float delta = beta * (vv[r] - old);
#pragma unroll
          for (int e = 0; e < 16; ++e) S[r][e] = fmaf(g, S[r][e], delta * kf[e]);
          if constexpr (INTER) RS::store(ip + r * 4 * kHeadDim, j, S[r]);
          if (j == 0) op[4 * r] = __float2bfloat16_rn(scale * fmaf(g, sq, delta * kq));
        }
      }
      ST* nsp =
          new_pool + ((size_t)slot * HV + h) * kHeadDim * kHeadDim + (size_t)row0 * kHeadDim;
#pragma unroll
      for (int r = 0; r < NG; ++r) RS::store(nsp + r * 4 * kHeadDim, j, S[r]);
    } else if (j == 0) {  // padding row: zero outputs, no state
      for (int t = 0; t < T; ++t)
#pragma unroll
        for (int r = 0; r < NG; ++r)
          op0[(size_t)t * HV * kHeadDim + 4 * r] = __float2bfloat16_rn(0.f);
    }
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(&empty[stage]);  // this warp is done with the stage
    if (issuer && issued < nmine) {  // refill it with item i + kStages once every warp is
      if (!mtp_wait(&empty[stage], (i / C::kStages) & 1, abort_flag, kMtpErrFreeTimeout)) break;
      issue(issued++);
    }
  }
  if (issuer && *abort_flag) {  // let copies still in flight land before the CTA exits
    for (int i = issued - C::kStages > 0 ? issued - C::kStages : 0; i < issued; ++i)
      sm100::mbar_wait(&full[i % C::kStages], (i / C::kStages) & 1, 1u << 20);
  }
}

template <bool L2, typename IdxT, typename ST>
cudaError_t launch_mtp_stream_t(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                const __nv_bfloat16* V, const ST* pool, const IdxT* I,
                                const float* A_log, const __nv_bfloat16* A,
                                const float* dt_bias, const __nv_bfloat16* Bt, float scale,
                                __nv_bfloat16* O, ST* new_pool, ST* inter, int T,
                                long long pool_size, int HQ, int HV, int items, int grid,
                                cudaStream_t st) {
  using C = MtpStreamCfg<ST>;
  auto kern = mtp_stream_kernel<L2, true, IdxT, ST>;
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  kern<<<grid, C::kThreads, C::kSmem, st>>>(Q, K, V, pool, I, A_log, A, dt_bias, Bt, scale, O,
                                             new_pool, inter, T, pool_size, HQ, HV, HV / HQ,
                                             items);
  return cudaGetLastError();
}

// Streaming variant for calls with the rollback buffer (see mtp_stream_kernel).
template <typename IdxT, typename ST>
cudaError_t launch_mtp_stream(const void* q, const void* k, const void* v, const ST* pool,
                              const void* indices, const float* A_log, const void* a,
                              const float* dt_bias, const void* b, float scale, void* out,
                              ST* new_pool, ST* inter, int batch, int T, long long pool_size,
                              int HQ, int HV, bool l2norm, cudaStream_t st) {
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (sms[dev] == 0 &&
      cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return cudaErrorInvalidValue;
  const int items = batch * HV;
  const int grid = items < sms[dev] ? items : sms[dev];
  auto Q = static_cast<const __nv_bfloat16*>(q);
  auto K = static_cast<const __nv_bfloat16*>(k);
  auto V = static_cast<const __nv_bfloat16*>(v);
  auto A = static_cast<const __nv_bfloat16*>(a);
  auto Bt = static_cast<const __nv_bfloat16*>(b);
  auto O = static_cast<__nv_bfloat16*>(out);
  auto I = static_cast<const IdxT*>(indices);
  return l2norm ? launch_mtp_stream_t<true, IdxT, ST>(Q, K, V, pool, I, A_log, A, dt_bias, Bt,
                                                     scale, O, new_pool, inter, T, pool_size,
                                                     HQ, HV, items, grid, st)
                : launch_mtp_stream_t<false, IdxT, ST>(Q, K, V, pool, I, A_log, A, dt_bias, Bt,
                                                      scale, O, new_pool, inter, T, pool_size,
                                                      HQ, HV, items, grid, st);
}

template <int RPW, typename IdxT, typename ST>
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
  mtp_kernel<RPW, L2, IN, IdxT, ST><<<grid, block, 0, st>>>(Q, K, V, pool, I, A_log, A, dt_bias, \
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
  // the streaming variant bulk-copies q, k and v rows: 16-byte aligned bases
  const bool rows16 = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                        reinterpret_cast<uintptr_t>(v)) & 15u) == 0;
  // same CTA sizing as the decode kernel: enough CTAs to fill 148 SMs several times;
  // with the rollback buffer (T + 1 state writes per read) and that many heads, the
  // streaming variant, whose reads run under the writes
  const long long heads = (long long)batch * HV;
  if (inter != nullptr && T >= 2 && T <= kMtpStreamMaxT && heads >= 4 * 148 && rows16)
    return launch_mtp_stream<IdxT, ST>(q, k, v, pool, indices, A_log, a, dt_bias, b, scale, out,
                                       new_pool, inter, batch, T, pool_size, HQ, HV, l2norm, st);
  if (heads >= 4 * 148)
    return launch_mtp_rpw<16, IdxT, ST>(q, k, v, pool, indices, A_log, a, dt_bias, b, scale, out,
                                    new_pool, inter, batch, T, pool_size, HQ, HV, l2norm, st);
  if (heads >= 2 * 148)
    return launch_mtp_rpw<8, IdxT, ST>(q, k, v, pool, indices, A_log, a, dt_bias, b, scale, out,
                                   new_pool, inter, batch, T, pool_size, HQ, HV, l2norm, st);
  return launch_mtp_rpw<4, IdxT, ST>(q, k, v, pool, indices, A_log, a, dt_bias, b, scale, out,
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

namespace gdn {
// Device error bits of the streaming multi-token decode kernel (bounded waits that ran out).
unsigned read_mtp_device_error(bool clear) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_mtp_device_error, sizeof(v)) != cudaSuccess) return ~0u;
  if (clear && v != 0) {
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_mtp_device_error, &zero, sizeof(zero)) != cudaSuccess) return ~0u;
  }
  return v;
}
}  // namespace gdn
