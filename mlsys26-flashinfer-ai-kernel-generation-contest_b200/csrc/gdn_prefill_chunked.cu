// GDN prefill, chunked WY/UT form on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces gdn_prefill_chunk_kernel (reference gdn_prefill/solution/triton/kernel.py:28-250)
// with a chunk of C = 64 tokens and the state in k-last layout S[v, k].
//
// Per chunk (tokens t = 0..C-1 of one sequence, one v-head; q/k rows of the
// GVA q/k head), with Lam_t the cumulative log decay inside the chunk and
// rk/rq the optional L2-norm factors (1 when off):
//
//   A[t,j] = beta_t exp(Lam_t - Lam_j) rk_t rk_j (k_t . k_j)      j < t
//   T      = (I + A)^-1                          (unit lower triangular, fp32)
//   T1     = T diag(beta gamma rk),  T2 = T diag(beta),  gamma_t = exp(Lam_t)
//   U      = T2 V - T1 (K S^T)                   (per-token corrected values)
//   O      = scale [ diag(gamma rq) Q S^T + P U ],  P[t,j] = exp(Lam_t-Lam_j) rq_t rk_j (q_t.k_j), j<=t
//   S     <- G S + U~^T K,  U~ = diag(rk exp(Lam_end - Lam_t)) U,  G = exp(Lam_end)
//
// which is the per-token recurrence of the definition reference
// (flashinfer/trace/templates/gdn.py:228-271) regrouped per chunk; the
// reference Triton kernel states the same algebra for 16-token chunks
// (gdn_prefill/solution/triton/kernel.py:60-79).  Every exponent above is <= 0
// (Lam is non-increasing), so nothing is clamped (the reference's clamp of
// log-gamma to [-88, 88], kernel.py:166, corrupts gamma ratios under strong decay).
//
// Precision: every MMA operand is bf16.  q, k, v are bf16 inputs (exact).  The
// fp32 quantities on the state path are split x = hi + lo (two bf16: hi the
// truncation, lo the rounded residual; integer ops, not cvt) and their
// products expanded, accumulated in fp32 in TMEM: S K^T -> 2 MMAs (S_hi, S_lo),
// T2 V -> 2, T1 (K S^T) -> 3 (hi.hi + lo.hi + hi.lo), U~^T K -> 2, so the fp32
// state keeps ~16 mantissa bits per step instead of bf16's 8.  Output terms
// use the hi parts, except P U for raw (un-normalised) q/k, which is split too.
//
// Orientation: the tensor-core D tiles are kept "v-major" (v = 128 TMEM lanes),
// so S (128 x 128), U^T, O^T and the state update are M = 128 MMAs.  Per chunk
// three MMA groups, each ended by one commit:
//   group 1 (needs only this chunk's tiles and S):
//     [Skk;Sqk] = [K;Q] K^T      M128 N64  K128   (A, B: TMA tiles, K-major)
//     (S K^T)   = S_hi K^T + S_lo K^T   M128 N64 K128
//     Oi        = S_hi Q^T              M128 N64 K128
//   group 2 (after the triangular inverse on the CUDA cores):
//     U^T = V^T T2^T - (S K^T) T1^T     M128 N64 K64  (A = V tile MN-major; negated A)
//   group 3:
//     dS  = U~^T K                      M128 N128 K64 (B = K tile MN-major)
//     Ot  = U^T P^T                     M128 N64 K64
// and O = scale (diag(gamma rq) Oi + Ot), S <- G S + dS on the CUDA cores.
// The next chunk's Q, V and K tiles are fetched as soon as the current ones
// are consumed (after groups 1, 2 and 3 respectively) and its gates are
// computed during group 2, so only the inverse and the MMA round trips remain
// on the serial path.
//
// One CTA (16 warps) owns one (sequence, v-head); warp w serves TMEM lanes
// 32*(w%4).. and column quarter w/4.  Thread 0 issues TMA and UMMA; completion is
// tracked by two mbarriers whose waits are bounded: a wait that runs out sets a
// device error flag (read by gdn_device_error) and the CTA releases TMEM and exits.
#include <cudaTypedefs.h>

#include "gdn_common.cuh"
#include "gdn_chunk_math.cuh"
#include "gdn_lpt.cuh"
#include "gdn_prefill.cuh"
#include "sm100.cuh"

namespace gdn {

__device__ unsigned int g_prefill_device_error = 0;

namespace {
using namespace sm100;
using namespace cm;

constexpr int kC = 64;          // chunk length
constexpr int kThreads = 512;   // 16 warps
constexpr int kLdA = 65;        // padded row stride of the fp32 A matrix (bank-conflict free)
constexpr int kLdT = 68;        // padded row stride of the fp32 T matrix (16-byte rows)

// ---- shared memory map (byte offsets from the 1024-byte aligned dynamic base) ----
constexpr uint32_t OFF_K0 = 0;        // K tile, d 0..63   [t][d]  (TMA, 128B swizzle)
constexpr uint32_t OFF_Q0 = 8192;     // Q tile, d 0..63
constexpr uint32_t OFF_K1 = 16384;    // K tile, d 64..127
constexpr uint32_t OFF_Q1 = 24576;    // Q tile, d 64..127
constexpr uint32_t OFF_V = 32768;     // V tile [t][v] 2 x 8 KB
constexpr uint32_t OFF_SHI = 49152;   // S hi [v][k] K-major, 2 k-blocks of 16 KB
constexpr uint32_t OFF_SLO = 81920;   // S lo
constexpr uint32_t OFF_SKHI = 114688; // (S K^T) hi [v][t] K-major 16 KB; then O staging [t][v]
constexpr uint32_t OFF_SKLO = 131072; // (S K^T) lo
constexpr uint32_t OFF_U = 147456;    // 64 KB, phase-dependent:
//   before group 2: Tmat f32[64][kLdT] @0, E scratch @17K, A f32[64][kLdA] @21K,
//                   then (A dead) T1hi @32K, T1lo @40K, T2hi @48K, T2lo @56K  [t][j] K-major
//   after group 2:  U~hi [v][t] @0, U~lo @16K, Uhi @32K, Ulo @48K (K-major A operands)
constexpr uint32_t OFF_P = 212992;    // P hi [t][j] K-major 8 KB
constexpr uint32_t OFF_PLO = 221184;  // P lo (raw q/k only)
constexpr uint32_t OFF_VEC = 229376;  // fp32[64] vectors + barriers
constexpr uint32_t VEC_BAR = 2304;    // 2 x (Lam, beta, gamma) + rk, rq, us = 9 x 256 B
constexpr uint32_t SMEM_ALLOC = OFF_VEC + VEC_BAR + 64;
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KB per-CTA shared memory limit");

constexpr uint32_t U_TMAT = 0, U_E = 17408, U_AMAT = 21504;
constexpr uint32_t U_T1HI = 32768, U_T1LO = 40960, U_T2HI = 49152, U_T2LO = 57344;
constexpr uint32_t U_UTHI = 0, U_UTLO = 16384, U_UHI = 32768, U_ULO = 49152;
constexpr uint32_t OFF_OST = OFF_SKHI;  // output staging, once group 2 has read S K^T

// TMEM columns (512 allocated, 448 used)
constexpr uint32_t TM_DS = 0;     // dS  128 lanes (v) x 128 (k)
constexpr uint32_t TM_UT = 128;   // U^T 128 (v) x 64 (t)
constexpr uint32_t TM_OT = 192;   // U^T P^T
constexpr uint32_t TM_OI = 256;   // S_hi Q^T
constexpr uint32_t TM_SK = 320;   // S K^T
constexpr uint32_t TM_KQ = 384;   // lanes 0..63: Skk rows, 64..127: Sqk rows; 64 cols
constexpr uint32_t TM_COLS = 512;

enum : unsigned { ERR_TMA_TIMEOUT = 1u, ERR_MMA_TIMEOUT = 2u, ERR_SMEM_ALIGN = 4u };

struct ChunkedParams {
  const __nv_bfloat16* a;
  const __nv_bfloat16* b;
  const float* A_log;
  const float* dt_bias;
  const void* cu;
  const float* state;
  float* new_state;
  __nv_bfloat16* out;
  const int* order;  // longest-first sequence order (may be null: natural order)
  long long a_rs, b_rs, o_rs;  // token strides of a, b and the output (elements)
  long long T;
  int cu64;
  int HV;
  int ratio;
  float scale;
  // precomputed gates (fp32 [T, HV] decay and beta, null = 1) instead of a / b
  // (pipelined kernel only)
  bool gates_pre;
  const float* g_alpha;
  const float* g_beta;
  // state checkpoints every ckpt_every tokens (0 = off; pipelined kernel only)
  float* ckpt;
  const long long* ckpt_starts;
  long long ckpt_cap;
  int ckpt_every;
};

// All threads wait on `bar`; returns false on every thread if any thread timed out.
__device__ __forceinline__ bool cta_wait(uint64_t* bar, uint32_t parity, unsigned code) {
  const bool ok = mbar_wait(bar, parity);
  const int bad = __syncthreads_or(ok ? 0 : 1);
  if (bad && threadIdx.x == 0) atomicOr(&g_prefill_device_error, code);
  return bad == 0;
}

// T = (I + A)^-1 for a strictly lower triangular fp32 A[64][kLdA] (row stride kLdA),
// written to Tm[64][kLdT].  Eight 8x8 diagonal blocks by forward substitution (one
// column per thread, the block's A entries held in registers), then three levels of
// block merges, each two small products:
//   [[L11, 0], [L21, L22]]^-1 = [[T11, 0], [-T22 (L21 T11), T22]].
// The padded strides keep the shared-memory access patterns conflict-free.
// Called by all kThreads (= 512) threads (contains __syncthreads).
__device__ __forceinline__ void invert_unit_lower64(const float* __restrict__ A,
                                                    float* __restrict__ Tm,
                                                    float* __restrict__ E) {
  const int tid = threadIdx.x;
  // ---- level 1: 8x8 diagonal blocks ----
  if (tid < 64) {
    const int o = 8 * (tid >> 3), col = tid & 7;
    float a[8][8];
#pragma unroll
    for (int r = 1; r < 8; ++r)
#pragma unroll
      for (int j = 0; j < r; ++j) a[r][j] = A[(o + r) * kLdA + o + j];
    float x[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < r; ++j) acc = fmaf(a[r][j], x[j], acc);
      x[r] = (r < col) ? 0.f : ((r == col) ? 1.f : -acc);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) Tm[(o + r) * kLdT + o + col] = x[r];
  } else {
    // zero everything above the 8x8 block diagonal
    for (int u = tid - 64; u < 64 * 64; u += kThreads - 64) {
      const int r = u >> 6, c = u & 63;
      if (c >= 8 * ((r >> 3) + 1)) Tm[r * kLdT + c] = 0.f;
    }
  }
  __syncthreads();
  // ---- level 2 (8 -> 16): pairs p = 0..3, rows bi = 16p + 8, cols bj = 16p ----
  {
    const int p = (tid >> 6) & 3, r = (tid >> 3) & 7, c = tid & 7;
    const int bi = 16 * p + 8, bj = 16 * p;
    if (tid < 256) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        acc = fmaf(A[(bi + r) * kLdA + bj + k], Tm[(bj + k) * kLdT + bj + c], acc);
      E[p * 64 + r * 8 + c] = acc;
    }
    __syncthreads();
    if (tid < 256) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) acc = fmaf(Tm[(bi + r) * kLdT + bi + k], E[p * 64 + k * 8 + c], acc);
      Tm[(bi + r) * kLdT + bj + c] = -acc;
    }
  }
  __syncthreads();
  // ---- level 3 (16 -> 32): pairs p = 0..1, rows bi = 32p + 16, cols bj = 32p ----
  {
    const int p = tid >> 8, r = (tid >> 4) & 15, c = tid & 15;
    const int bi = 32 * p + 16, bj = 32 * p;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k)
      acc = fmaf(A[(bi + r) * kLdA + bj + k], Tm[(bj + k) * kLdT + bj + c], acc);
    E[p * 256 + r * 16 + c] = acc;
    __syncthreads();
    acc = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) acc = fmaf(Tm[(bi + r) * kLdT + bi + k], E[p * 256 + k * 16 + c], acc);
    Tm[(bi + r) * kLdT + bj + c] = -acc;
  }
  __syncthreads();
  // ---- level 4 (32 -> 64): rows 32..63 x cols 0..31, 1x2 outputs per thread ----
  {
    const int r = tid >> 4, c = 2 * (tid & 15);
    float e0 = 0.f, e1 = 0.f;
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      const float a0 = A[(32 + r) * kLdA + k];
      const float2 t = *reinterpret_cast<const float2*>(Tm + k * kLdT + c);
      e0 = fmaf(a0, t.x, e0);
      e1 = fmaf(a0, t.y, e1);
    }
    *reinterpret_cast<float2*>(E + r * 32 + c) = make_float2(e0, e1);
    __syncthreads();
    e0 = e1 = 0.f;
#pragma unroll 2
    for (int k = 0; k < 32; k += 4) {
      const float4 a4 = *reinterpret_cast<const float4*>(Tm + (32 + r) * kLdT + 32 + k);
      const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float2 t = *reinterpret_cast<const float2*>(E + (k + kk) * 32 + c);
        e0 = fmaf(av[kk], t.x, e0);
        e1 = fmaf(av[kk], t.y, e1);
      }
    }
    *reinterpret_cast<float2*>(Tm + (32 + r) * kLdT + c) = make_float2(-e0, -e1);
  }
  __syncthreads();
}

template <bool L2NORM, bool HAS_STATE, typename CuT>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_chunked_kernel(const __grid_constant__ CUtensorMap tm_q,
                           const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const ChunkedParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sb = smem_u32(smem);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int sp = warp & 3, qtr = warp >> 2;  // TMEM subpartition, column quarter
  const int row = sp * 32 + lane;  // TMEM lane owned by this thread
  const int HV = p.HV;
  const int wi = blockIdx.x / HV;  // work item: the wi-th longest sequence
  const int h = blockIdx.x - wi * HV;
  const int n = p.order ? p.order[wi] : wi;
  const int qh = h / p.ratio;
  const CuT* cu = static_cast<const CuT*>(p.cu);
  const long long s1 = min(max((long long)cu[n + 1], 0LL), p.T);
  const long long s0 = min(max((long long)cu[n], 0LL), s1);
  const long long L = s1 - s0;
  float* nsrow = p.new_state + (((size_t)n * HV + h) * kHeadDim + row) * kHeadDim + 32 * qtr;

  if (L <= 0) {  // empty sequence: zero final state (definition semantics)
#pragma unroll
    for (int i = 0; i < 8; ++i) st_stream_f4(nsrow + 4 * i, make_float4(0.f, 0.f, 0.f, 0.f));
    return;
  }
  if ((sb & 1023u) != 0) {  // the swizzled layouts need a 1024-byte aligned base
    if (tid == 0) atomicOr(&g_prefill_device_error, ERR_SMEM_ALIGN);
    return;
  }

  // gate vectors are double-buffered: chunk c uses set (c & 1) while set (c + 1) & 1
  // is filled for the next chunk
  float* vec = reinterpret_cast<float*>(smem + OFF_VEC);
  float* Lam = vec;         // cumulative log decay within the chunk
  float* beta = vec + 64;
  float* gam = vec + 128;   // exp(Lam)
  float* rk = vec + 384;
  float* rq = vec + 448;
  float* us = vec + 512;    // rk exp(Lam_end - Lam)
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(smem + OFF_VEC + VEC_BAR);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_VEC + VEC_BAR + 16);
  float* Amat = reinterpret_cast<float*>(smem + OFF_U + U_AMAT);
  float* Tmat = reinterpret_cast<float*>(smem + OFF_U + U_TMAT);
  float* Escr = reinterpret_cast<float*>(smem + OFF_U + U_E);

  if (warp == 0) {
    tmem_alloc(tmem_slot, TM_COLS);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(bar_tma, 3);  // three arrivals per chunk: the Q, V and K tiles
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tl = tmem + ((uint32_t)(32 * sp) << 16);  // this warp's lane base

  // ---- initial state: this thread keeps S[v=row][32*qtr .. +32) in fp32 registers ----
  float s[32];
  if constexpr (HAS_STATE) {
    const float* srow = p.state + (((size_t)n * HV + h) * kHeadDim + row) * kHeadDim + 32 * qtr;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v4 = ld_stream_f4(srow + 4 * i);
      s[4 * i] = v4.x; s[4 * i + 1] = v4.y; s[4 * i + 2] = v4.z; s[4 * i + 3] = v4.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) s[i] = 0.f;
  }
  // S hi / lo -> shared (K-major [v][k]: k-block qtr/2, 16-byte chunks 4*(qtr&1)..+3)
  auto write_state_split = [&]() {
    const uint32_t kb = 16384u * (qtr >> 1), c0 = 4u * (qtr & 1);
    const uint32_t bhi = sb + OFF_SHI + kb, blo = sb + OFF_SLO + kb;
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      uint4 hi, lo;
      split8(&s[8 * q4], hi, lo);
      st_v4(bhi + sw128(row, c0 + q4), hi);
      st_v4(blo + sw128(row, c0 + q4), lo);
    }
  };
  write_state_split();

  const float nexpA = -expf(__ldg(p.A_log + h));
  const float dtb = __ldg(p.dt_bias + h);
  const float scale = default_scale(p.scale);
  const int nchunks = (int)((L + kC - 1) / kC);
  uint32_t ph_tma = 0, ph_mma = 0;
  bool ok = true;
  bool mma_pending = false, tma_pending = false;

  // Gates, by one warp (two tokens per lane): the raw a/b values of chunk cc are
  // loaded one chunk ahead (load_gates) and turned into log decay, its inclusive
  // prefix sum Lam, exp(Lam) and beta in vector set `buf` (finish_gates).
  // Padding tokens get decay 1 and beta 0.
  float ga[2] = {0.f, 0.f}, gb[2] = {0.f, 0.f};
  auto load_gates = [&](int cc) {
    const long long tc0 = s0 + (long long)kC * cc;
    const int Lcc = (int)min((long long)kC, s1 - tc0);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = 2 * lane + e;
      if (t < Lcc) {
        ga[e] = bf2f(p.a[(size_t)(tc0 + t) * p.a_rs + h]);
        gb[e] = bf2f(p.b[(size_t)(tc0 + t) * p.b_rs + h]);
      }
    }
  };
  auto finish_gates = [&](int cc, int buf) {
    const long long tc0 = s0 + (long long)kC * cc;
    const int Lcc = (int)min((long long)kC, s1 - tc0);
    float* Lm = vec + 192 * buf;
    float lg[2], bb[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const bool valid = 2 * lane + e < Lcc;
      lg[e] = valid ? nexpA * softplus_f(ga[e] + dtb) : 0.f;
      bb[e] = valid ? sigmoid_f(gb[e]) : 0.f;
    }
    float x = lg[0] + lg[1];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    const float x0 = x - lg[1];
    Lm[2 * lane] = x0;
    Lm[2 * lane + 1] = x;
    Lm[64 + 2 * lane] = bb[0];
    Lm[64 + 2 * lane + 1] = bb[1];
    Lm[128 + 2 * lane] = expf(x0);
    Lm[128 + 2 * lane + 1] = expf(x);
  };
  // TMA of chunk cc, one arrival each: the Q tile, the V tile, the K tile
  auto issue_tiles = [&](int cc, uint32_t off0, uint32_t off1, const CUtensorMap* m, int head) {
    const int y = (int)(s0 + (long long)kC * cc);
    fence_proxy_async();
    mbar_arrive_expect_tx(bar_tma, 2 * 8192);
    tma_load_2d(smem + off0, m, bar_tma, head * 128, y);
    tma_load_2d(smem + off1, m, bar_tma, head * 128 + 64, y);
  };
  if (tid == 0) {
    issue_tiles(0, OFF_Q0, OFF_Q1, &tm_q, qh);
    issue_tiles(0, OFF_V, OFF_V + 8192, &tm_v, h);
    issue_tiles(0, OFF_K0, OFF_K1, &tm_k, qh);
  }
  tma_pending = true;
  if (warp == 1) {
    load_gates(0);
    finish_gates(0, 0);
  }

  for (int c = 0; c < nchunks; ++c) {
    const long long t0 = s0 + (long long)kC * c;
    const int Lc = (int)min((long long)kC, s1 - t0);
    const bool more = c + 1 < nchunks;
    Lam = vec + 192 * (c & 1);
    beta = Lam + 64;
    gam = Lam + 128;

    // (1) wait for this chunk's K, Q and V tiles (issued during the previous chunk)
    fence_proxy_async();
    __syncthreads();
    if (!cta_wait(bar_tma, ph_tma, ERR_TMA_TIMEOUT)) { ok = false; break; }
    ph_tma ^= 1;
    tma_pending = false;
    if (warp == 1 && more) load_gates(c + 1);  // consumed during group 2

    // (2) MMA group 1: [Skk;Sqk] = [K;Q] K^T,  S K^T (hi + lo),  Oi = S_hi Q^T
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = umma_idesc_bf16(128, 64, false, false);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t off = 16384u * (ks >> 2) + 32u * (ks & 3);
        const uint64_t kdesc = umma_desc_k(sb + OFF_K0 + off);
        umma_bf16(tmem + TM_KQ, kdesc, kdesc, idesc, ks > 0);
        umma_bf16(tmem + TM_SK, umma_desc_k(sb + OFF_SHI + off), kdesc, idesc, ks > 0);
        umma_bf16(tmem + TM_SK, umma_desc_k(sb + OFF_SLO + off), kdesc, idesc, 1);
        umma_bf16(tmem + TM_OI, umma_desc_k(sb + OFF_SHI + off),
                  umma_desc_k(sb + ((ks >> 2) ? OFF_Q1 : OFF_Q0) + 32u * (ks & 3)), idesc, ks > 0);
      }
      umma_commit(bar_mma);
    }
    mma_pending = true;
    // meanwhile: q/k L2-norm factors
    if constexpr (L2NORM) {
      if (tid >= 256 && tid < 384) {
        const int t = tid & 63;
        const bool isq = tid < 320;
        const uint32_t b0 = sb + (isq ? OFF_Q0 : OFF_K0) + 128u * t;
        float ss = 0.f;
#pragma unroll
        for (int blk = 0; blk < 2; ++blk)
#pragma unroll
          for (int ci = 0; ci < 8; ++ci) {
            const int ch = (ci + t) & 7;  // rotate: rows t..t+7 hit distinct bank groups
            const uint4 u = ld_shared_v4(b0 + 16384u * blk + 16u * ch);
            const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = bf2x2_to_f2(w4[e]);
              ss = fmaf(f.x, f.x, ss);
              ss = fmaf(f.y, f.y, ss);
            }
          }
        const float r = rsqrtf(ss + kL2NormEps);
        if (isq) rq[t] = r; else rk[t] = r;
      }
    } else {
      if (tid < 64) { rk[tid] = 1.f; rq[tid] = 1.f; }
    }
    if (!cta_wait(bar_mma, ph_mma, ERR_MMA_TIMEOUT)) { ok = false; break; }
    ph_mma ^= 1;
    mma_pending = false;
    tc_fence_after();
    if (more) {  // the Q tile is consumed: fetch the next one
      if (tid == 0) issue_tiles(c + 1, OFF_Q0, OFF_Q1, &tm_q, qh);
      tma_pending = true;
    }

    // (3) A (from Skk) -> Amat;  P (from Sqk) -> bf16 [t][j] (hi, and lo for raw q/k);
    //     S K^T -> hi/lo K-major [v][t]
    {
      float kq[16];
      tmem_ld16(tl + TM_KQ + 16u * qtr, kq);
      float sk[16];
      tmem_ld16(tl + TM_SK + 16u * qtr, sk);
      // all shared-memory operands first (the stores below would otherwise order
      // every later load behind them)
      const int t = row & 63;
      const bool is_k = row < 64;
      const float lt = Lam[t];
      const float ft = is_k ? beta[t] * rk[t] : rq[t];
      float lv[16], rv[16];
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 lj = *reinterpret_cast<const float4*>(Lam + 16 * qtr + i);
        const float4 rj = *reinterpret_cast<const float4*>(rk + 16 * qtr + i);
        lv[i] = lj.x; lv[i + 1] = lj.y; lv[i + 2] = lj.z; lv[i + 3] = lj.w;
        rv[i] = rj.x; rv[i + 1] = rj.y; rv[i + 2] = rj.z; rv[i + 3] = rj.w;
      }
      tmem_wait_ld();
      float ej[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = 16 * qtr + i;
        // A: strictly lower (j < t); P: lower incl. diagonal (j <= t)
        const bool keep = is_k ? (j < t) : (j <= t);
        ej[i] = keep ? ft * rv[i] * kq[i] * __expf(lt - lv[i]) : 0.f;
      }
      if (is_k) {
#pragma unroll
        for (int i = 0; i < 16; ++i) Amat[t * kLdA + 16 * qtr + i] = ej[i];
      } else {
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          uint4 hi, lo;
          split8(&ej[8 * q2], hi, lo);
          st_v4(sb + OFF_P + sw128(t, 2 * qtr + q2), hi);
          if constexpr (!L2NORM) st_v4(sb + OFF_PLO + sw128(t, 2 * qtr + q2), lo);
        }
      }
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        uint4 hi, lo;
        split8(&sk[8 * q2], hi, lo);
        st_v4(sb + OFF_SKHI + sw128(row, 2 * qtr + q2), hi);
        st_v4(sb + OFF_SKLO + sw128(row, 2 * qtr + q2), lo);
      }
    }
    __syncthreads();

    // (4) T = (I + A)^-1;  T1 = T diag(beta gamma rk), T2 = T diag(beta) -> hi/lo bf16
    invert_unit_lower64(Amat, Tmat, Escr);
    {
      // thread -> 16-byte column chunk cidx of row t
      const int cidx = tid & 7, t = tid >> 3;
      float cb[8], cg[8], tv[8];
      const float* tr = Tmat + t * kLdT + 8 * cidx;
      const float4 ta = *reinterpret_cast<const float4*>(tr);
      const float4 tb = *reinterpret_cast<const float4*>(tr + 4);
      tv[0] = ta.x; tv[1] = ta.y; tv[2] = ta.z; tv[3] = ta.w;
      tv[4] = tb.x; tv[5] = tb.y; tv[6] = tb.z; tv[7] = tb.w;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = 8 * cidx + e;
        cb[e] = beta[j];
        cg[e] = beta[j] * gam[j] * rk[j];
      }
      float w1[8], w2[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        w1[e] = tv[e] * cg[e];
        w2[e] = tv[e] * cb[e];
      }
      uint4 hi, lo;
      split8(w1, hi, lo);
      st_v4(sb + OFF_U + U_T1HI + sw128(t, cidx), hi);
      st_v4(sb + OFF_U + U_T1LO + sw128(t, cidx), lo);
      split8(w2, hi, lo);
      st_v4(sb + OFF_U + U_T2HI + sw128(t, cidx), hi);
      st_v4(sb + OFF_U + U_T2LO + sw128(t, cidx), lo);
    }
    if (tid < 64) us[tid] = (tid < Lc) ? rk[tid] * expf(Lam[63] - Lam[tid]) : 0.f;
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();

    // (5) MMA group 2: U^T = V^T T2^T - (S K^T) T1^T
    if (tid == 0) {
      tc_fence_after();
      const uint32_t id_v = umma_idesc_bf16(128, 64, true, false);
      const uint32_t id_x = umma_idesc_bf16(128, 64, false, false, true);
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        const uint32_t t2 = sb + OFF_U + (part ? U_T2LO : U_T2HI);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tmem + TM_UT, umma_desc_mn(sb + OFF_V + 2048u * ks, 8192),
                    umma_desc_k(t2 + 32u * ks), id_v, (part | ks) != 0);
      }
#pragma unroll
      for (int term = 0; term < 3; ++term) {  // (SK_hi,T1_hi) (SK_lo,T1_hi) (SK_hi,T1_lo)
        const uint32_t a = sb + (term == 1 ? OFF_SKLO : OFF_SKHI);
        const uint32_t b = sb + OFF_U + (term == 2 ? U_T1LO : U_T1HI);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tmem + TM_UT, umma_desc_k(a + 32u * ks), umma_desc_k(b + 32u * ks), id_x, 1);
      }
      umma_commit(bar_mma);
    }
    mma_pending = true;
    if (warp == 1 && more) finish_gates(c + 1, (c + 1) & 1);
    if (!cta_wait(bar_mma, ph_mma, ERR_MMA_TIMEOUT)) { ok = false; break; }
    ph_mma ^= 1;
    mma_pending = false;
    tc_fence_after();
    if (more) {  // the V tile is consumed
      if (tid == 0) issue_tiles(c + 1, OFF_V, OFF_V + 8192, &tm_v, h);
      tma_pending = true;
    }

    // (6) U -> U~ = diag(us) U (hi/lo) and U hi (lo), K-major [v][t]
    {
      float uv[16], uw[16];
      tmem_ld16(tl + TM_UT + 16u * qtr, uv);
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 w4 = *reinterpret_cast<const float4*>(us + 16 * qtr + i);
        uw[i] = w4.x; uw[i + 1] = w4.y; uw[i + 2] = w4.z; uw[i + 3] = w4.w;
      }
      tmem_wait_ld();
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        float x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = uv[8 * q2 + e] * uw[8 * q2 + e];
        uint4 hi, lo;
        split8(x, hi, lo);
        const uint32_t o = sw128(row, 2 * qtr + q2);
        st_v4(sb + OFF_U + U_UTHI + o, hi);
        st_v4(sb + OFF_U + U_UTLO + o, lo);
        split8(&uv[8 * q2], hi, lo);
        st_v4(sb + OFF_U + U_UHI + o, hi);
        if constexpr (!L2NORM) st_v4(sb + OFF_U + U_ULO + o, lo);
      }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();

    // (7) MMA group 3: dS = U~^T K (hi + lo);  Ot = U^T P^T
    if (tid == 0) {
      tc_fence_after();
      const uint32_t id_s = umma_idesc_bf16(128, 128, false, true);
#pragma unroll
      for (int part = 0; part < 2; ++part)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tmem + TM_DS,
                    umma_desc_k(sb + OFF_U + (part ? U_UTLO : U_UTHI) + 32u * ks),
                    umma_desc_mn(sb + OFF_K0 + 2048u * ks, 16384), id_s, (part | ks) != 0);
      const uint32_t id_p = umma_idesc_bf16(128, 64, false, false);
      constexpr int kPTerms = L2NORM ? 1 : 3;  // (U_hi, P_hi) [, (U_lo, P_hi), (U_hi, P_lo)]
#pragma unroll
      for (int term = 0; term < kPTerms; ++term) {
        const uint32_t ua = sb + OFF_U + (term == 1 ? U_ULO : U_UHI);
        const uint32_t pb = sb + (term == 2 ? OFF_PLO : OFF_P);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tmem + TM_OT, umma_desc_k(ua + 32u * ks), umma_desc_k(pb + 32u * ks), id_p,
                    (term | ks) != 0);
      }
      umma_commit(bar_mma);
    }
    mma_pending = true;
    if (!cta_wait(bar_mma, ph_mma, ERR_MMA_TIMEOUT)) { ok = false; break; }
    ph_mma ^= 1;
    mma_pending = false;
    tc_fence_after();
    if (more && tid == 0) issue_tiles(c + 1, OFF_K0, OFF_K1, &tm_k, qh);  // K consumed

    // (8) S <- G S + dS ;  O = scale (diag(gamma rq) Oi + Ot) -> staging [t][v] ; S hi/lo
    {
      const float G = expf(Lam[63]);
      float dv[32];
      tmem_ld32(tl + TM_DS + 32u * qtr, dv);
      float oi[16], ot[16], fo[16];
      tmem_ld16(tl + TM_OI + 16u * qtr, oi);
      tmem_ld16(tl + TM_OT + 16u * qtr, ot);
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 g4 = *reinterpret_cast<const float4*>(gam + 16 * qtr + i);
        const float4 q4 = *reinterpret_cast<const float4*>(rq + 16 * qtr + i);
        fo[i] = g4.x * q4.x; fo[i + 1] = g4.y * q4.y; fo[i + 2] = g4.z * q4.z; fo[i + 3] = g4.w * q4.w;
      }
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) s[i] = fmaf(G, s[i], dv[i]);
      uint16_t* ostage = reinterpret_cast<uint16_t*>(smem + OFF_OST);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        ostage[(16 * qtr + i) * kHeadDim + row] = (uint16_t)(
            rn_bf16_bits(__float_as_uint(scale * fmaf(fo[i], oi[i], ot[i]))) >> 16);
      if (more) write_state_split();
    }
    tc_fence_before();
    __syncthreads();
    // coalesced output rows (t < Lc): 16 x 16-byte pieces per 256-byte row
    {
      __nv_bfloat16* obase = p.out + (size_t)t0 * p.o_rs + (size_t)h * kHeadDim;
      constexpr int kUnits = 64 * 16 / kThreads;  // 16-byte pieces per thread
      uint4 v4[kUnits];
#pragma unroll
      for (int k4 = 0; k4 < kUnits; ++k4) {
        const int u = tid + kThreads * k4;
        v4[k4] = ld_shared_v4(sb + OFF_OST + 256u * (u >> 4) + 16u * (u & 15));
      }
#pragma unroll
      for (int k4 = 0; k4 < kUnits; ++k4) {
        const int u = tid + kThreads * k4, t = u >> 4;
        if (t < Lc)
          *reinterpret_cast<uint4*>(obase + (size_t)t * p.o_rs + 8 * (u & 15)) = v4[k4];
      }
    }
  }

  if (ok) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      st_stream_f4(nsrow + 4 * i, make_float4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]));
  } else {
    // a wait ran out: give in-flight copies / MMAs one more bounded chance to land
    if (tma_pending) mbar_wait(bar_tma, ph_tma);
    if (mma_pending) mbar_wait(bar_mma, ph_mma);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TM_COLS);
}

// ---------------------------------------------------------------- pipelined kernel
// Warp-specialised variant for L2-normalised q/k.  The chunk's work splits into
//   prep  (depends only on the chunk's own q/k/gates): KQ MMA, A and P, the 64x64
//         inverse, T hi/lo, Q~ = diag(gamma rq) Q, the vectors;
//   state (depends on S): S K^T and S_hi Q~^T MMAs, R = diag(beta)(V - diag(gamma rk) K S^T),
//         U^T = R^T T^T, U~ and the state update dS = U~^T K, O += U^T P^T.
// Warps 8..15 ("prep group") run chunk c+1's prep while warps 0..7 ("state group")
// run chunk c's state work; they hand over through mbarriers (prep -> state: T(c)
// ready; state -> prep: T consumed; the state group also refills a K/Q buffer as
// soon as it has finished the chunk that used it).  S is kept in TMEM: fp32 as the
// accumulator of the state update (pre-scaled by the chunk decay), and as bf16
// hi/lo pairs that are the A operand of the S K^T and S Q~^T MMAs, so no shared
// memory holds the state.  U = T R is the "right-hand side" form of the same
// algebra: T is split hi/lo once, and R (fp32) is split hi/lo by the state group.
namespace pl {
constexpr int kThreads = 512;
constexpr uint32_t kGroup = 256;        // threads per warp group
constexpr uint32_t kBarState = 1, kBarPrep = 2, kBarGates = 3;
// shared memory
constexpr uint32_t KQ0 = 0, KQ1 = 32768;  // per buffer: K0 | Q0 | K1 | Q1 (8 KB each)
constexpr uint32_t V = 65536;             // V0 | V1
constexpr uint32_t RHI = 81920, RLO = 98304;  // R^T hi/lo [v][j]; RHI also stages the output
constexpr uint32_t UTHI = 114688, UTLO = 131072, UHI = 147456;
constexpr uint32_t THI = 163840, TLO = 172032;  // T hi/lo [t][j]
constexpr uint32_t P0 = 180224, P1 = 188416;    // P hi [t][j], one per chunk parity
constexpr uint32_t AT = 196608;                 // fp32 [64][kLd], A then T in place
constexpr uint32_t E = 214016;                  // fp32 scratch of the block merges (32 x 36)
constexpr uint32_t VEC = 218624;                // per chunk mod 3: Lam beta gam rk rq us (6 x 64 f32)
constexpr uint32_t BARS = VEC + 3 * 6 * 256;
// decay factors exp(Lam_t - Lam_j) of one chunk, built by the prep group before A and P:
constexpr uint32_t DEF = BARS + 256;            // fp32 [4][16][kLdDE]: inside the diagonal 16x16 blocks
constexpr uint32_t ROWF = DEF + 4 * 16 * 20 * 4;  // fp32 [4][64]: exp(Lam_t - Lam_{16b+15}), b < t/16
constexpr uint32_t COLF = ROWF + 4 * 64 * 4;    // fp32 [64]:    exp(Lam_{j|15} - Lam_j)
constexpr uint32_t SMEM = COLF + 64 * 4;
constexpr int kLdDE = 20;  // row stride of DEF (floats): conflict-free float4 rows
static_assert(SMEM <= 232448, "shared memory budget");
// TMEM columns
constexpr uint32_t TS = 0, TSH = 128, TSL = 192, TUT = 256, TSK = 320, TO = 384, TKQ = 448;

struct Bars {
  uint64_t kqtma[2], vtma, kq, g1, g2, g3, t_ready, t_free;
};

// bounded wait by every thread of a group; false on all of them if any ran out or
// the other group has given up
__device__ __forceinline__ bool group_wait(uint64_t* bar, uint32_t parity, uint32_t gid,
                                           volatile int* abort_flag, unsigned code) {
  bool ok = false;
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (mbar_try_wait(bar, parity)) { ok = true; break; }
    if ((i & 1023u) == 1023u && *abort_flag) break;
  }
  const bool bad = group_or(gid, kGroup, !ok);
  if (bad && (threadIdx.x & (kGroup - 1)) == 0) {
    atomicOr(&g_prefill_device_error, code);
    *abort_flag = 1;
  }
  return !bad;
}

}  // namespace pl

template <bool HAS_STATE, typename CuT>
__global__ void __launch_bounds__(pl::kThreads, 1)
    prefill_pipelined_kernel(const __grid_constant__ CUtensorMap tm_q,
                             const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v, const ChunkedParams p) {
  using namespace pl;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sb = smem_u32(smem);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const bool prep = warp >= 8;
  const int u = tid & (kGroup - 1);          // index within the group
  const int sp = warp & 3, half = (warp >> 2) & 1;
  const int row = sp * 32 + lane;            // TMEM lane of this thread
  const int HV = p.HV;
  const int wi = blockIdx.x / HV;
  const int h = blockIdx.x - wi * HV;
  const int n = p.order ? p.order[wi] : wi;
  const int qh = h / p.ratio;
  const CuT* cu = static_cast<const CuT*>(p.cu);
  const long long s1 = min(max((long long)cu[n + 1], 0LL), p.T);
  const long long s0 = min(max((long long)cu[n], 0LL), s1);
  const long long L = s1 - s0;
  float* nsbase = p.new_state + ((size_t)n * HV + h) * kHeadDim * kHeadDim;

  if (L <= 0) {  // empty sequence: zero final state (definition semantics)
    for (int i = tid; i < kHeadDim * kHeadDim / 4; i += pl::kThreads)
      st_stream_f4(nsbase + 4 * i, make_float4(0.f, 0.f, 0.f, 0.f));
    return;
  }
  if ((sb & 1023u) != 0) {
    if (tid == 0) atomicOr(&g_prefill_device_error, ERR_SMEM_ALIGN);
    return;
  }
  Bars* bars = reinterpret_cast<Bars*>(smem + BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + BARS + sizeof(Bars));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + BARS + sizeof(Bars) + 4);
  // vector set of chunk c is c % 3: the gates of chunk c + 1 are written while the state
  // group still reads the set of chunk c - 1
  auto vecp = [&](int set, int which) {  // which: 0 Lam 1 beta 2 gam 3 rk 4 rq 5 us
    return reinterpret_cast<float*>(smem + VEC + 1536u * set + 256u * which);
  };

  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (tid == 32) {
    uint64_t* b = reinterpret_cast<uint64_t*>(bars);
    for (int i = 0; i < (int)(sizeof(Bars) / 8); ++i) mbar_init(b + i, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tl = tmem + ((uint32_t)(32 * sp) << 16);
  const int nchunks = (int)((L + kC - 1) / kC);
  const float nexpA = p.gates_pre ? 0.f : -expf(__ldg(p.A_log + h));
  const float dtb = p.gates_pre ? 0.f : __ldg(p.dt_bias + h);
  bool ok = true;
  // async work issued but not yet waited for (drained, boundedly, if a wait runs out)
  uint64_t* pend_bar[2] = {nullptr, nullptr};
  uint32_t pend_par[2] = {0, 0};
  // K and Q tiles of chunk cc into buffer cc & 1 (one arrival on kqtma[cc & 1]).  Chunks 0
  // and 1 are fetched here; chunk c + 2 by the state group as soon as it has finished
  // chunk c, i.e. as soon as that buffer (and the P / vector set of that parity) is free.
  auto issue_kq = [&](int cc) {
    const int bpar = cc & 1;
    const uint32_t dst = bpar ? KQ1 : KQ0;
    const int y = (int)(s0 + (long long)kC * cc);
    fence_proxy_async();
    mbar_arrive_expect_tx(&bars->kqtma[bpar], 4 * 8192);
    tma_load_2d(smem + dst, &tm_k, &bars->kqtma[bpar], qh * 128, y);
    tma_load_2d(smem + dst + 16384, &tm_k, &bars->kqtma[bpar], qh * 128 + 64, y);
    tma_load_2d(smem + dst + 8192, &tm_q, &bars->kqtma[bpar], qh * 128, y);
    tma_load_2d(smem + dst + 24576, &tm_q, &bars->kqtma[bpar], qh * 128 + 64, y);
  };
  if (tid == 0) {
    issue_kq(0);
    if (nchunks > 1) issue_kq(1);
  }

  if (prep) {
    // =========================== prep group: chunk c one ahead of the state group
    // raw bf16 bits, converted where they are used one chunk later (so that nothing
    // waits for these loads while the current chunk is processed)
    // Gates: warps 14 and 15, one token per lane (gt = token; -1.. for the other warps).
    // Raw bits are loaded one chunk ahead and converted where they are used.
    const int gt = u - 192;
    uint32_t ga = 0u, gb = 0u;
    auto load_gates = [&](int cc) {
      const long long tc0 = s0 + (long long)kC * cc;
      const int Lcc = (int)min((long long)kC, s1 - tc0);
      const unsigned short* ra = reinterpret_cast<const unsigned short*>(p.a);
      const unsigned short* rb = reinterpret_cast<const unsigned short*>(p.b);
      // unconditional loads (tokens past the end re-read the last one; compute_gates
      // masks them), so that nothing waits for the values before they are used
      const size_t tok = (size_t)(tc0 + min(gt, Lcc - 1));
      if (p.gates_pre) {  // fp32 bits of the precomputed decay and beta (dense [T, HV])
        const size_t ti = tok * HV + h;
        ga = p.g_alpha ? __float_as_uint(p.g_alpha[ti]) : 0x3F800000u;
        gb = p.g_beta ? __float_as_uint(p.g_beta[ti]) : 0x3F800000u;
      } else {            // bf16 bits of a and b
        ga = ra[tok * p.a_rs + h];
        gb = rb[tok * p.b_rs + h];
      }
    };
    // log decays (inclusive cumsum), beta and gamma of chunk cc into its vector set
    auto compute_gates = [&](int cc) {
      const long long tc0 = s0 + (long long)kC * cc;
      const int Lcc = (int)min((long long)kC, s1 - tc0);
      float* Lam = vecp(cc % 3, 0);
      float* beta = vecp(cc % 3, 1);
      float* gam = vecp(cc % 3, 2);
      const bool valid = gt < Lcc;
      float lg, bb;
      if (p.gates_pre) {
        lg = valid ? log_alpha(__uint_as_float(ga)) : 0.f;
        bb = valid ? __uint_as_float(gb) : 0.f;
      } else {
        lg = valid ? nexpA * softplus_f(__uint_as_float(ga << 16) + dtb) : 0.f;
        bb = valid ? sigmoid_f(__uint_as_float(gb << 16)) : 0.f;
      }
      float x = lg;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
      }
      if (gt < 32) Lam[gt] = x;
      group_sync(kBarGates, 64);  // warp 15 continues from warp 14's last sum
      if (gt >= 32) {
        x += Lam[31];
        Lam[gt] = x;
      }
      beta[gt] = bb;
      gam[gt] = expf(x);
    };
    if (gt >= 0) {
      load_gates(0);
      compute_gates(0);
      if (nchunks > 1) load_gates(1);
    }
    group_sync(kBarPrep, kGroup);
    for (int c = 0; c < nchunks && ok; ++c) {
      const int par = c & 1;
      const long long t0 = s0 + (long long)kC * c;
      const int Lc = (int)min((long long)kC, s1 - t0);
      const uint32_t kqb = par ? KQ1 : KQ0;
      const int set = c % 3;
      const float* Lam = vecp(set, 0);
      const float* beta = vecp(set, 1);
      const float* gam = vecp(set, 2);
      float* rk = vecp(set, 3);
      float* rq = vecp(set, 4);
      float* us = vecp(set, 5);
      // decay factors exp(Lam_t - Lam_j), j <= t, with no positive exponent anywhere:
      // directly inside the diagonal 16x16 blocks; across blocks through the last
      // token e of j's block, exp(Lam_t - Lam_e) * exp(Lam_e - Lam_j).  (This chunk's
      // gates were computed during the previous chunk.)
      {
        float* DE = reinterpret_cast<float*>(smem + DEF);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int idx = u + 256 * k4;
          const int blk = idx >> 8, r = (idx >> 4) & 15, jj = idx & 15;
          DE[(16 * blk + r) * kLdDE + jj] =
              (jj <= r) ? __expf(Lam[16 * blk + r] - Lam[16 * blk + jj]) : 0.f;
        }
        if (u < 64) {
          float* RF = reinterpret_cast<float*>(smem + ROWF);
          reinterpret_cast<float*>(smem + COLF)[u] = __expf(Lam[u | 15] - Lam[u]);
#pragma unroll
          for (int blk = 0; blk < 3; ++blk)
            RF[64 * blk + u] = (16 * blk + 15 < u) ? __expf(Lam[u] - Lam[16 * blk + 15]) : 0.f;
        }
      }
      // this chunk's K/Q tiles (their arrival also means the state group has finished
      // chunk c - 2, so the P buffer of this parity and the vector set of chunk c + 1
      // are free)
      pend_bar[0] = &bars->kqtma[par];
      pend_par[0] = (c >> 1) & 1;
      if (!group_wait(&bars->kqtma[par], (c >> 1) & 1, kBarPrep, abort_flag, ERR_TMA_TIMEOUT)) {
        ok = false;
        break;
      }
      pend_bar[0] = &bars->kq;
      pend_par[0] = c & 1;
      if (u == 0) {  // [Skk; Sqk] = [K; Q] K^T
        tc_fence_after();
        const uint32_t idesc = umma_idesc_bf16(128, 64, false, false);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = 16384u * (ks >> 2) + 32u * (ks & 3);
          const uint64_t kd = umma_desc_k(sb + kqb + off);
          umma_bf16(tmem + TKQ, kd, kd, idesc, ks > 0);
        }
        umma_commit(&bars->kq);
      }
      // while the MMA runs: gates (warps 14-15) and q/k row norms (warps 10-13)
      if (gt >= 0 && c + 1 < nchunks) {  // gates of chunk c + 1, then prefetch c + 2
        compute_gates(c + 1);
        if (c + 2 < nchunks) load_gates(c + 2);
      }
      if (u >= 64 && u < 192) {  // q/k row norms
        const int t = u & 63;
        const bool isq = u < 128;
        const uint32_t b0 = sb + kqb + (isq ? 8192u : 0u) + 128u * t;
        float ss = 0.f;
#pragma unroll
        for (int blk = 0; blk < 2; ++blk)
#pragma unroll
          for (int ci = 0; ci < 8; ++ci) {
            const int ch = (ci + t) & 7;
            const uint4 w = ld_shared_v4(b0 + 16384u * blk + 16u * ch);
            const uint32_t w4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = bf2x2_to_f2(w4[e]);
              ss = fmaf(f.x, f.x, ss);
              ss = fmaf(f.y, f.y, ss);
            }
          }
        const float r = rsqrtf(ss + kL2NormEps);
        if (isq) rq[t] = r; else rk[t] = r;
      }
      group_sync(kBarPrep, kGroup);
      if (u < 64) us[u] = (u < Lc) ? rk[u] * expf(Lam[63] - Lam[u]) : 0.f;
      if (!group_wait(&bars->kq, c & 1, kBarPrep, abort_flag, ERR_MMA_TIMEOUT)) {
        ok = false;
        break;
      }
      pend_bar[0] = nullptr;
      tc_fence_after();
      // A (from Skk) -> AT in place; P hi (from Sqk) -> P[par]; Q~ = gamma rq Q in place
      {
        const int t = row & 63, bt = t >> 4;
        const bool is_k = row < 64;
        const float ft = is_k ? beta[t] * rk[t] : rq[t];
        const float* DE = reinterpret_cast<const float*>(smem + DEF) + t * kLdDE;
        const float* RF = reinterpret_cast<const float*>(smem + ROWF);
        const float* CF = reinterpret_cast<const float*>(smem + COLF);
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {  // one 16-token block of columns per pass
          const int j0 = 32 * half + 16 * pass, bj = j0 >> 4;
          float ej[16];
          if ((t | 31) < j0) {  // whole warp above the diagonal (warp-uniform)
#pragma unroll
            for (int i = 0; i < 16; ++i) ej[i] = 0.f;
          } else {
            float kq[16], rv[16], fv[16];
            tmem_ld16(tl + TKQ + (uint32_t)j0, kq);
            // factor row: diagonal block from DE, earlier blocks RF x CF, later ones 0
            const float rowf = ft * ((bj < bt) ? RF[64 * bj + t] : (bj == bt ? 1.f : 0.f));
            const float* fsrc = (bj == bt) ? DE : (CF + j0);
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
              const float4 rj = *reinterpret_cast<const float4*>(rk + j0 + i);
              const float4 f4 = *reinterpret_cast<const float4*>(fsrc + i);
              rv[i] = rj.x; rv[i + 1] = rj.y; rv[i + 2] = rj.z; rv[i + 3] = rj.w;
              fv[i] = f4.x; fv[i + 1] = f4.y; fv[i + 2] = f4.z; fv[i + 3] = f4.w;
            }
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int j = j0 + i;
              const bool keep = is_k ? (j < t) : (j <= t);
              ej[i] = keep ? rowf * fv[i] * rv[i] * kq[i] : 0.f;
            }
          }
          if (is_k) {
            float* Arow = reinterpret_cast<float*>(smem + AT) + t * kLd + j0;
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<float4*>(Arow + i) =
                  make_float4(ej[i], ej[i + 1], ej[i + 2], ej[i + 3]);
          } else {
            const uint32_t pb = sb + (par ? P1 : P0);
#pragma unroll
            for (int q2 = 0; q2 < 2; ++q2) {
              const float* e8 = &ej[8 * q2];
              st_v4(pb + sw128(t, (j0 >> 3) + q2),
                    make_uint4(cvt_bf16x2(e8[0], e8[1]), cvt_bf16x2(e8[2], e8[3]),
                               cvt_bf16x2(e8[4], e8[5]), cvt_bf16x2(e8[6], e8[7])));
            }
          }
        }
        if (!is_k) {
          // Q~ row t, d-block `half` (the KQ MMA that read Q has completed);
          // bf16x2 multiplies: this term only feeds the bf16 output
          const __nv_bfloat162 f2 = __float2bfloat162_rn(gam[t] * rq[t]);
          const uint32_t qb = sb + kqb + 8192u + 16384u * half + 128u * t;
#pragma unroll
          for (int ci = 0; ci < 8; ++ci) {
            const int ch = (ci + t) & 7;
            uint4 w = ld_shared_v4(qb + 16u * ch);
            __nv_bfloat162* w2 = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
            for (int e = 0; e < 4; ++e) w2[e] = __hmul2(w2[e], f2);
            st_v4(qb + 16u * ch, w);
          }
        }
      }
      tc_fence_before();
      group_sync(kBarPrep, kGroup);
      invert_in_place<kBarPrep>(reinterpret_cast<float*>(smem + AT), reinterpret_cast<float*>(smem + E), u);
      // T hi/lo once the state group has consumed the previous chunk's T
      if (c >= 1 && !group_wait(&bars->t_free, (c - 1) & 1, kBarPrep, abort_flag,
                                ERR_MMA_TIMEOUT)) { ok = false; break; }
#pragma unroll
      for (int k2 = 0; k2 < 2; ++k2) {
        const int unit = u + 256 * k2;
        const int t = unit >> 3, cidx = unit & 7;
        const float* tr = reinterpret_cast<const float*>(smem + AT) + t * kLd + 8 * cidx;
        const float4 ta = *reinterpret_cast<const float4*>(tr);
        const float4 tb = *reinterpret_cast<const float4*>(tr + 4);
        const float tv[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
        uint4 hi, lo;
        split8(tv, hi, lo);
        st_v4(sb + THI + sw128(t, cidx), hi);
        st_v4(sb + TLO + sw128(t, cidx), lo);
      }
      fence_proxy_async();
      group_sync(kBarPrep, kGroup);
      if (u == 0) mbar_arrive(&bars->t_ready);
    }
  } else {
    // =========================== state group
    const float scale = default_scale(p.scale);
    // initial state -> TMEM: fp32 (TS) and bf16 hi/lo (TSH / TSL), row v = row, k-half
    {
      float sv[64];
      if constexpr (HAS_STATE) {
        const float* srow = p.state + (((size_t)n * HV + h) * kHeadDim + row) * kHeadDim + 64 * half;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 v4 = ld_stream_f4(srow + 4 * i);
          sv[4 * i] = v4.x; sv[4 * i + 1] = v4.y; sv[4 * i + 2] = v4.z; sv[4 * i + 3] = v4.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) sv[i] = 0.f;
      }
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        uint32_t w[32], whi[16], wlo[16];
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(sv[32 * part + i]);
        tmem_st32(tl + TS + 64u * half + 32u * part, w);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float x0 = sv[32 * part + 2 * i], x1 = sv[32 * part + 2 * i + 1];
          const uint32_t b0 = __float_as_uint(x0), b1 = __float_as_uint(x1);
          whi[i] = pack_hi16(b0, b1);
          wlo[i] = pack_hi16(__float_as_uint(x0 - __uint_as_float(b0 & 0xFFFF0000u)),
                             __float_as_uint(x1 - __uint_as_float(b1 & 0xFFFF0000u)));
        }
        tmem_st16(tl + TSH + 32u * half + 16u * part, whi);
        tmem_st16(tl + TSL + 32u * half + 16u * part, wlo);
      }
      tmem_wait_st();
    }
    if (tid == 0) {
      fence_proxy_async();
      mbar_arrive_expect_tx(&bars->vtma, 2 * 8192);
      tma_load_2d(smem + V, &tm_v, &bars->vtma, h * 128, (int)s0);
      tma_load_2d(smem + V + 8192, &tm_v, &bars->vtma, h * 128 + 64, (int)s0);
    }
    tc_fence_before();
    group_sync(kBarState, kGroup);
    for (int c = 0; c < nchunks && ok; ++c) {
      const int par = c & 1;
      const long long t0 = s0 + (long long)kC * c;
      const int Lc = (int)min((long long)kC, s1 - t0);
      const uint32_t kqb = par ? KQ1 : KQ0;
      const float* Lam = vecp(c % 3, 0);
      const float* beta = vecp(c % 3, 1);
      const float* gam = vecp(c % 3, 2);
      const float* rk = vecp(c % 3, 3);
      const float* us = vecp(c % 3, 5);
      pend_bar[1] = &bars->vtma;
      pend_par[1] = c & 1;
      if (!group_wait(&bars->t_ready, c & 1, kBarState, abort_flag, ERR_MMA_TIMEOUT) ||
          !group_wait(&bars->vtma, c & 1, kBarState, abort_flag, ERR_TMA_TIMEOUT)) {
        ok = false;
        break;
      }
      pend_bar[1] = nullptr;
      // G1: S K^T (S hi + S lo) and O = S_hi Q~^T, A operands from TMEM
      if (tid == 0) {
        tc_fence_after();
        // S_hi [K; Q~]^T as one N = 128 MMA per k-step (K rows then Q~ rows are one
        // 128-row tile; D columns TSK.. then TO = TSK + 64), then S_lo K^T (N = 64)
        const uint32_t id128 = umma_idesc_bf16(128, 128, false, false);
        const uint32_t id64 = umma_idesc_bf16(128, 64, false, false);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = 16384u * (ks >> 2) + 32u * (ks & 3);
          const uint64_t kd = umma_desc_k(sb + kqb + off);
          umma_bf16_tmem_a(tmem + TSK, tmem + TSH + 8u * ks, kd, id128, ks > 0);
          umma_bf16_tmem_a(tmem + TSK, tmem + TSL + 8u * ks, kd, id64, 1);
        }
        umma_commit(&bars->g1);
      }
      pend_bar[0] = &bars->g1;
      pend_par[0] = c & 1;
      // meanwhile: pre-scale the fp32 state by this chunk's decay (the G3 MMA accumulates on it)
      {
        const float G = expf(Lam[63]);
        float sv[32];
        uint32_t w[32];
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          tmem_ld32(tl + TS + 64u * half + 32u * part, sv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(G * sv[i]);
          tmem_st32(tl + TS + 64u * half + 32u * part, w);
        }
        tmem_wait_st();
      }
      if (!group_wait(&bars->g1, c & 1, kBarState, abort_flag, ERR_MMA_TIMEOUT)) {
        ok = false;
        break;
      }
      pend_bar[0] = nullptr;
      tc_fence_after();
      // R^T[v][j] = beta_j (V[j][v] - gamma_j rk_j (S K^T)[v][j]) -> hi/lo K-major [v][j]
      {
        float sk[32], bj[32], gj[32];
        tmem_ld32(tl + TSK + 32u * half, sk);
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 b4 = *reinterpret_cast<const float4*>(beta + 32 * half + i);
          const float4 g4 = *reinterpret_cast<const float4*>(gam + 32 * half + i);
          const float4 r4 = *reinterpret_cast<const float4*>(rk + 32 * half + i);
          bj[i] = b4.x; bj[i + 1] = b4.y; bj[i + 2] = b4.z; bj[i + 3] = b4.w;
          gj[i] = g4.x * r4.x; gj[i + 1] = g4.y * r4.y; gj[i + 2] = g4.z * r4.z; gj[i + 3] = g4.w * r4.w;
        }
        // V tile element (t, v): box v/64, row t, 16-byte chunk ((v%64)/8) swizzled, 2-byte lane v%8
        const uint16_t* vt = reinterpret_cast<const uint16_t*>(smem + V + 8192u * (row >> 6));
        const int vc = (row & 63) >> 3, ve = row & 7;
        float vv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int t = 32 * half + i;
          const uint16_t bits = vt[t * 64 + ((vc ^ (t & 7)) << 3) + ve];
          vv[i] = __uint_as_float((uint32_t)bits << 16);
        }
        tmem_wait_ld();
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float x[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int i = 8 * q4 + e;
            x[e] = bj[i] * (vv[i] - gj[i] * sk[i]);
          }
          uint4 hi, lo;
          split8(x, hi, lo);
          st_v4(sb + RHI + sw128(row, 4 * half + q4), hi);
          st_v4(sb + RLO + sw128(row, 4 * half + q4), lo);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      group_sync(kBarState, kGroup);
      // G2: U^T = R^T T^T  (R_hi T_hi + R_lo T_hi + R_hi T_lo)
      if (tid == 0) {
        tc_fence_after();
        const uint32_t idesc = umma_idesc_bf16(128, 64, false, false);
#pragma unroll
        for (int term = 0; term < 3; ++term) {
          const uint32_t a = sb + (term == 1 ? RLO : RHI);
          const uint32_t b = sb + (term == 2 ? TLO : THI);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16(tmem + TUT, umma_desc_k(a + 32u * ks), umma_desc_k(b + 32u * ks), idesc,
                      (term | ks) != 0);
        }
        umma_commit(&bars->g2);
      }
      pend_bar[0] = &bars->g2;
      pend_par[0] = c & 1;
      if (!group_wait(&bars->g2, c & 1, kBarState, abort_flag, ERR_MMA_TIMEOUT)) {
        ok = false;
        break;
      }
      pend_bar[0] = nullptr;
      tc_fence_after();
      if (tid == 0) {
        mbar_arrive(&bars->t_free);  // T consumed: the prep group may write the next one
        if (c + 1 < nchunks) {       // V consumed (read into registers above)
          pend_bar[1] = &bars->vtma;
          pend_par[1] = (c + 1) & 1;
          fence_proxy_async();
          mbar_arrive_expect_tx(&bars->vtma, 2 * 8192);
          tma_load_2d(smem + V, &tm_v, &bars->vtma, h * 128, (int)(t0 + kC));
          tma_load_2d(smem + V + 8192, &tm_v, &bars->vtma, h * 128 + 64, (int)(t0 + kC));
        }
      }
      // U -> U~ = diag(us) U (hi/lo) and U hi, K-major [v][t]
      {
        float uv[32], uw[32];
        tmem_ld32(tl + TUT + 32u * half, uv);
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 w4 = *reinterpret_cast<const float4*>(us + 32 * half + i);
          uw[i] = w4.x; uw[i + 1] = w4.y; uw[i + 2] = w4.z; uw[i + 3] = w4.w;
        }
        tmem_wait_ld();
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float x[8];
          const float* u8 = &uv[8 * q4];
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = u8[e] * uw[8 * q4 + e];
          uint4 hi, lo;
          split8(x, hi, lo);
          const uint32_t o = sw128(row, 4 * half + q4);
          st_v4(sb + UTHI + o, hi);
          st_v4(sb + UTLO + o, lo);
          st_v4(sb + UHI + o, make_uint4(cvt_bf16x2(u8[0], u8[1]), cvt_bf16x2(u8[2], u8[3]),
                                         cvt_bf16x2(u8[4], u8[5]), cvt_bf16x2(u8[6], u8[7])));
        }
      }
      fence_proxy_async();
      tc_fence_before();
      group_sync(kBarState, kGroup);
      // G3: S += U~^T K (on the decay-scaled S);  O += U^T P^T
      if (tid == 0) {
        tc_fence_after();
        const uint32_t id_s = umma_idesc_bf16(128, 128, false, true);
#pragma unroll
        for (int part = 0; part < 2; ++part)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16(tmem + TS, umma_desc_k(sb + (part ? UTLO : UTHI) + 32u * ks),
                      umma_desc_mn(sb + kqb + 2048u * ks, 16384), id_s, 1);
        const uint32_t id_p = umma_idesc_bf16(128, 64, false, false);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tmem + TO, umma_desc_k(sb + UHI + 32u * ks),
                    umma_desc_k(sb + (par ? P1 : P0) + 32u * ks), id_p, 1);
        umma_commit(&bars->g3);
      }
      pend_bar[0] = &bars->g3;
      pend_par[0] = c & 1;
      if (!group_wait(&bars->g3, c & 1, kBarState, abort_flag, ERR_MMA_TIMEOUT)) {
        ok = false;
        break;
      }
      pend_bar[0] = nullptr;
      tc_fence_after();
      // K/Q buffer `par`, the P buffer of this parity and this chunk's vector set are
      // consumed: fetch chunk c + 2 now, so that its copy overlaps this epilogue
      if (tid == 0 && c + 2 < nchunks) issue_kq(c + 2);
      // epilogue: S(c+1) -> bf16 hi/lo in TMEM (or the final state to global); O -> staging
      const bool last = c + 1 == nchunks;
      // state checkpoint after this chunk, when one is due
      const long long ci = p.ckpt == nullptr ? -1
          : checkpoint_slot(p.ckpt_starts, n, min((long long)kC * (c + 1), L), p.ckpt_every,
                            p.ckpt_cap);
      {
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          float sv[32];
          tmem_ld32(tl + TS + 64u * half + 32u * part, sv);
          tmem_wait_ld();
          if (ci >= 0) {
            float* cp = p.ckpt + (((size_t)ci * HV + h) * kHeadDim + row) * kHeadDim +
                        64 * half + 32 * part;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              st_stream_f4(cp + i, make_float4(sv[i], sv[i + 1], sv[i + 2], sv[i + 3]));
          }
          if (last) {
            float* dst = nsbase + (size_t)row * kHeadDim + 64 * half + 32 * part;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              st_stream_f4(dst + i, make_float4(sv[i], sv[i + 1], sv[i + 2], sv[i + 3]));
          } else {
            uint32_t whi[16], wlo[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const uint32_t b0 = __float_as_uint(sv[2 * i]), b1 = __float_as_uint(sv[2 * i + 1]);
              whi[i] = pack_hi16(b0, b1);
              wlo[i] = pack_hi16(__float_as_uint(sv[2 * i] - __uint_as_float(b0 & 0xFFFF0000u)),
                                 __float_as_uint(sv[2 * i + 1] - __uint_as_float(b1 & 0xFFFF0000u)));
            }
            tmem_st16(tl + TSH + 32u * half + 16u * part, whi);
            tmem_st16(tl + TSL + 32u * half + 16u * part, wlo);
          }
        }
        float ov[32];
        tmem_ld32(tl + TO + 32u * half, ov);
        tmem_wait_ld();
        uint16_t* ostage = reinterpret_cast<uint16_t*>(smem + RHI);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const uint32_t pr = cvt_bf16x2(scale * ov[i], scale * ov[i + 1]);
          ostage[(32 * half + i) * kHeadDim + row] = (uint16_t)(pr & 0xFFFFu);
          ostage[(32 * half + i + 1) * kHeadDim + row] = (uint16_t)(pr >> 16);
        }
        if (!last) tmem_wait_st();
      }
      tc_fence_before();
      group_sync(kBarState, kGroup);
      {
        __nv_bfloat16* obase = p.out + (size_t)t0 * p.o_rs + (size_t)h * kHeadDim;
        uint4 v4[4];
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int unit = u + 256 * k4;
          v4[k4] = ld_shared_v4(sb + RHI + 256u * (unit >> 4) + 16u * (unit & 15));
        }
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int unit = u + 256 * k4, t = unit >> 4;
          if (t < Lc)
            *reinterpret_cast<uint4*>(obase + (size_t)t * p.o_rs + 8 * (unit & 15)) = v4[k4];
        }
      }
      group_sync(kBarState, kGroup);
    }
  }
  // a wait ran out: tell the other group, give our in-flight copies / MMAs one more
  // bounded chance to land, then release TMEM
  if (!ok) {
    *abort_flag = 1;
    if (u == 0)
      for (int i = 0; i < 2; ++i)
        if (pend_bar[i]) mbar_wait(pend_bar[i], pend_par[i], 1u << 20);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <bool HS, typename CuT>
cudaError_t launch_pipelined_t(const CUtensorMap& mq, const CUtensorMap& mk,
                               const CUtensorMap& mv, const ChunkedParams& cp, int nseq,
                               cudaStream_t st) {
  auto kern = prefill_pipelined_kernel<HS, CuT>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl::SMEM);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  kern<<<dim3((unsigned)((long long)nseq * cp.HV)), dim3(pl::kThreads), pl::SMEM, st>>>(mq, mk,
                                                                                         mv, cp);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- host side
template <bool L2, bool HS, typename CuT>
cudaError_t launch_chunked_t(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                             const ChunkedParams& cp, int nseq, cudaStream_t st) {
  auto kern = prefill_chunked_kernel<L2, HS, CuT>;
  static bool configured[64] = {};  // per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  kern<<<dim3((unsigned)((long long)nseq * cp.HV)), dim3(kThreads), SMEM_ALLOC, st>>>(mq, mk, mv,
                                                                                     cp);
  return cudaGetLastError();
}

template <typename CuT>
cudaError_t launch_chunked_cu(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                              const ChunkedParams& cp, bool l2, bool has_state, int nseq,
                              cudaStream_t st) {
  if (l2) {
    return has_state ? launch_chunked_t<true, true, CuT>(mq, mk, mv, cp, nseq, st)
                     : launch_chunked_t<true, false, CuT>(mq, mk, mv, cp, nseq, st);
  }
  return has_state ? launch_chunked_t<false, true, CuT>(mq, mk, mv, cp, nseq, st)
                   : launch_chunked_t<false, false, CuT>(mq, mk, mv, cp, nseq, st);
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// [rows][heads * 128] bf16 matrix with rows `row_stride` elements apart, 64 x 64 boxes,
// 128-byte swizzle.
bool make_tile_map_box(CUtensorMap* m, const void* base, int heads, long long rows,
                       long long row_stride, int box_x, bool swizzle128) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr || row_stride < (long long)heads * kHeadDim || row_stride % 8 != 0)
    return false;
  cuuint64_t dims[2] = {(cuuint64_t)heads * kHeadDim, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_x, 64};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_tile_map(CUtensorMap* m, const void* base, int heads, long long rows,
                   long long row_stride) {
  return make_tile_map_box(m, base, heads, rows, row_stride, 64, true);
}

size_t prefill_chunked_workspace(int num_seqs) {
  if (num_seqs <= 1 || num_seqs > kLptMaxSeqs) return 0;
  return ((size_t)num_seqs * sizeof(int) + 255) & ~(size_t)255;
}

bool prefill_chunked_supported(const PrefillArgs& p) {
  const auto a16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  // TMA rows and 16-byte output stores: every token row starts on a 16-byte boundary
  const bool rows16 = p.rs.q % 8 == 0 && p.rs.k % 8 == 0 && p.rs.v % 8 == 0 && p.rs.o % 8 == 0;
  return p.T > 0 && p.T < (1LL << 31) && a16(p.q) && a16(p.k) && a16(p.v) && a16(p.out) &&
         rows16 && tensor_map_encoder() != nullptr;
}

cudaError_t launch_prefill_chunked(const PrefillArgs& p, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  if (!make_tile_map(&mq, p.q, p.HQ, p.T, p.rs.q) || !make_tile_map(&mk, p.k, p.HQ, p.T, p.rs.k) ||
      !make_tile_map(&mv, p.v, p.HV, p.T, p.rs.v))
    return cudaErrorInvalidValue;
  int* order = nullptr;
  if (p.N > 1 && p.N <= kLptMaxSeqs && p.workspace != nullptr &&
      p.workspace_bytes >= (size_t)p.N * sizeof(int)) {
    order = static_cast<int*>(p.workspace);
    int P = 1;
    while (P < p.N) P <<= 1;
    const size_t sm = (size_t)P * sizeof(unsigned long long);
    static bool lpt_configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !lpt_configured[dev]) {
      cudaFuncSetAttribute(lpt_order_kernel<int>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kLptMaxSeqs * 8);
      cudaFuncSetAttribute(lpt_order_kernel<long long>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, kLptMaxSeqs * 8);
      if (dev >= 0 && dev < 64) lpt_configured[dev] = true;
    }
    if (p.cu_int64)
      lpt_order_kernel<long long><<<1, 1024, sm, st>>>(static_cast<const long long*>(p.cu), p.N,
                                                        p.T, order);
    else
      lpt_order_kernel<int><<<1, 1024, sm, st>>>(static_cast<const int*>(p.cu), p.N, p.T, order);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  ChunkedParams cp{static_cast<const __nv_bfloat16*>(p.a), static_cast<const __nv_bfloat16*>(p.b),
                   p.A_log, p.dt_bias, p.cu, p.state, p.new_state,
                   static_cast<__nv_bfloat16*>(p.out), order, p.rs.a, p.rs.b, p.rs.o, p.T,
                   p.cu_int64 ? 1 : 0, p.HV,
                   p.HV / p.HQ, p.scale, p.gates_pre, p.g_alpha, p.g_beta, p.ckpt,
                   p.ckpt_starts, p.ckpt_capacity, p.ckpt_every};
  if (!p.l2norm && (p.gates_pre || p.ckpt != nullptr))
    return cudaErrorInvalidValue;  // the raw-q/k fused kernel has neither (the entry routes
                                   // such calls to the split kernels)
  if (p.l2norm) {  // warp-specialised, pipelined kernel
    const bool hs = p.state != nullptr;
    if (p.cu_int64)
      return hs ? launch_pipelined_t<true, long long>(mq, mk, mv, cp, p.N, st)
                : launch_pipelined_t<false, long long>(mq, mk, mv, cp, p.N, st);
    return hs ? launch_pipelined_t<true, int>(mq, mk, mv, cp, p.N, st)
              : launch_pipelined_t<false, int>(mq, mk, mv, cp, p.N, st);
  }
  if (p.cu_int64)
    return launch_chunked_cu<long long>(mq, mk, mv, cp, p.l2norm, p.state != nullptr, p.N, st);
  return launch_chunked_cu<int>(mq, mk, mv, cp, p.l2norm, p.state != nullptr, p.N, st);
}

unsigned read_device_error(bool clear) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_prefill_device_error, sizeof(v)) != cudaSuccess) return ~0u;
  if (clear) {
    const unsigned zero = 0;
    cudaMemcpyToSymbol(g_prefill_device_error, &zero, sizeof(zero));
  }
  return v;
}

}  // namespace gdn
