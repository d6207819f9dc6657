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
#include "gdn_prefill.cuh"
#include "sm100.cuh"

namespace gdn {

__device__ unsigned int g_prefill_device_error = 0;

namespace {
using namespace sm100;

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
  long long T;
  int cu64;
  int HV;
  int ratio;
  float scale;
};

// bf16 conversions with integer operations (ALU pipe) rather than cvt (which
// shares the XU pipe with exp/rsqrt and was the kernel's busiest pipe).
// Round-to-nearest-even of a finite fp32 bit pattern to bf16, kept in the high half.
__device__ __forceinline__ uint32_t rn_bf16_bits(uint32_t xb) {
  return (xb + 0x7FFFu + ((xb >> 16) & 1u)) & 0xFFFF0000u;
}
// Two bf16 values held in the high halves of a and b -> one packed word (a low, b high).
__device__ __forceinline__ uint32_t pack_hi16(uint32_t a, uint32_t b) {
  return __byte_perm(a, b, 0x7632);
}
__device__ __forceinline__ uint32_t pack_bf16(float x, float y) {
  return pack_hi16(rn_bf16_bits(__float_as_uint(x)), rn_bf16_bits(__float_as_uint(y)));
}
// 8 floats -> (hi, lo) bf16 chunks with x ~= hi + lo: hi is x truncated to bf16
// (exact residual x - hi, |x - hi| < 2^-7 |x|), lo is that residual rounded to
// bf16, so hi + lo carries ~16 significant bits.
__device__ __forceinline__ void split8(const float* x, uint4& hi, uint4& lo) {
  uint32_t hb[8], lb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    hb[i] = __float_as_uint(x[i]) & 0xFFFF0000u;
    lb[i] = rn_bf16_bits(__float_as_uint(x[i] - __uint_as_float(hb[i])));
  }
  hi = make_uint4(pack_hi16(hb[0], hb[1]), pack_hi16(hb[2], hb[3]), pack_hi16(hb[4], hb[5]),
                  pack_hi16(hb[6], hb[7]));
  lo = make_uint4(pack_hi16(lb[0], lb[1]), pack_hi16(lb[2], lb[3]), pack_hi16(lb[4], lb[5]),
                  pack_hi16(lb[6], lb[7]));
}
// 16 consecutive fp32 TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void st_v4(uint32_t addr, uint4 v) {
  st_shared_v4(addr, v.x, v.y, v.z, v.w);
}

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
        const size_t ti = (size_t)(tc0 + t) * HV + h;
        ga[e] = bf2f(p.a[ti]);
        gb[e] = bf2f(p.b[ti]);
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
      __nv_bfloat16* obase = p.out + ((size_t)t0 * HV + h) * kHeadDim;
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
          *reinterpret_cast<uint4*>(obase + (size_t)t * HV * kHeadDim + 8 * (u & 15)) = v4[k4];
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

// ---------------------------------------------------------------- LPT order
// CTAs are scheduled roughly in blockIdx order and one CTA fills an SM, so
// handing out the longest sequences first (longest-processing-time) keeps the
// last wave short.  One CTA bitonic-sorts (length desc, index asc) keys in
// shared memory and writes the permutation.
constexpr int kLptMaxSeqs = 8192;

template <typename CuT>
__global__ void __launch_bounds__(1024) lpt_order_kernel(const CuT* __restrict__ cu, int N,
                                                         long long T, int* __restrict__ order) {
  extern __shared__ unsigned long long keys[];
  int P = 1;
  while (P < N) P <<= 1;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    unsigned long long key = 0ull;  // padding sorts last
    if (i < N) {
      const long long a = min(max((long long)cu[i], 0LL), T);
      const long long b = min(max((long long)cu[i + 1], 0LL), T);
      const unsigned long long len = (unsigned long long)max(b - a, 0LL);
      key = (len << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)i);
    }
    keys[i] = key;
  }
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long x = keys[i], y = keys[l];
          const bool desc = (i & k) == 0;  // descending overall
          if (desc ? (x < y) : (x > y)) {
            keys[i] = y;
            keys[l] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < N; i += blockDim.x)
    order[i] = (int)(0xFFFFFFFFu - (unsigned)(keys[i] & 0xFFFFFFFFull));
}

// ---------------------------------------------------------------- host side
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

// [rows][heads * 128] bf16 matrix, 64 x 64 boxes, 128-byte swizzle.
bool make_tile_map(CUtensorMap* m, const void* base, int heads, long long rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {(cuuint64_t)heads * kHeadDim, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)heads * kHeadDim * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

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

size_t prefill_chunked_workspace(int num_seqs) {
  if (num_seqs <= 1 || num_seqs > kLptMaxSeqs) return 0;
  return ((size_t)num_seqs * sizeof(int) + 255) & ~(size_t)255;
}

bool prefill_chunked_supported(const PrefillArgs& p) {
  const auto a16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  return p.T > 0 && p.T < (1LL << 31) && a16(p.q) && a16(p.k) && a16(p.v) && a16(p.out) &&
         tensor_map_encoder() != nullptr;
}

cudaError_t launch_prefill_chunked(const PrefillArgs& p, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  if (!make_tile_map(&mq, p.q, p.HQ, p.T) || !make_tile_map(&mk, p.k, p.HQ, p.T) ||
      !make_tile_map(&mv, p.v, p.HV, p.T))
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
                   static_cast<__nv_bfloat16*>(p.out), order, p.T, p.cu_int64 ? 1 : 0, p.HV,
                   p.HV / p.HQ, p.scale};
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
