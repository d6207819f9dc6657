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
//   W      = T diag(beta gamma rk) K,   U0 = T diag(beta) V,   gamma_t = exp(Lam_t)
//   U      = U0 - W S^T                          (per-token corrected values)
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
// fp32 quantities on the state path are split x = hi + lo (two bf16) and their
// products expanded: T diag(.) -> 2 MMAs, S W^T -> 3 MMAs (hi.hi + lo.hi + hi.lo),
// U~ -> 2 MMAs, all accumulated in fp32 in TMEM, so the fp32 state keeps ~16
// mantissa bits per step instead of bf16's 8.  Output-only terms (S Q^T, P U)
// use the hi part only.
//
// Orientation: the tensor-core D tiles are kept "v-major" (v = 128 TMEM lanes),
// so S (128 x 128), U^T, O^T and the state update all use M = 128 MMAs:
//   [Skk;Sqk] = [K;Q] K^T        M128 N64  K128   (A, B K-major, TMA tiles)
//   W^T       = K^T  T1^T        M128 N64  K64    (A = K tile MN-major)
//   U0^T      = V^T  T2^T        M128 N64  K64    (A = V tile MN-major)
//   O^T       = S_hi Q~^T        M128 N64  K128
//   U^T      -= S W^T            M128 N64  K128   (B = W^T MN-major, negated A)
//   dS        = U~^T K           M128 N128 K64    (B = K tile MN-major)
//   O^T      += U_hi^T P^T       M128 N64  K64    (+ U_lo P_hi, U_hi P_lo for raw q/k)
//
// One CTA (8 warps) owns one (sequence, v-head); warp w serves TMEM lanes
// 32*(w%4).. and column half w/4.  Thread 0 issues TMA and UMMA; completion is
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
constexpr int kThreads = 256;   // 8 warps
constexpr int kLdA = 65;        // padded row stride of the fp32 A matrix (bank-conflict free)

// ---- shared memory map (byte offsets from a 1024-byte aligned base) ----
constexpr uint32_t OFF_K0 = 0;        // K tile, d 0..63   [t][d]  (TMA, 128B swizzle)
constexpr uint32_t OFF_Q0 = 8192;     // Q tile, d 0..63
constexpr uint32_t OFF_K1 = 16384;    // K tile, d 64..127
constexpr uint32_t OFF_Q1 = 24576;    // Q tile, d 64..127
constexpr uint32_t OFF_V = 32768;     // V tile [t][v] 2 x 8 KB; then O staging [t][v] bf16
constexpr uint32_t OFF_SHI = 49152;   // S hi [v][k] K-major, 2 k-blocks of 16 KB
constexpr uint32_t OFF_SLO = 81920;   // S lo
constexpr uint32_t OFF_WHI = 114688;  // W^T hi [d][t] (MN-major B operand) 16 KB
constexpr uint32_t OFF_WLO = 131072;  // W^T lo
constexpr uint32_t OFF_U = 147456;    // 64 KB, phase-dependent:
//   A: Tmat f32[64][64] @16K, E scratch @32K,
//      then T1hi @32K, T1lo @40K, T2hi @48K, T2lo @56K (each [t][j] K-major 8 KB)
//   (the fp32 A matrix, [64][kLdA], lives in the W^T buffers, free until step 6)
//   B: U~hi [v][t] @0, U~lo @16K, Uhi @32K, Ulo @48K (K-major A operands, 16 KB each)
constexpr uint32_t OFF_P = 212992;    // P [t][j] K-major 8 KB
constexpr uint32_t OFF_VEC = 221184;  // fp32[64] vectors + barriers
constexpr uint32_t SMEM_USED = OFF_VEC + 2048;
constexpr uint32_t SMEM_ALLOC = SMEM_USED + 1024;  // + alignment slack

constexpr uint32_t U_TMAT = 16384, U_E = 32768;
constexpr uint32_t OFF_AMAT = OFF_WHI;  // 64 x 65 fp32 = 16.25 KB of the 32 KB W^T hi/lo region
constexpr uint32_t U_T1HI = 32768, U_T1LO = 40960, U_T2HI = 49152, U_T2LO = 57344;
constexpr uint32_t U_UTHI = 0, U_UTLO = 16384, U_UHI = 32768, U_ULO = 49152;
// Raw (un-normalised) q/k: |P| can reach |q||k| ~ 1e2 with heavy cancellation in
// P U, so that product is split too (P_hi U_hi + P_lo U_hi + P_hi U_lo).  P_lo is
// written into the W^T lo buffer once the S W^T MMAs that read it have completed.
constexpr uint32_t OFF_PLO = OFF_WLO;

// TMEM columns (512 allocated)
constexpr uint32_t TM_DS = 0;     // dS  128 lanes (v) x 128 (k)
constexpr uint32_t TM_UT = 128;   // U^T 128 (v) x 64 (t)
constexpr uint32_t TM_OT = 192;   // O^T 128 (v) x 64 (t)
constexpr uint32_t TM_WT = 256;   // W^T 128 (d) x 64 (t)
constexpr uint32_t TM_KQ = 320;   // lanes 0..63: Skk rows, 64..127: Sqk rows; 64 cols
constexpr uint32_t TM_COLS = 512;

enum : unsigned { ERR_TMA_TIMEOUT = 1u, ERR_MMA_TIMEOUT = 2u };

struct ChunkedParams {
  const __nv_bfloat16* a;
  const __nv_bfloat16* b;
  const float* A_log;
  const float* dt_bias;
  const void* cu;
  const float* state;
  float* new_state;
  __nv_bfloat16* out;
  long long T;
  int cu64;
  int HV;
  int ratio;
  float scale;
};

__device__ __forceinline__ uint32_t pack_bf16(float x, float y) {
  __nv_bfloat162 v = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
// 8 floats -> (hi, lo) bf16 chunks with x ~= hi + lo.
__device__ __forceinline__ void split8(const float* x, uint4& hi, uint4& lo) {
  float h[8], l[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    h[i] = bf16_round(x[i]);
    l[i] = x[i] - h[i];
  }
  hi = make_uint4(pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]), pack_bf16(h[4], h[5]),
                  pack_bf16(h[6], h[7]));
  lo = make_uint4(pack_bf16(l[0], l[1]), pack_bf16(l[2], l[3]), pack_bf16(l[4], l[5]),
                  pack_bf16(l[6], l[7]));
}
__device__ __forceinline__ uint4 pack8(const float* x) {
  return make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]), pack_bf16(x[4], x[5]),
                    pack_bf16(x[6], x[7]));
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
// by 16x16 diagonal-block forward substitution and two levels of block merges:
//   [[L11, 0], [L21, L22]]^-1 = [[T11, 0], [-T22 L21 T11, T22]].
// Called by all 256 threads (contains __syncthreads).
__device__ __forceinline__ void invert_unit_lower64(const float* __restrict__ A,
                                                    float* __restrict__ Tm,
                                                    float* __restrict__ E) {
  const int tid = threadIdx.x;
  // ---- level 1: four 16x16 diagonal blocks, one column per thread ----
  if (tid < 64) {
    const int blk = tid >> 4, col = tid & 15, o = 16 * blk;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < r; ++j) acc = fmaf(A[(o + r) * kLdA + o + j], x[j], acc);
      x[r] = (r < col) ? 0.f : ((r == col) ? 1.f : -acc);
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) Tm[(o + r) * 64 + o + col] = x[r];
  } else {
    // zero the blocks above the diagonal: rows 0..31 x cols 32..63, block (0,1), block (2,3)
    for (int u = tid - 64; u < 1536; u += kThreads - 64) {
      int r, c;
      if (u < 1024) { r = u >> 5; c = 32 + (u & 31); }
      else if (u < 1280) { r = (u - 1024) >> 4; c = 16 + ((u - 1024) & 15); }
      else { r = 32 + ((u - 1280) >> 4); c = 48 + ((u - 1280) & 15); }
      Tm[r * 64 + c] = 0.f;
    }
  }
  __syncthreads();
  // ---- level 2: blocks (1,0) and (3,2): T_ij = -D_i A_ij D_j ----
  {
    const int c = tid & 15, g = tid >> 4;  // 16 groups x 2 rows each
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int pr = g * 2 + rr;  // 0..31
      const int p = pr >> 4, r = pr & 15;
      const int bi = 16 * (2 * p + 1), bj = 16 * (2 * p);
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) acc = fmaf(A[(bi + r) * kLdA + bj + k], Tm[(bj + k) * 64 + bj + c], acc);
      E[p * 256 + r * 16 + c] = acc;
    }
  }
  __syncthreads();
  {
    const int c = tid & 15, g = tid >> 4;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int pr = g * 2 + rr;
      const int p = pr >> 4, r = pr & 15;
      const int bi = 16 * (2 * p + 1), bj = 16 * (2 * p);
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) acc = fmaf(Tm[(bi + r) * 64 + bi + k], E[p * 256 + k * 16 + c], acc);
      Tm[(bi + r) * 64 + bj + c] = -acc;
    }
  }
  __syncthreads();
  // ---- level 3: rows 32..63 x cols 0..31: -T22 A21 T11 ----
  {
    const int c = tid & 31, r0 = tid >> 5;  // rows r0, r0+8, r0+16, r0+24
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = r0 + 8 * i;
      float acc = 0.f;
#pragma unroll 8
      for (int k = 0; k < 32; ++k) acc = fmaf(A[(32 + r) * kLdA + k], Tm[k * 64 + c], acc);
      E[r * 32 + c] = acc;
    }
  }
  __syncthreads();
  {
    const int c = tid & 31, r0 = tid >> 5;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = r0 + 8 * i;
      float acc = 0.f;
#pragma unroll 8
      for (int k = 0; k < 32; ++k) acc = fmaf(Tm[(32 + r) * 64 + 32 + k], E[k * 32 + c], acc);
      Tm[(32 + r) * 64 + c] = -acc;
    }
  }
  __syncthreads();
}

template <bool L2NORM, bool HAS_STATE, typename CuT>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_chunked_kernel(const __grid_constant__ CUtensorMap tm_q,
                           const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const ChunkedParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int sp = warp & 3, half = warp >> 2;
  const int row = sp * 32 + lane;  // TMEM lane owned by this thread
  const int HV = p.HV;
  const int n = blockIdx.x / HV;
  const int h = blockIdx.x - n * HV;
  const int qh = h / p.ratio;
  const CuT* cu = static_cast<const CuT*>(p.cu);
  const long long s1 = min(max((long long)cu[n + 1], 0LL), p.T);
  const long long s0 = min(max((long long)cu[n], 0LL), s1);
  const long long L = s1 - s0;
  float* nsrow = p.new_state + (((size_t)n * HV + h) * kHeadDim + row) * kHeadDim + 64 * half;

  if (L <= 0) {  // empty sequence: zero final state (definition semantics)
#pragma unroll
    for (int i = 0; i < 16; ++i) st_stream_f4(nsrow + 4 * i, make_float4(0.f, 0.f, 0.f, 0.f));
    return;
  }

  float* vec = reinterpret_cast<float*>(smem + OFF_VEC);
  float* Lam = vec;         // cumulative log decay within the chunk
  float* beta = vec + 64;
  float* gam = vec + 128;   // exp(Lam)
  float* rk = vec + 192;
  float* rq = vec + 256;
  float* us = vec + 320;    // rk exp(Lam_end - Lam)
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(smem + OFF_VEC + 1536);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_VEC + 1552);
  float* Amat = reinterpret_cast<float*>(smem + OFF_AMAT);
  float* Tmat = reinterpret_cast<float*>(smem + OFF_U + U_TMAT);
  float* Escr = reinterpret_cast<float*>(smem + OFF_U + U_E);

  if (warp == 0) {
    tmem_alloc(tmem_slot, TM_COLS);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(bar_tma, 1);
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

  // ---- initial state: this thread keeps S[v=row][64*half .. +64) in fp32 registers ----
  float s[64];
  if constexpr (HAS_STATE) {
    const float* srow = p.state + (((size_t)n * HV + h) * kHeadDim + row) * kHeadDim + 64 * half;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 v4 = ld_stream_f4(srow + 4 * i);
      s[4 * i] = v4.x; s[4 * i + 1] = v4.y; s[4 * i + 2] = v4.z; s[4 * i + 3] = v4.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) s[i] = 0.f;
  }
  // S hi / lo -> shared (K-major [v][k], k-block = half)
  auto write_state_split = [&]() {
    const uint32_t bhi = sb + OFF_SHI + 16384u * half, blo = sb + OFF_SLO + 16384u * half;
#pragma unroll
    for (int cidx = 0; cidx < 8; ++cidx) {
      uint4 hi, lo;
      split8(&s[8 * cidx], hi, lo);
      st_v4(bhi + sw128(row, cidx), hi);
      st_v4(blo + sw128(row, cidx), lo);
    }
  };
  write_state_split();

  // P[t][j] = exp(Lam_t - Lam_j) rq_t rk_j Sqk[t][j] (j <= t) for this thread's row
  // t = row - 64 and 32-column half, as bf16 hi (or, with lo_part, the lo residual).
  auto write_p = [&](const float (&kq)[32], bool lo_part) {
    const int t = row - 64;
    const float qt = rq[t], lt = Lam[t];
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      float pv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = 32 * half + 8 * q4 + e;
        pv[e] = (j <= t) ? expf(lt - Lam[j]) * qt * rk[j] * kq[8 * q4 + e] : 0.f;
      }
      uint4 hi, lo;
      split8(pv, hi, lo);
      st_v4(sb + (lo_part ? OFF_PLO : OFF_P) + sw128(t, 4 * half + q4), lo_part ? lo : hi);
    }
  };

  const float nexpA = -expf(__ldg(p.A_log + h));
  const float dtb = __ldg(p.dt_bias + h);
  const float scale = default_scale(p.scale);
  const int nchunks = (int)((L + kC - 1) / kC);
  uint32_t ph_tma = 0, ph_mma = 0;
  bool ok = true;
  bool mma_pending = false, tma_pending = false;

  for (int c = 0; c < nchunks; ++c) {
    const long long t0 = s0 + (long long)kC * c;
    const int Lc = (int)min((long long)kC, s1 - t0);

    // (1) TMA: K, Q (GVA q/k head) and V tiles of this chunk
    fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      mbar_arrive_expect_tx(bar_tma, 6 * 8192);
      const int y = (int)t0;
      tma_load_2d(smem + OFF_K0, &tm_k, bar_tma, qh * 128, y);
      tma_load_2d(smem + OFF_K1, &tm_k, bar_tma, qh * 128 + 64, y);
      tma_load_2d(smem + OFF_Q0, &tm_q, bar_tma, qh * 128, y);
      tma_load_2d(smem + OFF_Q1, &tm_q, bar_tma, qh * 128 + 64, y);
      tma_load_2d(smem + OFF_V, &tm_v, bar_tma, h * 128, y);
      tma_load_2d(smem + OFF_V + 8192, &tm_v, bar_tma, h * 128 + 64, y);
    }
    tma_pending = true;
    // gates of the chunk (padding tokens: decay 1, beta 0), inclusive scan of log decay
    if (tid < 64) {
      float lg = 0.f, bt = 0.f;
      if (tid < Lc) {
        const size_t ti = (size_t)(t0 + tid) * HV + h;
        lg = nexpA * softplus_f(bf2f(p.a[ti]) + dtb);
        bt = sigmoid_f(bf2f(p.b[ti]));
      }
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, lg, off);
        if (lane >= off) lg += y;
      }
      Lam[tid] = lg;
      beta[tid] = bt;
    }
    __syncthreads();
    if (tid >= 32 && tid < 64) Lam[tid] += Lam[31];
    if (!cta_wait(bar_tma, ph_tma, ERR_TMA_TIMEOUT)) { ok = false; break; }
    ph_tma ^= 1;
    tma_pending = false;

    // (2) [Skk; Sqk] = [K; Q] K^T  (M128 N64 K128)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = umma_idesc_bf16(128, 64, false, false);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t off = 16384u * (ks >> 2) + 32u * (ks & 3);
        umma_bf16(tmem + TM_KQ, umma_desc_k(sb + OFF_K0 + off), umma_desc_k(sb + OFF_K0 + off),
                  idesc, ks > 0);
      }
      umma_commit(bar_mma);
    }
    mma_pending = true;
    // meanwhile: gamma, q/k L2-norm factors
    if (tid < 64) gam[tid] = expf(Lam[tid]);
    if constexpr (L2NORM) {
      if (tid >= 64 && tid < 192) {
        const int t = (tid - 64) & 63;
        const bool isq = tid < 128;
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

    // (3) A (from Skk) -> Amat;  P (from Sqk) -> bf16 [t][j];  Q~ = gamma rq Q in place
    {
      float kq[32];
      tmem_ld32(tl + TM_KQ + 32u * half, kq);
      tmem_wait_ld();
      if (row < 64) {
        const int t = row;
        const float bt = beta[t] * rk[t], lt = Lam[t];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int j = 32 * half + i;
          Amat[t * kLdA + j] = (j < t) ? bt * expf(lt - Lam[j]) * rk[j] * kq[i] : 0.f;
        }
      } else {
        const int t = row - 64;
        const float qt = rq[t];
        write_p(kq, false);
        // scale this thread's half of Q row t
        const float f = gam[t] * qt;
        const uint32_t qb = sb + (half ? OFF_Q1 : OFF_Q0);
#pragma unroll
        for (int ci = 0; ci < 8; ++ci) {
          const int ch = (ci + t) & 7;
          const uint32_t addr = qb + 128u * t + 16u * ch;
          const uint4 u = ld_shared_v4(addr);
          const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
          float x[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f2 = bf2x2_to_f2(w4[e]);
            x[2 * e] = f2.x * f;
            x[2 * e + 1] = f2.y * f;
          }
          st_v4(addr, pack8(x));
        }
      }
    }
    __syncthreads();

    // (4) T = (I + A)^-1;  T1 = T diag(beta gamma rk), T2 = T diag(beta) -> hi/lo bf16
    invert_unit_lower64(Amat, Tmat, Escr);
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2) {
      const int u = tid + kThreads * k2;  // 512 (row, 16B chunk) units
      const int t = u >> 3, cidx = u & 7;
      float w1[8], w2[8];
      const float4 ta = *reinterpret_cast<const float4*>(Tmat + t * 64 + 8 * cidx);
      const float4 tb = *reinterpret_cast<const float4*>(Tmat + t * 64 + 8 * cidx + 4);
      const float tv8[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = 8 * cidx + e;
        w2[e] = tv8[e] * beta[j];
        w1[e] = w2[e] * gam[j] * rk[j];
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

    // (5) W^T = K^T T1^T,  U0^T = V^T T2^T,  O^T = S_hi Q~^T
    if (tid == 0) {
      tc_fence_after();
      const uint32_t id_w = umma_idesc_bf16(128, 64, true, false);
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        const uint32_t t1 = sb + OFF_U + (part ? U_T1LO : U_T1HI);
        const uint32_t t2 = sb + OFF_U + (part ? U_T2LO : U_T2HI);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          umma_bf16(tmem + TM_WT, umma_desc_mn(sb + OFF_K0 + 2048u * ks, 16384),
                    umma_desc_k(t1 + 32u * ks), id_w, (part | ks) != 0);
          umma_bf16(tmem + TM_UT, umma_desc_mn(sb + OFF_V + 2048u * ks, 8192),
                    umma_desc_k(t2 + 32u * ks), id_w, (part | ks) != 0);
        }
      }
      const uint32_t id_o = umma_idesc_bf16(128, 64, false, false);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t kb = 32u * (ks & 3);
        umma_bf16(tmem + TM_OT, umma_desc_k(sb + OFF_SHI + 16384u * (ks >> 2) + kb),
                  umma_desc_k(sb + ((ks >> 2) ? OFF_Q1 : OFF_Q0) + kb), id_o, ks > 0);
      }
      umma_commit(bar_mma);
    }
    mma_pending = true;
    if (!cta_wait(bar_mma, ph_mma, ERR_MMA_TIMEOUT)) { ok = false; break; }
    ph_mma ^= 1;
    mma_pending = false;
    tc_fence_after();

    // (6) W^T -> hi/lo, MN-major [d][t]
    {
      float wv[32];
      tmem_ld32(tl + TM_WT + 32u * half, wv);
      tmem_wait_ld();
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint4 hi, lo;
        split8(&wv[8 * q4], hi, lo);
        st_v4(sb + OFF_WHI + sw128(row, 4 * half + q4), hi);
        st_v4(sb + OFF_WLO + sw128(row, 4 * half + q4), lo);
      }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();

    // (7) U^T -= S W^T  (hi.hi + lo.hi + hi.lo)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t id_x = umma_idesc_bf16(128, 64, false, true, true);
#pragma unroll
      for (int term = 0; term < 3; ++term) {
        const uint32_t sa = sb + (term == 1 ? OFF_SLO : OFF_SHI);
        const uint32_t wb = sb + (term == 2 ? OFF_WLO : OFF_WHI);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_bf16(tmem + TM_UT, umma_desc_k(sa + 16384u * (ks >> 2) + 32u * (ks & 3)),
                    umma_desc_mn(wb + 2048u * ks, 8192), id_x, 1);
      }
      umma_commit(bar_mma);
    }
    mma_pending = true;
    if (!cta_wait(bar_mma, ph_mma, ERR_MMA_TIMEOUT)) { ok = false; break; }
    ph_mma ^= 1;
    mma_pending = false;
    tc_fence_after();

    // (8) U -> U~ = diag(us) U (hi/lo) and U hi, K-major [v][t]
    {
      float uv[32];
      tmem_ld32(tl + TM_UT + 32u * half, uv);
      tmem_wait_ld();
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        float x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = uv[8 * q4 + e] * us[32 * half + 8 * q4 + e];
        uint4 hi, lo;
        split8(x, hi, lo);
        const uint32_t o = sw128(row, 4 * half + q4);
        st_v4(sb + OFF_U + U_UTHI + o, hi);
        st_v4(sb + OFF_U + U_UTLO + o, lo);
        split8(&uv[8 * q4], hi, lo);
        st_v4(sb + OFF_U + U_UHI + o, hi);
        if constexpr (!L2NORM) st_v4(sb + OFF_U + U_ULO + o, lo);
      }
      if constexpr (!L2NORM) {
        if (row >= 64) {  // P lo residual from Sqk, still resident in TMEM
          float kq[32];
          tmem_ld32(tl + TM_KQ + 32u * half, kq);
          tmem_wait_ld();
          write_p(kq, true);
        } else {
          float kq[32];  // keep the warp-collective load uniform across warps
          tmem_ld32(tl + TM_KQ + 32u * half, kq);
          tmem_wait_ld();
        }
      }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();

    // (9) dS = U~^T K (hi + lo);  O^T += U_hi^T P^T
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
          umma_bf16(tmem + TM_OT, umma_desc_k(ua + 32u * ks), umma_desc_k(pb + 32u * ks), id_p, 1);
      }
      umma_commit(bar_mma);
    }
    mma_pending = true;
    if (!cta_wait(bar_mma, ph_mma, ERR_MMA_TIMEOUT)) { ok = false; break; }
    ph_mma ^= 1;
    mma_pending = false;
    tc_fence_after();

    // (10) S <- G S + dS ; O^T -> staging [t][v] bf16 ; new S hi/lo
    {
      const float G = expf(Lam[63]);
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        float dv[32];
        tmem_ld32(tl + TM_DS + 64u * half + 32u * part, dv);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[32 * part + i] = fmaf(G, s[32 * part + i], dv[i]);
      }
      float ov[32];
      tmem_ld32(tl + TM_OT + 32u * half, ov);
      tmem_wait_ld();
      __nv_bfloat16* ostage = reinterpret_cast<__nv_bfloat16*>(smem + OFF_V);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        ostage[(32 * half + i) * kHeadDim + row] = __float2bfloat16_rn(scale * ov[i]);
      if (c + 1 < nchunks) write_state_split();
    }
    tc_fence_before();
    __syncthreads();
    // coalesced output rows (t < Lc): 16 x 16-byte pieces per 256-byte row
    {
      __nv_bfloat16* obase = p.out + ((size_t)t0 * HV + h) * kHeadDim;
      for (int u = tid; u < Lc * 16; u += kThreads) {
        const int t = u >> 4, ch = u & 15;
        const uint4 v4 = ld_shared_v4(sb + OFF_V + 256u * t + 16u * ch);
        *reinterpret_cast<uint4*>(obase + (size_t)t * HV * kHeadDim + 8 * ch) = v4;
      }
    }
  }

  if (ok) {
#pragma unroll
    for (int i = 0; i < 16; ++i)
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
  ChunkedParams cp{static_cast<const __nv_bfloat16*>(p.a), static_cast<const __nv_bfloat16*>(p.b),
                   p.A_log, p.dt_bias, p.cu, p.state, p.new_state,
                   static_cast<__nv_bfloat16*>(p.out), p.T, p.cu_int64 ? 1 : 0, p.HV,
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
