// GDN prefill, split form for sm_100a: a chunk-parallel preparation kernel and a
// sequential state kernel split over v-blocks.
//
// Same algebra as the fused chunked kernel (reference gdn_prefill/solution/triton/
// kernel.py:60-79, regrouped per chunk of C = 64 tokens), with k-last state S[v, k]:
//
//   A[t,j] = beta_t exp(Lam_t - Lam_j) rk_t rk_j (k_t . k_j)   j < t,   T = (I + A)^-1
//   P[t,j] = exp(Lam_t - Lam_j) rq_t rk_j (q_t . k_j)          j <= t
//   R      = diag(beta) (V - diag(gamma rk) K S^T)
//   U      = T R,   O = scale diag(gamma rq) Q S^T + scale (P T) R
//   S     <- G S + U~^T K,  U~ = diag(rk exp(Lam_end - Lam_t)) U,  G = exp(Lam_end)
//
// Everything that does not depend on the state -- the gates, the q/k norms, A, the
// triangular inverse T and the product P T -- is computed for every chunk of every
// sequence at once by the preparation kernel (one CTA per (chunk, v-head), three
// CTAs per SM), which stores a record per (chunk, v-head):
//
//   [T; P T]: a 128 x 64 bf16 tile in the 128-byte-swizzled K-major image the
//       tensor cores read (rows 0..63 T, rows 64..127 P T), and the lo image of T
//       (T = hi + lo; P T only feeds the output and is rounded to bf16);
//   beta, gamma rk, us = rk exp(Lam_end - Lam), scale gamma rq (64 fp32 each), G.
//
// The state recurrence is separable in v (row v of S only ever meets column v of
// V, U and O), so the sequential kernel runs one CTA per (sequence, v-head,
// 32-row v-block).  It keeps S^T[k][v] (fp32) in TMEM and per chunk issues three
// M = 128 MMA groups:
//   G1  [K; Q] S^T              -> rows 0..63 K S^T, rows 64..127 Q S^T  (S hi + S lo)
//   G2  [T; P T] R              -> rows 0..63 U,     rows 64..127 P U    ((hi + lo)(hi + lo))
//   G3  S^T += K^T U~                                                    (U~ hi + lo)
// each split operand read as one N = 64 tile [hi | lo] into two accumulator halves.
// Warp 16 issues the MMAs, warp 17 the copies, and warps 0..15 the TMEM epilogues;
// they hand over through mbarriers.
// with the R / U~ / output / state epilogues on the CUDA cores.  The next two
// chunks' K/Q tiles, V block and record are in flight while a chunk is processed.
//
// Every wait is bounded: a wait that runs out sets a device error flag (read by
// gdn_device_error), lets its copies and MMAs in flight land (again boundedly),
// releases TMEM and returns.
#include <cudaTypedefs.h>
#include <algorithm>
#include <climits>
#include <cmath>
#include <mutex>

#include "gdn_chunk_math.cuh"
#include "gdn_common.cuh"
#include "gdn_lpt.cuh"
#include "gdn_prefill.cuh"
#include "sm100.cuh"

namespace gdn {

__device__ unsigned int g_split_device_error = 0;

namespace {
using namespace sm100;
using namespace cm;

constexpr int kC = 64;
enum : unsigned { ERR_TMA_TIMEOUT = 1u, ERR_MMA_TIMEOUT = 2u, ERR_SMEM_ALIGN = 4u };

// ---- per (chunk, v-head) record
//   [0, 16 KB)   hi image of [T; P T] (rows 0..63 T, rows 64..127 P T)
//   [16 KB, ..)  lo image: rows 0..63 (T) with normalised q/k, where P T only
//                feeds the bf16 output and is rounded to bf16; all 128 rows with
//                raw q/k, whose P T entries span a far wider range
//   then         beta | gamma rk | us | scale gamma rq (4 x 64 f32), G, pad (1040 B)
constexpr uint32_t kRecTpHi = 0, kRecTpLo = 16384;
constexpr uint32_t kRecVecBytes = 1040;
__host__ __device__ constexpr uint32_t rec_lo_bytes(bool l2) { return l2 ? 8192u : 16384u; }
__host__ __device__ constexpr uint32_t rec_vec(bool l2) { return kRecTpLo + rec_lo_bytes(l2); }
__host__ __device__ constexpr uint32_t rec_bytes(bool l2) { return rec_vec(l2) + kRecVecBytes; }
constexpr size_t kRecBytesMax = rec_bytes(false);  // workspace sizing (16-byte multiple)

struct SplitParams {
  const __nv_bfloat16* a;
  const __nv_bfloat16* b;
  const float* A_log;
  const float* dt_bias;
  const void* cu;
  const float* state;
  float* new_state;
  __nv_bfloat16* out;
  const int* order;       // longest-first sequence order (null: natural order)
  const int* chunk_base;  // [N + 1] exclusive prefix of chunks per sequence
  uint8_t* rec;           // records, (chunk, v-head) major
  uint32_t rec_stride;    // bytes per record (rec_bytes(l2norm))
  uint32_t rec_lo;        // bytes of the record's lo image (rec_lo_bytes(l2norm))
  long long T;
  int N;
  int HV;
  int ratio;
  float scale;
  // precomputed gates (fp32 [T, HV] decay and beta, null = 1) instead of a / b
  bool gates_pre;
  const float* g_alpha;
  const float* g_beta;
  // state checkpoints every ckpt_every tokens (0 = off)
  float* ckpt;
  const long long* ckpt_starts;
  long long ckpt_cap;
  int ckpt_every;
  long long a_rs = 0, b_rs = 0, o_rs = 0;  // token strides of a, b and the output (elements)
  // segmented call of one sequence (token rows are virtual): rows r >= vsplit belong to the
  // identity runs, which read input row r - vsplit + vsrc, take v = 0, start from the
  // identity state and write their outputs to out_alt row r - vsplit; only runs
  // n < state_runs start from `state`, the others from zero
  long long vsplit = LLONG_MAX, vsrc = 0;
  __nv_bfloat16* out_alt = nullptr;
  int state_runs = INT_MAX;
  // records: only runs n < prep_runs are prepared; an identity run (rows >= vsplit) reads
  // the records of run n - rec_alias (the same tokens, hence the same records)
  int prep_runs = INT_MAX, rec_alias = 0;
  // an empty sequence passes its initial state through instead of ending at zero (the
  // second piece of a pipelined call, whose tokens may all lie in the first piece)
  bool empty_keeps_state = false;
};

// Input row of virtual token row r (a chunk never straddles vsplit).
__device__ __forceinline__ long long src_row(const SplitParams& p, long long r) {
  return r >= p.vsplit ? r - p.vsplit + p.vsrc : r;
}

template <typename CuT>
__device__ __forceinline__ void seq_range(const CuT* cu, int n, long long T, long long& s0,
                                          long long& s1) {
  s1 = min(max((long long)cu[n + 1], 0LL), T);
  s0 = min(max((long long)cu[n], 0LL), s1);
}

// All threads wait on `bar`; false on every thread if any thread's wait ran out.
__device__ __forceinline__ bool cta_wait(uint64_t* bar, uint32_t parity, unsigned code) {
  const bool ok = mbar_wait(bar, parity);
  const int bad = __syncthreads_or(ok ? 0 : 1);
  if (bad && threadIdx.x == 0) atomicOr(&g_split_device_error, code);
  return bad == 0;
}

// ------------------------------------------------------------ chunk offsets
// base[i] = number of 64-token chunks of sequences 0..i-1 (base[N] = total), one CTA.
template <typename CuT>
__global__ void __launch_bounds__(1024) chunk_base_kernel(const CuT* __restrict__ cu, int N,
                                                          long long T, int* __restrict__ base) {
  __shared__ int part[1024];
  const int tid = threadIdx.x;
  const int per = (N + 1023) / 1024;
  const int i0 = min(tid * per, N), i1 = min(i0 + per, N);
  auto nch = [&](int i) {
    long long s0, s1;
    seq_range(cu, i, T, s0, s1);
    return (int)((s1 - s0 + kC - 1) / kC);
  };
  int sum = 0;
  for (int i = i0; i < i1; ++i) sum += nch(i);
  part[tid] = sum;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const int add = tid >= off ? part[tid - off] : 0;
    __syncthreads();
    part[tid] += add;
    __syncthreads();
  }
  int run = part[tid] - sum;
  for (int i = i0; i < i1; ++i) {
    base[i] = run;
    run += nch(i);
  }
  if (tid == 1023) base[N] = part[1023];
}

// Token and chunk offsets of the two pieces of a pipelined one-sequence call: piece 1 is
// the sequence's first T1 tokens (or all of it), piece 2 the rest; out = [cu1 (2) | cu2 (2) |
// base1 (2) | base2 (2)].
template <typename CuT>
__global__ void piece_offsets_kernel(const CuT* __restrict__ cu, long long T, long long T1,
                                     int* __restrict__ out) {
  if (threadIdx.x != 0) return;
  const long long c1 = min(max((long long)cu[1], 0LL), T);
  const long long c0 = min(max((long long)cu[0], 0LL), c1);
  const long long m = min(c0 + T1, c1);
  out[0] = (int)c0;
  out[1] = (int)m;
  out[2] = (int)m;
  out[3] = (int)c1;
  out[4] = 0;
  out[5] = (int)((m - c0 + kC - 1) / kC);
  out[6] = 0;
  out[7] = (int)((c1 - m + kC - 1) / kC);
}

// ============================================================ preparation kernel
namespace prep {
constexpr int kThreads = 256;
constexpr uint32_t KQ = 0;        // K0 | Q0 | K1 | Q1 (8 KB each); then [P hi; P lo] (16 KB)
constexpr uint32_t TIMG = 32768;  // T hi | T lo, K-major [t][j] (8 KB each)
constexpr uint32_t AT = 49152;    // fp32 [64][kLd]: A, T in place, then (P lo T) partials
constexpr uint32_t E = AT + 64 * kLd * 4;  // merge scratch; before it the diagonal decay blocks
constexpr uint32_t ROWF = E + 64 * 20 * 4;  // fp32 [3][64]: exp(Lam_t - Lam_{16b+15}), b < t/16
constexpr uint32_t COLF = ROWF + 1024;      // fp32 [64]:    exp(Lam_{j|15} - Lam_j)
constexpr uint32_t VEC = COLF + 256;        // rk rq, then per v-head: Lam beta gam (64 f32 each)
constexpr uint32_t BARS = VEC + 8 * 256;
constexpr uint32_t SMEM = BARS + 64;
constexpr int kLdDE = 20;
constexpr uint32_t TKQ = 0, TPT = 64;  // TMEM columns (128 allocated)
static_assert(64 * 20 * 4 >= 32 * kLdE4 * 4, "merge scratch fits the decay table");
static_assert(3 * (SMEM + 1024) <= 233472, "three CTAs per SM");
}  // namespace prep

template <bool L2NORM, typename CuT>
__global__ void __launch_bounds__(prep::kThreads, 3)
    split_prep_kernel(const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k, const SplitParams p) {
  using namespace prep;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sb = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sp = warp & 3, half = warp >> 2;
  const int row = sp * 32 + lane;  // TMEM lane of this thread
  // One CTA per (chunk, pair of v-heads sharing a q/k head) when the GVA ratio is even
  // (one v-head otherwise): K/Q tiles, [K; Q] K^T and the norms serve both.
  const int hpc = (p.ratio % 2 == 0) ? 2 : 1;
  const int hgroups = p.HV / hpc;
  const int g = blockIdx.x / hgroups, h0 = (blockIdx.x - g * hgroups) * hpc;
  const int total = p.chunk_base[p.prep_runs < p.N ? p.prep_runs : p.N];
  if (g >= total) return;
  int lo = 0, hi = p.N - 1;  // the sequence of chunk g: largest n with base[n] <= g
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.chunk_base[mid] <= g) lo = mid; else hi = mid - 1;
  }
  const int n = lo, c = g - p.chunk_base[n];
  long long s0, s1;
  seq_range(static_cast<const CuT*>(p.cu), n, p.T, s0, s1);
  const long long tv = s0 + (long long)kC * c;  // virtual row of the chunk's first token
  const int Lc = (int)min((long long)kC, s1 - tv);
  const long long t0 = src_row(p, tv);           // its input row
  const int qh = h0 / p.ratio;
  if ((sb & 1023u) != 0) {
    if (tid == 0) atomicOr(&g_split_device_error, ERR_SMEM_ALIGN);
    return;
  }
  float* rk = reinterpret_cast<float*>(smem + VEC);
  float* rq = rk + 64;
  auto head_vec = [&](int i) { return rk + 128 + 192 * i; };  // Lam | beta | gam of head i
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BARS);  // kqtma, kq, pt
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + BARS + 32);
  if (warp == 0) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < 3; ++i) mbar_init(bars + i, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tl = tmem + ((uint32_t)(32 * sp) << 16);
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], 4 * 8192);
    tma_load_2d(smem + KQ, &tm_k, &bars[0], qh * 128, (int)t0);
    tma_load_2d(smem + KQ + 16384, &tm_k, &bars[0], qh * 128 + 64, (int)t0);
    tma_load_2d(smem + KQ + 8192, &tm_q, &bars[0], qh * 128, (int)t0);
    tma_load_2d(smem + KQ + 24576, &tm_q, &bars[0], qh * 128 + 64, (int)t0);
  }
  if (warp >= 1 && warp <= hpc) {  // gates of head warp - 1: cumulative log decay, beta, gamma
    const int h = h0 + warp - 1;
    float* Lam = head_vec(warp - 1);
    float* beta = Lam + 64;
    float* gam = Lam + 128;
    float lg[2], bb[2];
    if (p.gates_pre) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = 2 * lane + e;
        const bool valid = t < Lc;
        const size_t ti = (size_t)(t0 + (valid ? t : 0)) * p.HV + h;
        lg[e] = valid ? log_alpha(p.g_alpha ? __ldg(p.g_alpha + ti) : 1.f) : 0.f;
        bb[e] = valid ? (p.g_beta ? __ldg(p.g_beta + ti) : 1.f) : 0.f;
      }
    } else {
      const float nexpA = -expf(__ldg(p.A_log + h));
      const float dtb = __ldg(p.dt_bias + h);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = 2 * lane + e;
        const bool valid = t < Lc;
        const size_t tok = (size_t)(t0 + (valid ? t : 0));
        lg[e] = valid ? nexpA * softplus_f(bf2f(p.a[tok * p.a_rs + h]) + dtb) : 0.f;
        bb[e] = valid ? sigmoid_f(bf2f(p.b[tok * p.b_rs + h])) : 0.f;
      }
    }
    float x = lg[0] + lg[1];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    const float x0 = x - lg[1];
    Lam[2 * lane] = x0;
    Lam[2 * lane + 1] = x;
    beta[2 * lane] = bb[0];
    beta[2 * lane + 1] = bb[1];
    gam[2 * lane] = expf(x0);
    gam[2 * lane + 1] = expf(x);
  }
  bool ok = true;
  uint64_t* pend = nullptr;  // copy or MMA group in flight
  uint32_t pend_par = 0;
  do {
    pend = &bars[0];
    if (!(ok = cta_wait(&bars[0], 0, ERR_TMA_TIMEOUT))) break;
    pend = nullptr;
    if (tid == 0) {  // [Skk; Sqk] = [K; Q] K^T
      tc_fence_after();
      const uint32_t idesc = umma_idesc_bf16(128, 64, false, false);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t off = 16384u * (ks >> 2) + 32u * (ks & 3);
        const uint64_t kd = umma_desc_k(sb + KQ + off);
        umma_bf16(tmem + TKQ, kd, kd, idesc, ks > 0);
      }
      umma_commit(&bars[1]);
    }
    pend = &bars[1];
    if constexpr (L2NORM) {
      if (tid >= 64 && tid < 192) {  // q/k row norms
        const int t = tid & 63;
        const bool isq = tid < 128;
        const uint32_t b0 = sb + KQ + (isq ? 8192u : 0u) + 128u * t;
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
    } else {
      if (tid < 64) {
        rk[tid] = 1.f;
        rq[tid] = 1.f;
      }
    }
    if (!(ok = cta_wait(&bars[1], 0, ERR_MMA_TIMEOUT))) break;  // also orders the norms
    pend = nullptr;
    for (int hi = 0; hi < hpc && ok; ++hi) {
    const int h = h0 + hi;
    uint8_t* rec = p.rec + ((size_t)g * p.HV + h) * rec_bytes(L2NORM);
    const float* Lam = head_vec(hi);
    const float* beta = Lam + 64;
    const float* gam = Lam + 128;
    // decay factors exp(Lam_t - Lam_j), j <= t, with no positive exponent: directly
    // inside the diagonal 16x16 blocks; across blocks through the last token e of j's
    // block, exp(Lam_t - Lam_e) exp(Lam_e - Lam_j)
    {
      float* DE = reinterpret_cast<float*>(smem + E);
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4) {
        const int idx = tid + 256 * k4;
        const int blk = idx >> 8, r = (idx >> 4) & 15, jj = idx & 15;
        DE[(16 * blk + r) * kLdDE + jj] =
            (jj <= r) ? __expf(Lam[16 * blk + r] - Lam[16 * blk + jj]) : 0.f;
      }
      if (tid < 64) {
        float* RF = reinterpret_cast<float*>(smem + ROWF);
        reinterpret_cast<float*>(smem + COLF)[tid] = __expf(Lam[tid | 15] - Lam[tid]);
#pragma unroll
        for (int blk = 0; blk < 3; ++blk)
          RF[64 * blk + tid] = (16 * blk + 15 < tid) ? __expf(Lam[tid] - Lam[16 * blk + 15]) : 0.f;
      }
    }
    __syncthreads();
    tc_fence_after();
    // A (from Skk) -> AT; P (from Sqk) -> [P hi; P lo] image over the consumed K/Q tiles
    {
      const int t = row & 63, bt = t >> 4;
      const bool is_k = row < 64;
      const float ft = is_k ? beta[t] * rk[t] : rq[t];
      const float* DE = reinterpret_cast<const float*>(smem + E) + t * kLdDE;
      const float* RF = reinterpret_cast<const float*>(smem + ROWF);
      const float* CF = reinterpret_cast<const float*>(smem + COLF);
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int j0 = 32 * half + 16 * pass, bj = j0 >> 4;
        float ej[16];
        if ((t | 31) < j0) {  // whole warp above the diagonal (warp-uniform)
#pragma unroll
          for (int i = 0; i < 16; ++i) ej[i] = 0.f;
        } else {
          float kq[16], rv[16], fv[16];
          tmem_ld16(tl + TKQ + (uint32_t)j0, kq);
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
            *reinterpret_cast<float4*>(Arow + i) = make_float4(ej[i], ej[i + 1], ej[i + 2], ej[i + 3]);
        } else {
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            uint4 phi, plo;
            split8(&ej[8 * q2], phi, plo);
            st_v4(sb + KQ + sw128(t, (j0 >> 3) + q2), phi);
            st_v4(sb + KQ + 8192u + sw128(t, (j0 >> 3) + q2), plo);
          }
        }
      }
    }
    __syncthreads();
    if (tid < 64) {  // the record's row vectors
      float* rv = reinterpret_cast<float*>(rec + rec_vec(L2NORM));
      const int t = tid;
      const float lend = Lam[63];
      rv[t] = beta[t];
      rv[64 + t] = gam[t] * rk[t];
      rv[128 + t] = (t < Lc) ? rk[t] * expf(lend - Lam[t]) : 0.f;
      rv[192 + t] = default_scale(p.scale) * gam[t] * rq[t];
      if (t < 4) rv[256 + t] = (t == 0) ? expf(lend) : 0.f;
    }
    invert_in_place<1>(reinterpret_cast<float*>(smem + AT), reinterpret_cast<float*>(smem + E), tid);
    // T -> hi/lo: the B operand of P T here, rows 0..63 of the record
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2) {
      const int unit = tid + 256 * k2;
      const int t = unit >> 3, cidx = unit & 7;
      const float* tr = reinterpret_cast<const float*>(smem + AT) + t * kLd + 8 * cidx;
      const float4 ta = *reinterpret_cast<const float4*>(tr);
      const float4 tb = *reinterpret_cast<const float4*>(tr + 4);
      const float tv[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
      uint4 thi, tlo;
      split8(tv, thi, tlo);
      const uint32_t o = sw128(t, cidx);
      st_v4(sb + TIMG + o, thi);
      st_v4(sb + TIMG + 8192u + o, tlo);
      *reinterpret_cast<uint4*>(rec + kRecTpHi + o) = thi;
      *reinterpret_cast<uint4*>(rec + kRecTpLo + o) = tlo;
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // [P hi; P lo] T  (T hi + T lo; B = T as MN-major [s][j])
      tc_fence_after();
      const uint32_t idesc = umma_idesc_bf16(128, 64, false, true);
#pragma unroll
      for (int term = 0; term < 2; ++term)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tmem + TPT, umma_desc_k(sb + KQ + 32u * ks),
                    umma_desc_mn(sb + TIMG + 8192u * term + 2048u * ks, 8192), idesc,
                    (term | ks) != 0);
      umma_commit(&bars[2]);
    }
    pend = &bars[2];
    pend_par = hi & 1;
    if (!(ok = cta_wait(&bars[2], hi & 1, ERR_MMA_TIMEOUT))) break;
    pend = nullptr;
    tc_fence_after();
    // P T = (P hi T) + (P lo T): lanes 64..127 hand their part over through AT
    if (sp >= 2) {
      float v[32];
      tmem_ld32(tl + TPT + 32u * half, v);
      tmem_wait_ld();
      float* dst = reinterpret_cast<float*>(smem + AT) + (row - 64) * kLd + 32 * half;
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
    __syncthreads();
    if (sp < 2) {
      float v[32];
      tmem_ld32(tl + TPT + 32u * half, v);
      tmem_wait_ld();
      const float* src = reinterpret_cast<const float*>(smem + AT) + row * kLd + 32 * half;
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(src + i);
        v[i] += a4.x; v[i + 1] += a4.y; v[i + 2] += a4.z; v[i + 3] += a4.w;
      }
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const float* x = &v[8 * q4];
        const uint32_t o = sw128(64 + row, 4 * half + q4);
        if constexpr (L2NORM) {
          *reinterpret_cast<uint4*>(rec + kRecTpHi + o) =
              make_uint4(cvt_bf16x2(x[0], x[1]), cvt_bf16x2(x[2], x[3]), cvt_bf16x2(x[4], x[5]),
                         cvt_bf16x2(x[6], x[7]));
        } else {
          uint4 xhi, xlo;
          split8(x, xhi, xlo);
          *reinterpret_cast<uint4*>(rec + kRecTpHi + o) = xhi;
          *reinterpret_cast<uint4*>(rec + kRecTpLo + o) = xlo;
        }
      }
    }
    // the next head reuses AT, the P image and the P T columns
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    }  // per v-head
  } while (0);
  if (!ok && tid == 0 && pend != nullptr) {  // let the copy / MMA in flight land
    mbar_wait(pend, pend_par, 1u << 20);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// ============================================================ sequential state kernel
namespace st {
constexpr int kCompute = 512;             // warps 0..15: TMEM epilogues on the CUDA cores
constexpr int kMmaWarp = kCompute / 32;   // warp 16 issues the MMA groups
constexpr int kTmaWarp = kMmaWarp + 1;    // warp 17 issues the copies
constexpr int kThreads = kCompute + 64;
constexpr int kVB = 32;                   // v-rows per CTA (four CTAs per v-head)
constexpr int kSplitV = kHeadDim / kVB;
constexpr uint32_t KQ0 = 0, KQ1 = 32768;  // K0 | Q0 | K1 | Q1 (8 KB each), per buffer
constexpr uint32_t TP0 = 65536, TP1 = 98304;  // record tiles: hi (16 KB) | lo (16 KB; rows
                                              // 64..127 stay zero), per buffer
// MMA B images, 128-byte rows [hi (32 v) | lo (32 v)] in the 128-byte swizzle, MN-major:
constexpr uint32_t SIMG = 131072;  // S [k][v]   (G1)
constexpr uint32_t RIMG = 147456;  // R [j][v]   (G2)
constexpr uint32_t UIMG = 155648;  // U~ [t][v]  (G3)
constexpr uint32_t V0 = 163840, V1 = 167936;  // V block [t][32 v], 64-byte rows, per buffer
constexpr uint32_t VEC0 = 172032, VEC1 = 173312;  // record vectors (1040 B), per buffer
constexpr uint32_t BARS = 174592;
constexpr uint32_t SMEM = BARS + 256;
// TMEM columns (256 allocated).  Each MMA reads its split operand as one N = 64 B
// tile [hi | lo], so each D tile holds two 32-column halves whose sum is the product:
//   TST: state S^T = (cols 0..31) + (cols 32..63), both decayed; G3 adds U~ hi / U~ lo
//   TG1: [K; Q] S_hi^T | [K; Q] S_lo^T       TG2: [T; P T] R_hi | [T; P T] R_lo
constexpr uint32_t TST = 0, TG1 = 64, TG2 = 128;
static_assert(SMEM <= 232448, "shared memory budget");
struct Bars {
  uint64_t kq[2], vt[2];          // copies landed (transaction counts)
  uint64_t kq_free[2], vt_free[2];  // buffers consumed (MMA commit / + 16 compute warps)
  uint64_t g1, g2, g3;            // MMA groups completed (commit)
  uint64_t s_ready;               // 16 compute warps: S images written
  uint64_t r_ready, u_ready;      // 8 warps of TMEM lanes 0..63: R / U~ images written
  uint64_t o_done;                // 8 warps of TMEM lanes 64..127: outputs read out
};

// Bounded wait that gives up early once another thread has aborted; a wait that
// runs out records `code` and raises the abort flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity,
                                              volatile int* abort_flag, unsigned code) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort_flag) return false;
  }
  atomicOr(&g_split_device_error, code);
  *abort_flag = 1;
  return false;
}
// One arrival per warp, after every lane's shared-memory and TMEM accesses are
// ordered for the async proxy / tensor cores.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  fence_proxy_async();
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}
// 8 fp32 values of columns 8q.. -> row r of a [hi | lo] image: hi in 16-byte chunk q,
// lo in chunk 4 + q (128-byte swizzle).
__device__ __forceinline__ void store_split8(uint32_t base, int r, int q, const float* x) {
  uint4 xhi, xlo;
  split8(x, xhi, xlo);
  st_v4(base + sw128(r, q), xhi);
  st_v4(base + sw128(r, 4 + q), xlo);
}
}  // namespace st

template <bool HAS_STATE, typename CuT>
__global__ void __launch_bounds__(st::kThreads, 1)
    split_state_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const SplitParams p) {
  using namespace st;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sb = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sp = warp & 3, qc = (warp >> 2) & 3;  // TMEM lane quarter, 16-column quarter
  const int row = sp * 32 + lane;  // TMEM lane: k for the state, token for G1 / G2 rows
  const int HV = p.HV;
  const int per = kSplitV * HV;
  const int wi = blockIdx.x / per;
  const int rem = blockIdx.x - wi * per;
  const int h = rem / kSplitV, vb = rem % kSplitV;
  const int n = p.order ? p.order[wi] : wi;
  const int qh = h / p.ratio;
  long long s0, s1;
  seq_range(static_cast<const CuT*>(p.cu), n, p.T, s0, s1);
  const long long L = s1 - s0;
  // a compute thread's state elements: S[v][k], k = row, v = v_lo + i (i < 8)
  const int vq = 8 * qc;  // column offset inside the v-block
  const int v_lo = kVB * vb + vq;
  float* ns = p.new_state + ((size_t)n * HV + h) * kHeadDim * kHeadDim;
  if (L <= 0) {  // empty sequence: zero final state (definition semantics)
    if (tid < kCompute) {
      const float* src = p.state + ((size_t)n * HV + h) * kHeadDim * kHeadDim;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        ns[(size_t)(v_lo + i) * kHeadDim + row] =
            (HAS_STATE && p.empty_keeps_state) ? src[(size_t)(v_lo + i) * kHeadDim + row] : 0.f;
    }
    return;
  }
  if ((sb & 1023u) != 0) {
    if (tid == 0) atomicOr(&g_split_device_error, ERR_SMEM_ALIGN);
    return;
  }
  const int nchunks = (int)((L + kC - 1) / kC);
  const bool ident = s0 >= p.vsplit;  // identity run of a segmented call: v = 0, no V copies
  if (ident) {
    for (int i = tid; i < (int)((V1 + 4096u - V0) / 16u); i += kThreads)
      st_shared_v4(sb + V0 + 16u * (uint32_t)i, 0u, 0u, 0u, 0u);
  }
  Bars* bars = reinterpret_cast<Bars*>(smem + BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + BARS + sizeof(Bars));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + BARS + sizeof(Bars) + 4);
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(&bars->kq[0], 1);
    mbar_init(&bars->kq[1], 1);
    mbar_init(&bars->vt[0], 1);
    mbar_init(&bars->vt[1], 1);
    mbar_init(&bars->kq_free[0], 1);
    mbar_init(&bars->kq_free[1], 1);
    mbar_init(&bars->vt_free[0], kCompute / 32 + 1);
    mbar_init(&bars->vt_free[1], kCompute / 32 + 1);
    mbar_init(&bars->g1, 1);
    mbar_init(&bars->g2, 1);
    mbar_init(&bars->g3, 1);
    mbar_init(&bars->s_ready, kCompute / 32);
    mbar_init(&bars->r_ready, kCompute / 64);
    mbar_init(&bars->u_ready, kCompute / 64);
    mbar_init(&bars->o_done, kCompute / 64);
    *abort_flag = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  int kq_issued = 0, vt_issued = 0;  // copy warp: chunks whose copies were issued
  uint64_t* mma_bar = nullptr;       // MMA warp: group in flight when a wait ran out
  uint32_t mma_par = 0;

  if (warp == kTmaWarp) {
    // =========================================================== copy warp
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const size_t rstride = (size_t)HV * p.rec_stride;
      const int nrec = ident ? n - p.rec_alias : n;  // the run whose records these are
      const uint8_t* rec0 = p.rec + ((size_t)p.chunk_base[nrec] * HV + h) * p.rec_stride;
      for (int cc = 0; cc < nchunks; ++cc) {
        const int bf = cc & 1;
        const uint32_t free_par = ((cc >> 1) + 1) & 1;  // phase cc/2 - 1 of the free barrier
        const int y = (int)src_row(p, s0 + (long long)kC * cc);
        if (cc >= 2 && !wait_or_abort(&bars->kq_free[bf], free_par, abort_flag, ERR_MMA_TIMEOUT))
          break;
        const uint32_t kq = bf ? KQ1 : KQ0;
        fence_proxy_async();
        mbar_arrive_expect_tx(&bars->kq[bf], 4 * 8192);
        tma_load_2d(smem + kq, &tm_k, &bars->kq[bf], qh * 128, y);
        tma_load_2d(smem + kq + 16384, &tm_k, &bars->kq[bf], qh * 128 + 64, y);
        tma_load_2d(smem + kq + 8192, &tm_q, &bars->kq[bf], qh * 128, y);
        tma_load_2d(smem + kq + 24576, &tm_q, &bars->kq[bf], qh * 128 + 64, y);
        kq_issued = cc + 1;
        if (cc >= 2 && !wait_or_abort(&bars->vt_free[bf], free_par, abort_flag, ERR_MMA_TIMEOUT))
          break;
        const uint8_t* r = rec0 + (size_t)cc * rstride;
        fence_proxy_async();
        mbar_arrive_expect_tx(&bars->vt[bf], (ident ? 0u : 64u * kVB * 2u) + p.rec_stride);
        if (!ident) tma_load_2d(smem + (bf ? V1 : V0), &tm_v, &bars->vt[bf], h * 128 + kVB * vb, y);
        bulk_load(smem + (bf ? TP1 : TP0), r, kRecTpLo + p.rec_lo, &bars->vt[bf]);  // hi | lo
        bulk_load(smem + (bf ? VEC1 : VEC0), r + kRecTpLo + p.rec_lo, kRecVecBytes, &bars->vt[bf]);
        vt_issued = cc + 1;
      }
    }
  } else if (warp == kMmaWarp) {
    // =========================================================== MMA warp
    if (lane == 0) {
      const uint32_t id_nn = umma_idesc_bf16(128, 64, false, true);  // A K-major, B MN-major
      const uint32_t id_mm = umma_idesc_bf16(128, 64, true, true);   // A and B MN-major
      bool ok = true;
      for (int c = 0; c < nchunks && ok; ++c) {
        const int bf = c & 1;
        const uint32_t par = c & 1, par2 = (c >> 1) & 1;
        const uint32_t kqb = bf ? KQ1 : KQ0, tpb = bf ? TP1 : TP0;
        if (!(ok = wait_or_abort(&bars->kq[bf], par2, abort_flag, ERR_TMA_TIMEOUT))) break;
        if (!(ok = wait_or_abort(&bars->vt[bf], par2, abort_flag, ERR_TMA_TIMEOUT))) break;
        if (!(ok = wait_or_abort(&bars->s_ready, par, abort_flag, ERR_MMA_TIMEOUT))) break;
        if (c > 0 && !(ok = wait_or_abort(&bars->o_done, par ^ 1u, abort_flag, ERR_MMA_TIMEOUT)))
          break;
        tc_fence_after();
        // G1: [K; Q] [S_hi | S_lo]^T
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_bf16(tmem + TG1, umma_desc_k(sb + kqb + 16384u * (ks >> 2) + 32u * (ks & 3)),
                    umma_desc_mn(sb + SIMG + 2048u * ks, 8192), id_nn, ks > 0);
        umma_commit(&bars->g1);
        mma_bar = &bars->g1;
        mma_par = par;
        if (!(ok = wait_or_abort(&bars->r_ready, par, abort_flag, ERR_MMA_TIMEOUT))) break;
        tc_fence_after();
        // G2: ([T; P T] hi + lo) [R_hi | R_lo]
#pragma unroll
        for (int term = 0; term < 2; ++term)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16(tmem + TG2, umma_desc_k(sb + tpb + 16384u * term + 32u * ks),
                      umma_desc_mn(sb + RIMG + 2048u * ks, 8192), id_nn, (term | ks) != 0);
        umma_commit(&bars->g2);
        umma_commit(&bars->vt_free[bf]);  // record tiles consumed once G2 completes
        mma_bar = &bars->g2;
        if (!(ok = wait_or_abort(&bars->u_ready, par, abort_flag, ERR_MMA_TIMEOUT))) break;
        tc_fence_after();
        // G3: S^T += K^T [U~_hi | U~_lo]  (A = K tile as MN-major [t][k])
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tmem + TST, umma_desc_mn(sb + kqb + 2048u * ks, 16384),
                    umma_desc_mn(sb + UIMG + 2048u * ks, 8192), id_mm, 1);
        umma_commit(&bars->g3);
        umma_commit(&bars->kq_free[bf]);  // K (G3) and Q (G1) consumed once G3 completes
        mma_bar = &bars->g3;
      }
      if (ok) {
        // the buffer-free arrivals of the last two chunks are waited by nobody else:
        // let them land before the CTA's shared memory is released
        mma_bar = nullptr;
        for (int c = max(nchunks - 2, 0); c < nchunks; ++c) {
          mbar_wait(&bars->kq_free[c & 1], (c >> 1) & 1, 1u << 20);
          mbar_wait(&bars->vt_free[c & 1], (c >> 1) & 1, 1u << 20);
        }
      }
    }
  } else {
    // =========================================================== compute warps
    const uint32_t tl = tmem + ((uint32_t)(32 * sp) << 16);
    const float scale = default_scale(p.scale);
    // records without a P T lo part: rows 64..127 of both lo tiles stay zero
    if (p.rec_lo < 16384u) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint32_t a = (i ? TP1 : TP0) + 16384u + 8192u + 16u * (uint32_t)tid;
        st_shared_v4(sb + a, 0u, 0u, 0u, 0u);
      }
    }
    // initial state: S^T[k][v] -> TMEM (fp32; second half 0) and G1's [hi | lo] image
    {
      float sv[8];
      bool loaded = false;
      if constexpr (HAS_STATE) {
        if (n < p.state_runs) {
          const float* src = p.state + ((size_t)n * HV + h) * kHeadDim * kHeadDim;
#pragma unroll
          for (int i = 0; i < 8; ++i) sv[i] = __ldg(src + (size_t)(v_lo + i) * kHeadDim + row);
          loaded = true;
        }
      }
      if (!loaded) {  // zero, or the identity for an identity run (S^T[k][v] = [k == v])
#pragma unroll
        for (int i = 0; i < 8; ++i) sv[i] = (ident && v_lo + i == row) ? 1.f : 0.f;
      }
      const float zero[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      tmem_st8(tl + TST + vq, sv);
      tmem_st8(tl + TST + 32u + vq, zero);
      store_split8(sb + SIMG, row, qc, sv);
      tmem_wait_st();
      warp_arrive(&bars->s_ready);
    }
    for (int c = 0; c < nchunks; ++c) {
      const int bf = c & 1;
      const uint32_t par = c & 1, par2 = (c >> 1) & 1;
      const long long t0 = s0 + (long long)kC * c;
      const int Lc = (int)min((long long)kC, s1 - t0);
      const float* vec = reinterpret_cast<const float*>(smem + (bf ? VEC1 : VEC0));
      if (!wait_or_abort(&bars->vt[bf], par2, abort_flag, ERR_TMA_TIMEOUT)) break;
      {  // decay both halves of the fp32 state while G1 runs (G3 accumulates onto them)
        const float G = vec[256];
        float sa[8], sc[8];
        tmem_ld8(tl + TST + vq, sa);
        tmem_ld8(tl + TST + 32u + vq, sc);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          sa[i] *= G;
          sc[i] *= G;
        }
        tmem_st8(tl + TST + vq, sa);
        tmem_st8(tl + TST + 32u + vq, sc);
        tmem_wait_st();
      }
      // this thread's V slice and vectors, read while G1 runs
      const int rr = sp < 2 ? row : row - 64;
      const float bj = vec[rr], cj = vec[64 + rr], ut = vec[128 + rr], ct = vec[192 + rr];
      const uint4 va = ld_shared_v4(sb + (bf ? V1 : V0) + rr * (2 * kVB) + 16 * qc);
      if (!wait_or_abort(&bars->g1, par, abort_flag, ERR_MMA_TIMEOUT)) break;
      tc_fence_after();
      if (sp < 2) {
        // R[j][v] = beta_j (V[j][v] - gamma_j rk_j (K S^T)[j][v])  (j = row)
        float sk[8], sk2[8];
        tmem_ld8(tl + TG1 + vq, sk);
        tmem_ld8(tl + TG1 + 32u + vq, sk2);
        tmem_wait_ld();
        const uint32_t vw[4] = {va.x, va.y, va.z, va.w};
        float x[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = bf2x2_to_f2(vw[e]);
          x[2 * e] = bj * (f.x - cj * (sk[2 * e] + sk2[2 * e]));
          x[2 * e + 1] = bj * (f.y - cj * (sk[2 * e + 1] + sk2[2 * e + 1]));
        }
        store_split8(sb + RIMG, row, qc, x);
        warp_arrive(&bars->r_ready);
        if (!wait_or_abort(&bars->g2, par, abort_flag, ERR_MMA_TIMEOUT)) break;
        tc_fence_after();
        // U~ = diag(us) U -> [hi | lo] image [t][v]
        float uv[8], uv2[8];
        tmem_ld8(tl + TG2 + vq, uv);
        tmem_ld8(tl + TG2 + 32u + vq, uv2);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = ut * (uv[i] + uv2[i]);
        store_split8(sb + UIMG, row, qc, x);
        warp_arrive(&bars->u_ready);
      } else {
        // O = scale gamma rq (Q S^T) + scale (P T) R  (t = row - 64)
        if (!wait_or_abort(&bars->g2, par, abort_flag, ERR_MMA_TIMEOUT)) break;
        tc_fence_after();
        const int t = row - 64;
        float qs[8], q2[8], pu[8], p2[8];
        tmem_ld8(tl + TG1 + vq, qs);
        tmem_ld8(tl + TG1 + 32u + vq, q2);
        tmem_ld8(tl + TG2 + vq, pu);
        tmem_ld8(tl + TG2 + 32u + vq, p2);
        tmem_wait_ld();
        warp_arrive(&bars->o_done);  // TG1 / TG2 read out: the next G1 / G2 may overwrite
        if (t < Lc) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = 2 * e;
            w[e] = cvt_bf16x2(ct * (qs[i] + q2[i]) + scale * (pu[i] + p2[i]),
                              ct * (qs[i + 1] + q2[i + 1]) + scale * (pu[i + 1] + p2[i + 1]));
          }
          __nv_bfloat16* orow = ident ? p.out_alt + (size_t)(t0 + t - p.vsplit) * p.o_rs
                                      : p.out + (size_t)(t0 + t) * p.o_rs;
          *reinterpret_cast<uint4*>(orow + (size_t)h * kHeadDim + v_lo) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      warp_arrive(&bars->vt_free[bf]);  // this warp's V / vector reads of buffer bf are done
      if (!wait_or_abort(&bars->g3, par, abort_flag, ERR_MMA_TIMEOUT)) break;
      tc_fence_after();
      // epilogue: S^T -> next chunk's [hi | lo] image, or the final state
      {
        float sv[8], s2[8];
        tmem_ld8(tl + TST + vq, sv);
        tmem_ld8(tl + TST + 32u + vq, s2);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i) sv[i] += s2[i];
        if (p.ckpt != nullptr) {  // state checkpoint after this chunk, when one is due
          const long long ci = checkpoint_slot(p.ckpt_starts, n, min((long long)kC * (c + 1), L),
                                               p.ckpt_every, p.ckpt_cap);
          if (ci >= 0) {
            float* cp = p.ckpt + ((size_t)ci * HV + h) * kHeadDim * kHeadDim;
#pragma unroll
            for (int i = 0; i < 8; ++i) cp[(size_t)(v_lo + i) * kHeadDim + row] = sv[i];
          }
        }
        if (c + 1 == nchunks) {
#pragma unroll
          for (int i = 0; i < 8; ++i) ns[(size_t)(v_lo + i) * kHeadDim + row] = sv[i];
        } else {
          store_split8(sb + SIMG, row, qc, sv);
          warp_arrive(&bars->s_ready);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {  // a wait ran out: copies and MMAs still in flight land first (bounded)
    if (warp == kTmaWarp && lane == 0) {
      for (int cc = max(kq_issued - 2, 0); cc < kq_issued; ++cc)
        mbar_wait(&bars->kq[cc & 1], (cc >> 1) & 1, 1u << 20);
      for (int cc = max(vt_issued - 2, 0); cc < vt_issued; ++cc)
        mbar_wait(&bars->vt[cc & 1], (cc >> 1) & 1, 1u << 20);
    }
    if (warp == kMmaWarp && lane == 0 && mma_bar != nullptr) mbar_wait(mma_bar, mma_par, 1u << 20);
    __syncthreads();
  }
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ------------------------------------------------------------ host side
struct SplitLayout {
  size_t order, base, rec, total;
  long long slots;
};
SplitLayout split_layout(long long T, int N, int HV) {
  SplitLayout l{};
  const auto up = [](size_t x, size_t a) { return (x + a - 1) / a * a; };
  l.order = 0;
  l.base = up((size_t)N * sizeof(int), 256);
  l.rec = up(l.base + (size_t)(N + 1) * sizeof(int), 1024);
  l.slots = (T + kC - 1) / kC + N;
  l.total = l.rec + (size_t)l.slots * HV * kRecBytesMax;
  return l;
}

template <auto kern>
bool configure(uint32_t smem) {  // once per (kernel, device)
  static bool done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return true;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return false;
  // all of the unified L1 / shared storage as shared memory (the preparation kernel
  // relies on three CTAs per SM)
  if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return false;
  if (dev >= 0 && dev < 64) done[dev] = true;
  return true;
}

// ------------------------------------------------------------ pipelined one-sequence call
// One sequence whose state kernel leaves SMs idle (4 CTAs per v-head: 128 of 148 SMs for 32
// v-heads) runs as two pieces with the state carried between them, so that the second
// piece's preparation kernel runs on the idle SMs while the first piece's state kernel runs:
//   stream s:    offsets | prep(piece 1, whole GPU) | state(piece 1) ...... | state(piece 2)
//   side stream:                                    | prep(piece 2, idle SMs) |
// The state kernels launch at the highest stream priority and the side preparation at the
// lowest, so that the state kernel's CTAs take their SMs first.  The pieces meet on a
// 64-token chunk boundary and piece 1's fp32 final state is piece 2's initial state, so the
// results equal the one-piece call's bit for bit.  Piece 1's length balances its state
// kernel against piece 2's preparation on the idle SMs (measured on B200: ~2.15 us per
// state chunk step; ~16.3 us per preparation CTA at three per SM).
constexpr double kStateChunkUs = 2.15, kPrepCtaUs = 16.3;

size_t pipe_workspace(long long T, int HV) {
  // offsets | carried state | piece-1 layout | piece-2 layout (each 1024-aligned)
  const auto up = [](size_t x) { return (x + 1023) / 1024 * 1024; };
  return 1024 + up((size_t)HV * kHeadDim * kHeadDim * sizeof(float)) +
         up(split_layout(T, 1, HV).total) + (size_t)HV * kRecBytesMax + 2048;
}

struct PipeRes {
  bool tried = false, ok = false;
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  int prio_hi = 0, prio_lo = 0, sms = 0;
};
std::mutex g_pipe_mu;

// The side stream and events of the current device, created on its first pipelined call
// (null if they could not be created: the call then runs unpipelined).
PipeRes* pipe_res() {
  static PipeRes res[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  PipeRes& r = res[dev];
  std::lock_guard<std::mutex> g(g_pipe_mu);
  if (!r.tried) {
    r.tried = true;
    int least = 0, greatest = 0;
    r.ok = cudaDeviceGetStreamPriorityRange(&least, &greatest) == cudaSuccess &&
           cudaDeviceGetAttribute(&r.sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
           cudaStreamCreateWithPriority(&r.side, cudaStreamNonBlocking, least) == cudaSuccess &&
           cudaEventCreateWithFlags(&r.fork, cudaEventDisableTiming) == cudaSuccess &&
           cudaEventCreateWithFlags(&r.join, cudaEventDisableTiming) == cudaSuccess;
    r.prio_hi = greatest;
    r.prio_lo = least;
  }
  return r.ok ? &r : nullptr;
}

// Tokens of piece 1 (a multiple of 64), or 0 when the call should not be pipelined.
long long pipe_split(const PrefillArgs& p, int sms) {
  if (p.N != 1 || p.ckpt != nullptr || p.vsplit != LLONG_MAX || p.ready_base != nullptr ||
      p.ready_order != nullptr || p.src_rows > 0)
    return 0;
  const long long chunks = (p.T + kC - 1) / kC;
  const int idle = sms - p.HV * st::kSplitV;
  if (chunks < 64 || idle < 8) return 0;
  const int hpc = (p.HV / p.HQ) % 2 == 0 ? 2 : 1;
  const double prep_idle_us = (double)(p.HV / hpc) * kPrepCtaUs / (3.0 * idle);  // per chunk
  const double r = prep_idle_us / kStateChunkUs;
  const long long m = (long long)std::llround((double)chunks * r / (1.0 + r));
  if (m < 16 || m > chunks - 16) return 0;
  return kC * m;
}

template <auto kern, typename... Args>
cudaError_t launch_prio(dim3 grid, dim3 block, uint32_t smem, cudaStream_t s, int prio,
                        Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributePriority;
  attr[0].val.priority = prio;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <bool L2, bool HS>
cudaError_t launch_pipe_t(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                          const SplitParams& sp1, const SplitParams& sp2, long long slots1,
                          long long slots2, const PipeRes& r, cudaStream_t s) {
  constexpr auto ka = split_prep_kernel<L2, int>;
  constexpr auto kb1 = split_state_kernel<HS, int>;
  constexpr auto kb2 = split_state_kernel<true, int>;  // starts from piece 1's state
  if (!configure<ka>(prep::SMEM) || !configure<kb1>(st::SMEM) || !configure<kb2>(st::SMEM))
    return cudaErrorInvalidValue;
  const int hpc = (sp1.ratio % 2 == 0) ? 2 : 1;
  const dim3 sgrid((unsigned)(sp1.HV * st::kSplitV));
  cudaError_t e;
  ka<<<dim3((unsigned)(slots1 * (sp1.HV / hpc))), dim3(prep::kThreads), prep::SMEM, s>>>(mq, mk,
                                                                                        sp1);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if ((e = cudaEventRecord(r.fork, s)) != cudaSuccess) return e;
  if ((e = cudaStreamWaitEvent(r.side, r.fork, 0)) != cudaSuccess) return e;
  if ((e = launch_prio<kb1>(sgrid, dim3(st::kThreads), st::SMEM, s, r.prio_hi, mq, mk, mv,
                            sp1)) != cudaSuccess)
    return e;
  if ((e = launch_prio<ka>(dim3((unsigned)(slots2 * (sp2.HV / hpc))), dim3(prep::kThreads),
                           prep::SMEM, r.side, r.prio_lo, mq, mk, sp2)) != cudaSuccess)
    return e;
  if ((e = cudaEventRecord(r.join, r.side)) != cudaSuccess) return e;
  if ((e = cudaStreamWaitEvent(s, r.join, 0)) != cudaSuccess) return e;
  return launch_prio<kb2>(sgrid, dim3(st::kThreads), st::SMEM, s, r.prio_hi, mq, mk, mv, sp2);
}

template <bool L2, bool HS, typename CuT>
cudaError_t launch_split_t(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                           const SplitParams& sp, long long slots, bool base_ready,
                           cudaStream_t s) {
  constexpr auto ka = split_prep_kernel<L2, CuT>;
  constexpr auto kb = split_state_kernel<HS, CuT>;
  if (!configure<ka>(prep::SMEM) || !configure<kb>(st::SMEM)) return cudaErrorInvalidValue;
  cudaError_t e;
  if (!base_ready) {
    chunk_base_kernel<CuT><<<1, 1024, 0, s>>>(static_cast<const CuT*>(sp.cu), sp.N, sp.T,
                                              const_cast<int*>(sp.chunk_base));
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const int hpc = (sp.ratio % 2 == 0) ? 2 : 1;  // v-heads per preparation CTA
  ka<<<dim3((unsigned)(slots * (sp.HV / hpc))), dim3(prep::kThreads), prep::SMEM, s>>>(mq, mk,
                                                                                      sp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  kb<<<dim3((unsigned)((long long)sp.N * sp.HV * st::kSplitV)), dim3(st::kThreads), st::SMEM,
       s>>>(mq, mk, mv, sp);
  return cudaGetLastError();
}

template <typename CuT>
cudaError_t launch_split_cu(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                            const SplitParams& sp, bool l2, bool hs, long long slots,
                            bool base_ready, cudaStream_t s) {
  if (l2) return hs ? launch_split_t<true, true, CuT>(mq, mk, mv, sp, slots, base_ready, s)
                    : launch_split_t<true, false, CuT>(mq, mk, mv, sp, slots, base_ready, s);
  return hs ? launch_split_t<false, true, CuT>(mq, mk, mv, sp, slots, base_ready, s)
            : launch_split_t<false, false, CuT>(mq, mk, mv, sp, slots, base_ready, s);
}

}  // namespace

size_t prefill_split_workspace(long long T, int num_seqs, int HV) {
  if (T <= 0 || num_seqs <= 0) return 0;
  if (num_seqs == 1) return pipe_workspace(T, HV);  // room for a pipelined call
  return split_layout(T, num_seqs, HV).total;
}

namespace {
template <typename CuT>
cudaError_t launch_prefill_split_piped(const PrefillArgs& p, long long T1, const PipeRes& r,
                                       cudaStream_t s) {
  const auto up = [](size_t x) { return (x + 1023) / 1024 * 1024; };
  if (p.workspace == nullptr || p.workspace_bytes < pipe_workspace(p.T, p.HV))
    return cudaErrorInvalidValue;
  CUtensorMap mq, mk, mv;
  if (!make_tile_map(&mq, p.q, p.HQ, p.T, p.rs.q) || !make_tile_map(&mk, p.k, p.HQ, p.T, p.rs.k) ||
      !make_tile_map_box(&mv, p.v, p.HV, p.T, p.rs.v, st::kVB, false))
    return cudaErrorInvalidValue;
  uint8_t* ws = static_cast<uint8_t*>(p.workspace);
  int* offs = reinterpret_cast<int*>(ws);  // cu1 | cu2 | base1 | base2
  float* carried = reinterpret_cast<float*>(ws + 1024);  // piece 1's final state
  uint8_t* w1 = ws + 1024 + up((size_t)p.HV * kHeadDim * kHeadDim * sizeof(float));
  const SplitLayout l1 = split_layout(T1, 1, p.HV), l2 = split_layout(p.T - T1, 1, p.HV);
  uint8_t* w2 = w1 + up(l1.total);
  if ((size_t)(w2 - ws) + l2.total > p.workspace_bytes) return cudaErrorInvalidValue;
  piece_offsets_kernel<CuT><<<1, 32, 0, s>>>(static_cast<const CuT*>(p.cu), p.T, T1, offs);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  SplitParams sp1{static_cast<const __nv_bfloat16*>(p.a), static_cast<const __nv_bfloat16*>(p.b),
                  p.A_log, p.dt_bias, offs, p.state, carried,
                  static_cast<__nv_bfloat16*>(p.out), nullptr, offs + 4, w1 + l1.rec,
                  rec_bytes(p.l2norm), rec_lo_bytes(p.l2norm), p.T, 1, p.HV, p.HV / p.HQ,
                  p.scale, p.gates_pre, p.g_alpha, p.g_beta, nullptr, nullptr, 0, 0};
  sp1.a_rs = p.rs.a;
  sp1.b_rs = p.rs.b;
  sp1.o_rs = p.rs.o;
  SplitParams sp2 = sp1;
  sp2.cu = offs + 2;
  sp2.state = carried;
  sp2.new_state = p.new_state;
  sp2.chunk_base = offs + 6;
  sp2.rec = w2 + l2.rec;
  sp2.empty_keeps_state = true;
  const long long slots1 = T1 / kC + 1, slots2 = (p.T - T1 + kC - 1) / kC + 1;
  std::lock_guard<std::mutex> g(g_pipe_mu);  // the side stream and events serve one call at a time
  const bool hs = p.state != nullptr;
  if (p.l2norm) return hs ? launch_pipe_t<true, true>(mq, mk, mv, sp1, sp2, slots1, slots2, r, s)
                          : launch_pipe_t<true, false>(mq, mk, mv, sp1, sp2, slots1, slots2, r, s);
  return hs ? launch_pipe_t<false, true>(mq, mk, mv, sp1, sp2, slots1, slots2, r, s)
            : launch_pipe_t<false, false>(mq, mk, mv, sp1, sp2, slots1, slots2, r, s);
}
}  // namespace

cudaError_t launch_prefill_split(const PrefillArgs& p, cudaStream_t s) {
  if (p.N == 1 && p.ckpt == nullptr && p.vsplit == LLONG_MAX && p.ready_base == nullptr) {
    const PipeRes* r = pipe_res();
    const long long T1 = r != nullptr ? pipe_split(p, r->sms) : 0;
    if (T1 > 0)
      return p.cu_int64 ? launch_prefill_split_piped<long long>(p, T1, *r, s)
                        : launch_prefill_split_piped<int>(p, T1, *r, s);
  }
  const SplitLayout lay = split_layout(p.T, p.N, p.HV);
  if (p.workspace == nullptr || p.workspace_bytes < lay.total) return cudaErrorInvalidValue;
  if (lay.slots * p.HV > 0x7fffffffLL || (long long)p.N * p.HV * st::kSplitV > 0x7fffffffLL)
    return cudaErrorInvalidValue;
  CUtensorMap mq, mk, mv;  // V in [64 tokens][32 v] boxes, unswizzled (read by the CUDA cores)
  const long long rows = p.src_rows > 0 ? p.src_rows : p.T;  // rows of q, k, v
  if (!make_tile_map(&mq, p.q, p.HQ, rows, p.rs.q) || !make_tile_map(&mk, p.k, p.HQ, rows, p.rs.k) ||
      !make_tile_map_box(&mv, p.v, p.HV, rows, p.rs.v, st::kVB, false))
    return cudaErrorInvalidValue;
  uint8_t* ws = static_cast<uint8_t*>(p.workspace);
  int* order = const_cast<int*>(p.ready_order);
  if (order == nullptr && p.N > 1 && p.N <= kLptMaxSeqs) {
    order = reinterpret_cast<int*>(ws + lay.order);
    int P = 1;
    while (P < p.N) P <<= 1;
    const size_t sm = (size_t)P * sizeof(unsigned long long);
    if (!configure<lpt_order_kernel<int>>(kLptMaxSeqs * 8) ||
        !configure<lpt_order_kernel<long long>>(kLptMaxSeqs * 8))
      return cudaErrorInvalidValue;
    if (p.cu_int64)
      lpt_order_kernel<long long><<<1, 1024, sm, s>>>(static_cast<const long long*>(p.cu), p.N,
                                                       p.T, order);
    else
      lpt_order_kernel<int><<<1, 1024, sm, s>>>(static_cast<const int*>(p.cu), p.N, p.T, order);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  SplitParams sp{static_cast<const __nv_bfloat16*>(p.a), static_cast<const __nv_bfloat16*>(p.b),
                 p.A_log, p.dt_bias, p.cu, p.state, p.new_state,
                 static_cast<__nv_bfloat16*>(p.out), order,
                 p.ready_base ? p.ready_base : reinterpret_cast<const int*>(ws + lay.base),
                 ws + lay.rec,
                 rec_bytes(p.l2norm), rec_lo_bytes(p.l2norm), p.T, p.N, p.HV, p.HV / p.HQ,
                 p.scale, p.gates_pre, p.g_alpha, p.g_beta, p.ckpt, p.ckpt_starts,
                 p.ckpt_capacity, p.ckpt_every};
  sp.a_rs = p.rs.a;
  sp.b_rs = p.rs.b;
  sp.o_rs = p.rs.o;
  sp.vsplit = p.vsplit;
  sp.vsrc = p.vsrc;
  sp.out_alt = static_cast<__nv_bfloat16*>(p.out_alt);
  sp.state_runs = p.state_runs;
  sp.prep_runs = p.prep_runs;
  sp.rec_alias = p.rec_alias;
  // chunks to prepare: those of the first prep_runs runs (each run's chunks are at most
  // its tokens / 64 + 1, and those runs' tokens are the input rows)
  const long long prep_slots =
      p.prep_runs < p.N ? std::min(lay.slots, (rows + kC - 1) / kC + p.prep_runs) : lay.slots;
  if (p.cu_int64)
    return launch_split_cu<long long>(mq, mk, mv, sp, p.l2norm, p.state != nullptr, prep_slots,
                                      p.ready_base != nullptr, s);
  return launch_split_cu<int>(mq, mk, mv, sp, p.l2norm, p.state != nullptr, prep_slots,
                              p.ready_base != nullptr, s);
}

unsigned read_split_device_error(bool clear) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_split_device_error, sizeof(v)) != cudaSuccess) return ~0u;
  if (clear) {
    const unsigned zero = 0;
    cudaMemcpyToSymbol(g_split_device_error, &zero, sizeof(zero));
  }
  return v;
}

}  // namespace gdn
