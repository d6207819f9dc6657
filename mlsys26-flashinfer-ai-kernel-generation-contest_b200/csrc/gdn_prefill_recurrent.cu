// GDN prefill, token-serial recurrent form on CUDA cores (sm_100a).
//
// The per-token recurrence of the flashinfer-bench definition reference
// (flashinfer/trace/templates/gdn.py:228-271) executed directly: each CTA owns
// 16 rows (v) of one (sequence, v-head) state and walks the sequence's tokens
// in order, keeping its 16 x 128 fp32 state slice in registers (8 lanes per
// row, 16 columns per lane).  Rows of the state are independent given the
// token stream, so the 8 row-tiles of a head run in parallel CTAs.
//
// It is exact to fp32 rounding and is used for short sequences, where the
// chunked tensor-core kernel's per-chunk overhead dominates, and as the
// second opinion in the GPU tests.
#include "gdn_common.cuh"
#include "gdn_prefill.cuh"

namespace gdn {
namespace {

constexpr int kRecRows = 16;  // rows per CTA (4 warps x 4 rows)

struct TokIn {
  uint2 k[4], q[4];
  float v, a, b;
};

// Per-token gate inputs: the raw projections (a, b) or precomputed decay / beta (fp32,
// null = 1).  `a`/`b` then hold alpha and beta themselves.
struct GateSrc {
  const __nv_bfloat16* a;
  const __nv_bfloat16* b;
  const float* alpha;
  const float* beta;
  bool pre;
};

__device__ __forceinline__ void load_tok(TokIn& t, const __nv_bfloat16* q, const __nv_bfloat16* k,
                                         const __nv_bfloat16* v, const GateSrc& gs,
                                         long long tok, const RowStrides& rs, int HV,
                                         int qh, int h, int row, int j) {
  const __nv_bfloat16* qp = q + (size_t)tok * rs.q + qh * kHeadDim + 4 * j;
  const __nv_bfloat16* kp = k + (size_t)tok * rs.k + qh * kHeadDim + 4 * j;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    t.q[m] = __ldg(reinterpret_cast<const uint2*>(qp + 32 * m));
    t.k[m] = __ldg(reinterpret_cast<const uint2*>(kp + 32 * m));
  }
  t.v = bf2f(v[(size_t)tok * rs.v + h * kHeadDim + row]);
  if (gs.pre) {  // precomputed gates: dense fp32 [T, HV]
    const size_t ti = (size_t)tok * HV + h;
    t.a = gs.alpha ? __ldg(gs.alpha + ti) : 1.f;
    t.b = gs.beta ? __ldg(gs.beta + ti) : 1.f;
  } else {
    t.a = bf2f(gs.a[(size_t)tok * rs.a + h]);
    t.b = bf2f(gs.b[(size_t)tok * rs.b + h]);
  }
}

template <bool L2NORM, bool HAS_STATE, typename CuT>
__global__ void __launch_bounds__(128)
    prefill_recurrent_kernel(const __nv_bfloat16* __restrict__ q,
                             const __nv_bfloat16* __restrict__ k,
                             const __nv_bfloat16* __restrict__ v, const float* state,
                             const float* __restrict__ A_log, const __nv_bfloat16* __restrict__ a,
                             const float* __restrict__ dt_bias,
                             const __nv_bfloat16* __restrict__ b, const CuT* __restrict__ cu,
                             float scale, __nv_bfloat16* __restrict__ out, float* new_state,
                             long long T, const RowStrides rs, int HV, int ratio, int seq_offset,
                             const float* __restrict__ g_alpha, const float* __restrict__ g_beta,
                             bool gates_pre, float* __restrict__ ckpt,
                             const long long* __restrict__ ckpt_starts, long long ckpt_cap,
                             int ckpt_every) {
  constexpr int VT = kHeadDim / kRecRows;
  const int cta = blockIdx.x;
  const int vt = cta % VT;
  const int nh = cta / VT;
  const int h = nh % HV;
  const int n = nh / HV + seq_offset;
  const int qh = h / ratio;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane >> 3, j = lane & 7;
  const int row = vt * kRecRows + warp * 4 + sub;
  // cu_seqlens is caller data: clamp it into [0, T] so a malformed table can
  // never address tokens outside q/k/v/a/b/output.
  const long long s1 = min(max((long long)cu[n + 1], 0LL), T);
  const long long s0 = min(max((long long)cu[n], 0LL), s1);
  const size_t sbase = ((size_t)n * HV + h) * kHeadDim * kHeadDim + (size_t)row * kHeadDim + 4 * j;

  float4 S[4];
  if (HAS_STATE && s1 > s0) {
#pragma unroll
    for (int m = 0; m < 4; ++m) S[m] = ld_stream_f4(state + sbase + 32 * m);
  } else {
#pragma unroll
    for (int m = 0; m < 4; ++m) S[m] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float nexpA = gates_pre ? 0.f : -expf(__ldg(A_log + h));
  const float dtb = gates_pre ? 0.f : __ldg(dt_bias + h);
  scale = default_scale(scale);
  const GateSrc gs{a, b, g_alpha, g_beta, gates_pre};

  TokIn cur, nxt;
  if (s1 > s0) load_tok(cur, q, k, v, gs, s0, rs, HV, qh, h, row, j);
  for (long long t = s0; t < s1; ++t) {
    if (t + 1 < s1) load_tok(nxt, q, k, v, gs, t + 1, rs, HV, qh, h, row, j);
    float kf[16], qf[16];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      float2 f;
      f = bf2x2_to_f2(cur.k[m].x); kf[4 * m] = f.x; kf[4 * m + 1] = f.y;
      f = bf2x2_to_f2(cur.k[m].y); kf[4 * m + 2] = f.x; kf[4 * m + 3] = f.y;
      f = bf2x2_to_f2(cur.q[m].x); qf[4 * m] = f.x; qf[4 * m + 1] = f.y;
      f = bf2x2_to_f2(cur.q[m].y); qf[4 * m + 2] = f.x; qf[4 * m + 3] = f.y;
    }
    const float g = gates_pre ? cur.a : expf(nexpA * softplus_f(cur.a + dtb));
    const float beta = gates_pre ? cur.b : sigmoid_f(cur.b);
    float kq = 0.f, sk = 0.f, sq = 0.f, ssk = 0.f, ssq = 0.f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float sv[4] = {S[m].x, S[m].y, S[m].z, S[m].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        kq = fmaf(kf[4 * m + e], qf[4 * m + e], kq);
        sk = fmaf(sv[e], kf[4 * m + e], sk);
        sq = fmaf(sv[e], qf[4 * m + e], sq);
        if (L2NORM) {
          ssk = fmaf(kf[4 * m + e], kf[4 * m + e], ssk);
          ssq = fmaf(qf[4 * m + e], qf[4 * m + e], ssq);
        }
      }
    }
    kq = xor_sum8(kq);
    sk = xor_sum8(sk);
    sq = xor_sum8(sq);
    float rk = 1.f;
    if (L2NORM) {
      ssk = xor_sum8(ssk);
      ssq = xor_sum8(ssq);
      rk = rsqrtf(ssk + kL2NormEps);
      const float rq = rsqrtf(ssq + kL2NormEps);
      kq *= rk * rq;
      sk *= rk;
      sq *= rq;
    }
    const float old = g * sk;
    const float delta = beta * (cur.v - old);
    const float dk = delta * rk;  // delta * k_hat = (delta * rk) * k
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      S[m].x = fmaf(g, S[m].x, dk * kf[4 * m + 0]);
      S[m].y = fmaf(g, S[m].y, dk * kf[4 * m + 1]);
      S[m].z = fmaf(g, S[m].z, dk * kf[4 * m + 2]);
      S[m].w = fmaf(g, S[m].w, dk * kf[4 * m + 3]);
    }
    if (j == 0)
      out[(size_t)t * rs.o + h * kHeadDim + row] =
          __float2bfloat16_rn(scale * fmaf(g, sq, delta * kq));
    if (ckpt != nullptr) {
      const long long ci = checkpoint_slot(ckpt_starts, n, t - s0 + 1, ckpt_every, ckpt_cap);
      if (ci >= 0) {
        float* cp = ckpt + ((size_t)ci * HV + h) * kHeadDim * kHeadDim + (size_t)row * kHeadDim + 4 * j;
#pragma unroll
        for (int m = 0; m < 4; ++m) st_stream_f4(cp + 32 * m, S[m]);
      }
    }
    cur = nxt;
  }
#pragma unroll
  for (int m = 0; m < 4; ++m) st_stream_f4(new_state + sbase + 32 * m, S[m]);
}

template <typename CuT>
cudaError_t launch_rec_t(const PrefillArgs& p, const CuT* cu, int seq_offset, int nseq,
                         cudaStream_t st) {
  const dim3 grid((unsigned)((long long)nseq * p.HV * (kHeadDim / kRecRows))), block(128);
  const int ratio = p.HV / p.HQ;
  auto Q = static_cast<const __nv_bfloat16*>(p.q);
  auto K = static_cast<const __nv_bfloat16*>(p.k);
  auto V = static_cast<const __nv_bfloat16*>(p.v);
  auto A = static_cast<const __nv_bfloat16*>(p.a);
  auto Bt = static_cast<const __nv_bfloat16*>(p.b);
  auto O = static_cast<__nv_bfloat16*>(p.out);
#define GDN_REC_LAUNCH(L2, HS)                                                              \
  prefill_recurrent_kernel<L2, HS, CuT><<<grid, block, 0, st>>>(                            \
      Q, K, V, p.state, p.A_log, A, p.dt_bias, Bt, cu, p.scale, O, p.new_state, p.T, p.rs,    \
      p.HV, ratio, seq_offset, p.g_alpha, p.g_beta, p.gates_pre, p.ckpt, p.ckpt_starts,        \
      p.ckpt_capacity, p.ckpt_every)
  if (p.state) {
    if (p.l2norm) GDN_REC_LAUNCH(true, true); else GDN_REC_LAUNCH(false, true);
  } else {
    if (p.l2norm) GDN_REC_LAUNCH(true, false); else GDN_REC_LAUNCH(false, false);
  }
#undef GDN_REC_LAUNCH
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill_recurrent(const PrefillArgs& p, int seq_offset, int nseq,
                                     cudaStream_t st) {
  if (nseq <= 0) return cudaSuccess;
  if (p.cu_int64)
    return launch_rec_t<long long>(p, static_cast<const long long*>(p.cu), seq_offset, nseq, st);
  return launch_rec_t<int>(p, static_cast<const int*>(p.cu), seq_offset, nseq, st);
}

}  // namespace gdn
