// Segmented prefill of ONE sequence on one GPU (no counterpart in the reference, whose
// prefill walks every sequence's chunks in order, gdn_prefill/solution/triton/
// kernel.py:122-247): for a sequence whose v-heads alone leave most SMs idle (one sequence
// of a model sharded by q/k-head group over several GPUs), the tokens are cut into S
// segments on 64-token chunk boundaries, and the split kernels run every segment at once
// as the 2 S - 1 runs of one call:
//   run 0            segment 0 from the initial state           -> output rows, B_0
//   runs 1 .. S-1    segment s from a zero state (real v)        -> o^0 in the output rows, B_s
//   runs S .. 2S-2   segment s from the identity with v = 0      -> o^I in a scratch buffer, A_s
// The runs read their tokens straight from q, k, v, a, b through virtual token rows (the
// identity runs' rows map back onto the segment's tokens; see PrefillArgs), so nothing is
// copied.  Over a segment the recurrence is affine in its start state, so the chain kernel
// then composes S_{s+1} = S_s A_s + B_s (every segment's start state in one pass, the last
// map giving the final state) and the output kernel forms o = S_s o^I + o^0 for every later
// segment in one launch, in place over o^0.  The serial chunk chain shrinks from the whole
// sequence to one segment, at the price of the extra runs and the two assembly kernels.
#include <cuda_runtime.h>

#include <algorithm>

#include "gdn_b200.h"
#include "gdn_common.cuh"
#include "gdn_prefill.cuh"

namespace {

constexpr int kMaxSegments = 64;           // runs' offsets travel as kernel parameters
constexpr long long kMaxTokens = 1LL << 30;
constexpr size_t kMat = (size_t)gdn::kHeadDim * gdn::kHeadDim * sizeof(float);

struct RunOffsets {
  int n;                          // entries of v (runs + 1)
  int v[2 * kMaxSegments];
};

__global__ void run_offsets_kernel(const RunOffsets ro, int* cu) {
  for (int i = threadIdx.x; i < ro.n; i += blockDim.x) cu[i] = ro.v[i];
}

// Segment bounds of `segments` equal shares of the sequence's chunks: b[0] = 0,
// b[s] = 64 floor(chunks s / S) for 0 < s < S, b[S] = T.
struct Plan {
  int S = 1;
  long long T = 0;
  long long b[kMaxSegments + 1] = {};
  int runs() const { return 2 * S - 1; }
  long long virtual_rows() const { return S > 1 ? 2 * T - b[1] : T; }
};

Plan make_plan(long long T, int segments) {
  Plan p;
  p.T = T;
  const long long chunks = (T + 63) / 64;
  p.S = (int)std::max(1LL, std::min<long long>({(long long)segments, chunks, kMaxSegments}));
  for (int s = 0; s < p.S; ++s) p.b[s] = std::min(64 * (chunks * s / p.S), T);
  p.b[p.S] = T;
  return p;
}

int sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  return sms;
}

int resolve_segments(long long T, int HV, int segments) {
  if (segments > 0) return segments;
  // the largest count whose runs all hold an SM at once: 4 state CTAs per (run, v-head)
  const int sms = sm_count();
  const int per_run = std::max(1, 4 * HV);
  return std::max(1, (sms / per_run + 1) / 2);
}

struct Layout {
  size_t cu, split, fin, starts, alt, total;
};

Layout make_layout(const Plan& p, int HV) {
  const auto up = [](size_t x) { return (x + 1023) / 1024 * 1024; };
  Layout l{};
  l.cu = 0;
  l.split = up((size_t)(p.runs() + 1) * sizeof(int));
  l.fin = up(l.split + gdn::prefill_split_workspace(p.virtual_rows(), p.runs(), HV));
  l.starts = up(l.fin + (p.S > 1 ? (size_t)p.runs() * HV * kMat : 0));
  l.alt = up(l.starts + (size_t)(p.S - 1) * HV * kMat);
  l.total = l.alt + (size_t)(p.T - p.b[1]) * HV * gdn::kHeadDim * 2 * (p.S > 1);
  return l;
}

inline bool misaligned(const void* p, uintptr_t n) {
  return (reinterpret_cast<uintptr_t>(p) % n) != 0;
}

}  // namespace

extern "C" int gdn_prefill_segments_auto(int total_tokens, int num_v_heads) {
  if (total_tokens < 0 || num_v_heads <= 0) return GDN_ERR_INVALID_ARGUMENT;
  return make_plan(total_tokens, resolve_segments(total_tokens, num_v_heads, 0)).S;
}

extern "C" size_t gdn_prefill_segmented_workspace_size(int total_tokens, int num_v_heads,
                                                       int segments) {
  if (total_tokens <= 0 || num_v_heads <= 0 || segments < 0) return 0;
  const Plan p = make_plan(total_tokens, resolve_segments(total_tokens, num_v_heads, segments));
  return make_layout(p, num_v_heads).total;
}

extern "C" int gdn_prefill_segmented_launch(
    const void* q, const void* k, const void* v, const float* state, const float* A_log,
    const void* a, const float* dt_bias, const void* b, float scale, void* output,
    float* new_state, int total_tokens, int num_q_heads, int num_k_heads, int num_v_heads,
    int head_size, int use_qk_l2norm, int segments, long long q_stride, long long k_stride,
    long long v_stride, long long a_stride, long long b_stride, void* workspace,
    size_t workspace_bytes, void* stream) {
  using namespace gdn;
  if (total_tokens < 0 || total_tokens > kMaxTokens || num_q_heads <= 0 || num_k_heads <= 0 ||
      num_v_heads <= 0 || segments < 0)
    return GDN_ERR_INVALID_ARGUMENT;
  if (head_size != kHeadDim || num_k_heads != num_q_heads || num_v_heads % num_q_heads != 0)
    return GDN_ERR_UNSUPPORTED;
  if (!new_state || !A_log || !dt_bias) return GDN_ERR_INVALID_ARGUMENT;
  if (misaligned(new_state, 16) || (state && misaligned(state, 16)))
    return GDN_ERR_INVALID_ARGUMENT;
  const int HV = num_v_heads;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (total_tokens == 0)  // an empty sequence's final state is zero (definition semantics)
    return cudaMemsetAsync(new_state, 0, (size_t)HV * kMat, st) == cudaSuccess ? GDN_OK
                                                                               : GDN_ERR_LAUNCH;
  if (!q || !k || !v || !a || !b || !output) return GDN_ERR_INVALID_ARGUMENT;
  const RowStrides rs{q_stride, k_stride, v_stride, a_stride, b_stride,
                      (long long)HV * kHeadDim};
  {  // rows never overlap; the tensor-core kernels read q / k / v rows by TMA
    const long long qk_row = (long long)num_q_heads * kHeadDim;
    const long long v_row = (long long)HV * kHeadDim;
    if (rs.q < qk_row || rs.k < qk_row || rs.v < v_row || rs.a < HV || rs.b < HV)
      return GDN_ERR_INVALID_ARGUMENT;
  }
  const Plan plan = make_plan(total_tokens, resolve_segments(total_tokens, HV, segments));
  const Layout lay = make_layout(plan, HV);
  if (workspace == nullptr || workspace_bytes < lay.total) return GDN_ERR_WORKSPACE;
  if (misaligned(workspace, 1024)) return GDN_ERR_INVALID_ARGUMENT;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int S = plan.S;
  const long long T = plan.T, b1 = plan.b[1];

  int* cu = reinterpret_cast<int*>(ws + lay.cu);
  float* fin = reinterpret_cast<float*>(ws + lay.fin);
  PrefillArgs p{q, k, v, state, A_log, a, dt_bias, b, cu, false, scale, output,
                S > 1 ? fin : new_state, plan.virtual_rows(), plan.runs(), num_q_heads, HV,
                use_qk_l2norm != 0, ws + lay.split, lay.fin - lay.split};
  p.rs = rs;
  p.src_rows = T;
  p.state_runs = 1;
  if (S > 1) {
    p.vsplit = T;
    p.vsrc = b1;
    p.out_alt = ws + lay.alt;
  }
  if (!prefill_chunked_supported(p)) return GDN_ERR_UNSUPPORTED;

  // run offsets (virtual rows): [b_0 .. b_S], then T + b_s - b_1 for the identity runs
  RunOffsets ro{};
  ro.n = plan.runs() + 1;
  for (int s = 0; s <= S; ++s) ro.v[s] = (int)plan.b[s];
  for (int s = 2; s <= S; ++s) ro.v[S + s - 1] = (int)(T + plan.b[s] - b1);
  run_offsets_kernel<<<1, 128, 0, st>>>(ro, cu);
  if (cudaGetLastError() != cudaSuccess) return GDN_ERR_LAUNCH;
  if (launch_prefill_split(p, st) != cudaSuccess) return GDN_ERR_LAUNCH;
  if (S == 1) return GDN_OK;

  // maps in run order: B_s = fin[s] (s < S), A_s = fin[S - 1 + s] (s >= 1)
  float* starts = reinterpret_cast<float*>(ws + lay.starts);
  const size_t per = (size_t)HV * kHeadDim * kHeadDim;
  if (launch_segment_chain(fin, S - 1, 1, 0, 1, S - 1, HV, starts + (size_t)(S - 2) * per,
                           new_state, starts, st) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  // o = S_s o^I + o^0 over rows [b_1, T): o^I in the scratch rows, o^0 in the output
  int off[kMaxSegments], len[kMaxSegments];
  for (int s = 1; s < S; ++s) {
    off[s - 1] = (int)(plan.b[s] - b1);
    len[s - 1] = (int)(plan.b[s + 1] - plan.b[s]);
  }
  uint8_t* out_rows = static_cast<uint8_t*>(output) + (size_t)b1 * HV * kHeadDim * 2;
  if (launch_segment_outputs(ws + lay.alt, T - b1, out_rows, T - b1, starts, out_rows, S - 1, off,
                             len, HV, st) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  return GDN_OK;
}
