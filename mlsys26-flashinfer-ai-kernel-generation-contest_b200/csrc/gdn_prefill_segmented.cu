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
#include <cmath>
#include <map>
#include <mutex>
#include <queue>
#include <tuple>
#include <vector>

#include "gdn_b200.h"
#include "gdn_common.cuh"
#include "gdn_prefill.cuh"

namespace {

constexpr int kMaxSegments = 64;           // runs' offsets travel as kernel parameters
constexpr long long kMaxTokens = 1LL << 30;
constexpr size_t kMat = (size_t)gdn::kHeadDim * gdn::kHeadDim * sizeof(float);

// The runs' token offsets (cu), chunk offsets and longest-first order, known on the host,
// written to the workspace by one small launch (no device-side scans).
struct RunOffsets {
  int n;                          // entries of v and base (runs + 1); order has n - 1
  int v[2 * kMaxSegments];
  int base[2 * kMaxSegments];
  int order[2 * kMaxSegments];
};

__global__ void run_offsets_kernel(const RunOffsets ro, int* cu, int* base, int* order) {
  for (int i = threadIdx.x; i < ro.n; i += blockDim.x) {
    cu[i] = ro.v[i];
    base[i] = ro.base[i];
    if (i + 1 < ro.n) order[i] = ro.order[i];
  }
}

// Segment bounds b[0] = 0 < b[1] < .. < b[S] = T, interior bounds on 64-token chunks.
struct Plan {
  int S = 1;
  long long T = 0;
  long long b[kMaxSegments + 1] = {};
  int runs() const { return 2 * S - 1; }
  long long virtual_rows() const { return S > 1 ? 2 * T - b[1] : T; }
};

// Segment 0 of x chunks, the other chunks - x in S - 1 equal shares.
Plan lead_plan(long long T, int S, long long x) {
  Plan p;
  p.T = T;
  p.S = S;
  const long long chunks = (T + 63) / 64;
  p.b[0] = 0;
  for (int s = 1; s < S; ++s)
    p.b[s] = std::min(64 * (x + (chunks - x) * (s - 1) / (S - 1)), T);
  p.b[S] = T;
  return p;
}

// `segments` equal shares of the sequence's chunks: b[s] = 64 floor(chunks s / S).
Plan equal_plan(long long T, int segments) {
  const long long chunks = (T + 63) / 64;
  const int S = (int)std::max(1LL, std::min<long long>({(long long)segments, chunks,
                                                        (long long)kMaxSegments}));
  Plan p;
  p.T = T;
  p.S = S;
  for (int s = 0; s < S; ++s) p.b[s] = std::min(64 * (chunks * s / S), T);
  p.b[S] = T;
  return p;
}

// Cost model of a plan, in units of one chunk step of the split state kernel (2.2 us on
// B200): the state kernel's makespan when its CTAs (4 per run and v-head, longest run
// first, one per SM) are dealt to the SMs as they free up, each costing its run's chunks
// plus kCtaStart; the preparation kernel before it (3 CTAs per SM, one per chunk and pair
// of v-heads, ~20 us per wave); one chain step per later segment (~3.5 us); the output
// pass over the later segments' tokens (3 x 256 bytes per token and v-head at ~3.5 TB/s).
// Constants measured on B200 with P2's head shares of 2, 4 and 8 GPUs.
constexpr double kStepUs = 2.2, kCtaStart = 3.0, kPrepWaveUs = 20.0, kChainStepUs = 3.5;
constexpr double kOutBytesPerUs = 3.5e6;

double plan_cost(const Plan& p, int HV, int sms) {
  std::vector<long long> len;
  len.reserve(p.runs());
  for (int s = 0; s < p.S; ++s) {
    const long long c = (p.b[s + 1] - p.b[s] + 63) / 64;
    len.push_back(c);
    if (s > 0) len.push_back(c);
  }
  std::stable_sort(len.begin(), len.end(), [](long long a, long long b) { return a > b; });
  std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
  for (int i = 0; i < sms; ++i) free_at.push(0.0);
  double makespan = 0.0;
  long long vchunks = 0;
  for (int s = 0; s < p.S; ++s) vchunks += (p.b[s + 1] - p.b[s] + 63) / 64;  // prepared once
  for (long long c : len) {
    for (int j = 0; j < 4 * HV; ++j) {
      const double t = free_at.top() + (double)c + kCtaStart;
      free_at.pop();
      free_at.push(t);
      makespan = std::max(makespan, t);
    }
  }
  const double prep_ctas = (double)vchunks * std::max(1, HV / 2);
  double us = std::ceil(prep_ctas / (3.0 * sms)) * kPrepWaveUs;
  if (p.S > 1)
    us += kChainStepUs * (p.S - 1) + (double)(p.T - p.b[1]) * HV * 768.0 / kOutBytesPerUs;
  return makespan + us / kStepUs;
}

// The plan for segments = 0: segment 0 of x chunks (run once) and S - 1 equal later
// segments (run twice each), S <= 16 and x chosen by the cost model; segmenting is taken
// only when the model predicts at least 5 % less time than one segment.  When every run
// fits on the SMs at once this gives about equal segments; with more runs x v-heads x 4
// CTAs than SMs it lets segment 0 run long on its own SMs while the shorter later runs
// pass over the other SMs in several waves.
Plan auto_plan(long long T, int HV, int sms) {
  const long long chunks = (T + 63) / 64;
  Plan best = equal_plan(T, 1);
  if (sms <= 0 || chunks < 2) return best;
  const double one = plan_cost(best, HV, sms);
  double best_cost = one;
  const int smax = (int)std::min<long long>(16, chunks);
  for (int S = 2; S <= smax; ++S) {
    // x from chunks / S (equal) up to chunks - (S - 1): a coarse scan, then halving steps
    const long long lo = (chunks + S - 1) / S, hi = chunks - (S - 1);
    if (lo > hi) continue;
    long long step = std::max(1LL, (hi - lo) / 32), bx = lo;
    double bc = plan_cost(lead_plan(T, S, lo), HV, sms);
    for (long long x = lo + step; x <= hi; x += step) {
      const double c = plan_cost(lead_plan(T, S, x), HV, sms);
      if (c < bc) bc = c, bx = x;
    }
    while (step > 1) {
      step /= 2;
      for (long long x : {bx - step, bx + step}) {
        if (x < lo || x > hi) continue;
        const double c = plan_cost(lead_plan(T, S, x), HV, sms);
        if (c < bc) bc = c, bx = x;
      }
    }
    if (bc < best_cost) best_cost = bc, best = lead_plan(T, S, bx);
  }
  return best_cost < 0.95 * one ? best : equal_plan(T, 1);
}

// A plan from caller-given bounds (host memory, S + 1 token offsets): b[0] = 0, strictly
// increasing, interior bounds on 64-token chunks, b[S] = T, S <= 64.
bool bounds_plan(long long T, int S, const int* bounds, Plan* p) {
  if (S < 1 || S > kMaxSegments || bounds == nullptr || bounds[0] != 0 || bounds[S] != T)
    return false;
  p->T = T;
  p->S = S;
  for (int s = 0; s <= S; ++s) {
    if (s > 0 && bounds[s] <= bounds[s - 1]) return false;
    if (s > 0 && s < S && bounds[s] % 64 != 0) return false;
    p->b[s] = bounds[s];
  }
  return true;
}

int sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  return sms;
}

// Plans for segments = 0 are cached per (T, HV, SMs): the search takes milliseconds.
Plan make_plan(long long T, int HV, int segments, int sms) {
  if (segments > 0 || T <= 0) return equal_plan(T, std::max(1, segments));
  static std::mutex mu;
  static std::map<std::tuple<long long, int, int>, Plan> cache;
  const auto key = std::make_tuple(T, HV, sms);
  {
    std::lock_guard<std::mutex> g(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const Plan p = auto_plan(T, HV, sms);
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 256) cache.clear();
  cache[key] = p;
  return p;
}

struct Layout {
  size_t cu, split, fin, starts, alt, total;
};

Layout make_layout(const Plan& p, int HV) {
  const auto up = [](size_t x) { return (x + 1023) / 1024 * 1024; };
  Layout l{};
  l.cu = 0;
  l.split = up((size_t)3 * (2 * kMaxSegments) * sizeof(int));  // cu | base | order
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

extern "C" int gdn_prefill_segment_plan(int total_tokens, int num_v_heads, int segments,
                                        int num_sms, int* bounds, int capacity) {
  if (total_tokens < 0 || num_v_heads <= 0 || segments < 0 || capacity < 0 ||
      (capacity > 0 && bounds == nullptr))
    return GDN_ERR_INVALID_ARGUMENT;
  const Plan p = make_plan(total_tokens, num_v_heads, segments,
                           num_sms > 0 ? num_sms : (segments > 0 ? 0 : sm_count()));
  for (int s = 0; s <= p.S && s < capacity; ++s) bounds[s] = (int)p.b[s];
  return p.S;
}

extern "C" int gdn_prefill_segments_auto(int total_tokens, int num_v_heads) {
  return gdn_prefill_segment_plan(total_tokens, num_v_heads, 0, 0, nullptr, 0);
}

extern "C" size_t gdn_prefill_segmented_workspace_size(int total_tokens, int num_v_heads,
                                                       int segments, const int* segment_bounds) {
  if (total_tokens <= 0 || num_v_heads <= 0 || segments < 0) return 0;
  Plan p;
  if (segment_bounds != nullptr) {
    if (!bounds_plan(total_tokens, segments, segment_bounds, &p)) return 0;
  } else {
    p = make_plan(total_tokens, num_v_heads, segments, segments > 0 ? 0 : sm_count());
  }
  return make_layout(p, num_v_heads).total;
}

extern "C" int gdn_prefill_segmented_launch(
    const void* q, const void* k, const void* v, const float* state, const float* A_log,
    const void* a, const float* dt_bias, const void* b, float scale, void* output,
    float* new_state, int total_tokens, int num_q_heads, int num_k_heads, int num_v_heads,
    int head_size, int use_qk_l2norm, int segments, const int* segment_bounds,
    long long q_stride, long long k_stride,
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
  Plan plan;
  if (segment_bounds != nullptr) {
    if (!bounds_plan(total_tokens, segments, segment_bounds, &plan)) return GDN_ERR_INVALID_ARGUMENT;
  } else {
    plan = make_plan(total_tokens, HV, segments, segments > 0 ? 0 : sm_count());
  }
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
  p.ready_base = cu + 2 * kMaxSegments;
  p.ready_order = plan.runs() > 1 ? cu + 4 * kMaxSegments : nullptr;
  if (S > 1) {
    p.vsplit = T;
    p.vsrc = b1;
    p.out_alt = ws + lay.alt;
    p.prep_runs = S;     // the identity run of segment s reads the records of run s
    p.rec_alias = S - 1;
  }
  if (!prefill_chunked_supported(p)) return GDN_ERR_UNSUPPORTED;

  // run offsets (virtual rows): [b_0 .. b_S], then T + b_s - b_1 for the identity runs
  RunOffsets ro{};
  ro.n = plan.runs() + 1;
  for (int s = 0; s <= S; ++s) ro.v[s] = (int)plan.b[s];
  for (int s = 2; s <= S; ++s) ro.v[S + s - 1] = (int)(T + plan.b[s] - b1);
  ro.base[0] = 0;
  for (int r = 0; r < plan.runs(); ++r) {
    ro.base[r + 1] = ro.base[r] + (ro.v[r + 1] - ro.v[r] + 63) / 64;
    ro.order[r] = r;
  }
  // longest run first, ties by index (the order the library's device-side sort gives)
  std::stable_sort(ro.order, ro.order + plan.runs(), [&](int x, int y) {
    return ro.v[x + 1] - ro.v[x] > ro.v[y + 1] - ro.v[y];
  });
  run_offsets_kernel<<<1, 128, 0, st>>>(ro, cu, cu + 2 * kMaxSegments, cu + 4 * kMaxSegments);
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
