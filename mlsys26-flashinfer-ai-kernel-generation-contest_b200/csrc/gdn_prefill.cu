// C-ABI entry point of the GDN prefill: argument checks and kernel selection.
//
// Replaces the reference host wrapper gdn_prefill (reference
// gdn_prefill/solution/triton/kernel.py:253-337).  Unlike that wrapper it
// needs no output zero-fill pass and no state -> new_state copy pass: every
// output row of every token and every new_state slice (zero for an empty
// sequence) is written by the kernels themselves.
#include "gdn_common.cuh"
#include "gdn_prefill.cuh"

namespace {
inline bool misaligned(const void* p, uintptr_t n) {
  return (reinterpret_cast<uintptr_t>(p) % n) != 0;
}
}  // namespace

extern "C" size_t gdn_prefill_workspace_size(int total_tokens, int num_seqs, int num_q_heads,
                                             int num_v_heads, int head_size) {
  (void)num_q_heads;
  (void)num_v_heads;
  (void)head_size;
  if (total_tokens <= 0) return 0;
  return gdn::prefill_chunked_workspace(num_seqs);  // longest-first sequence order
}

namespace {
enum class PrefillPath { kAuto, kRecurrent };

int prefill_entry(PrefillPath path, const void* q, const void* k, const void* v, const float* state,
                                  const float* A_log, const void* a, const float* dt_bias,
                                  const void* b, const void* cu_seqlens, int cu_seqlens_int64,
                                  float scale, void* output, float* new_state, int total_tokens,
                                  int num_seqs, int num_q_heads, int num_k_heads, int num_v_heads,
                                  int head_size, int use_qk_l2norm, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  using namespace gdn;
  if (total_tokens < 0 || num_seqs < 0 || num_q_heads <= 0 || num_k_heads <= 0 ||
      num_v_heads <= 0)
    return GDN_ERR_INVALID_ARGUMENT;
  if (head_size != kHeadDim || num_k_heads != num_q_heads || num_v_heads % num_q_heads != 0)
    return GDN_ERR_UNSUPPORTED;
  if (num_seqs == 0) return GDN_OK;
  if (!cu_seqlens || !A_log || !dt_bias || !new_state) return GDN_ERR_INVALID_ARGUMENT;
  if (total_tokens > 0 && (!q || !k || !v || !a || !b || !output)) return GDN_ERR_INVALID_ARGUMENT;
  if (misaligned(q, 8) || misaligned(k, 8) || misaligned(new_state, 16) ||
      (state && misaligned(state, 16)) || misaligned(cu_seqlens, cu_seqlens_int64 ? 8 : 4))
    return GDN_ERR_INVALID_ARGUMENT;
  if ((long long)num_seqs * num_v_heads * 8 > 0x7fffffffLL) return GDN_ERR_INVALID_ARGUMENT;
  const size_t need =
      gdn_prefill_workspace_size(total_tokens, num_seqs, num_q_heads, num_v_heads, head_size);
  if (path == PrefillPath::kAuto && need > 0 && (workspace == nullptr || workspace_bytes < need))
    return GDN_ERR_WORKSPACE;  // (the recurrent kernel uses no workspace)

  PrefillArgs p{q,        k,     v,      state,      A_log,        a,           dt_bias,
                b,        cu_seqlens, cu_seqlens_int64 != 0, scale, output, new_state,
                (long long)total_tokens, num_seqs, num_q_heads, num_v_heads,
                use_qk_l2norm != 0, workspace, workspace_bytes};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  if (path == PrefillPath::kAuto && prefill_chunked_supported(p))
    err = launch_prefill_chunked(p, st);
  else
    err = launch_prefill_recurrent(p, 0, num_seqs, st);
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
}  // namespace

extern "C" int gdn_prefill_launch(const void* q, const void* k, const void* v, const float* state,
                                  const float* A_log, const void* a, const float* dt_bias,
                                  const void* b, const void* cu_seqlens, int cu_seqlens_int64,
                                  float scale, void* output, float* new_state, int total_tokens,
                                  int num_seqs, int num_q_heads, int num_k_heads, int num_v_heads,
                                  int head_size, int use_qk_l2norm, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  return prefill_entry(PrefillPath::kAuto, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                       cu_seqlens_int64, scale, output, new_state, total_tokens, num_seqs,
                       num_q_heads, num_k_heads, num_v_heads, head_size, use_qk_l2norm, workspace,
                       workspace_bytes, stream);
}

extern "C" int gdn_prefill_launch_recurrent(
    const void* q, const void* k, const void* v, const float* state, const float* A_log,
    const void* a, const float* dt_bias, const void* b, const void* cu_seqlens,
    int cu_seqlens_int64, float scale, void* output, float* new_state, int total_tokens,
    int num_seqs, int num_q_heads, int num_k_heads, int num_v_heads, int head_size,
    int use_qk_l2norm, void* workspace, size_t workspace_bytes, void* stream) {
  return prefill_entry(PrefillPath::kRecurrent, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                       cu_seqlens_int64, scale, output, new_state, total_tokens, num_seqs,
                       num_q_heads, num_k_heads, num_v_heads, head_size, use_qk_l2norm, workspace,
                       workspace_bytes, stream);
}

extern "C" int gdn_device_error(int clear) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  return (int)gdn::read_device_error(clear != 0);
}
