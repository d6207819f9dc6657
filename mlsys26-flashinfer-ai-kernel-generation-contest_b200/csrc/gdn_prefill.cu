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

namespace {
// The fused kernel runs one CTA per (sequence, v-head) for the whole scan; with
// fewer such pairs than B200 has SMs (148), most SMs would idle, and the split
// kernels (chunk-parallel preparation, then the scan on two CTAs per pair) are
// faster.  With at least one pair per SM the fused kernel is faster.
constexpr long long kSplitBelowPairs = 148;
bool auto_uses_split(long long T, int N, int HV) {
  return T > 0 && N > 0 && (long long)N * HV < kSplitBelowPairs;
}

// Precomputed gates or checkpoints with raw q/k: only the split kernels have both.
bool ext_needs_split(bool l2norm, bool ext) { return ext && !l2norm; }

size_t variant_workspace(int variant, long long T, int N, int HV, bool force_split = false) {
  if (T <= 0 || N <= 0) return 0;
  if (force_split && variant == GDN_PREFILL_AUTO) variant = GDN_PREFILL_SPLIT;
  switch (variant) {
    case GDN_PREFILL_RECURRENT: return 0;
    case GDN_PREFILL_FUSED: return gdn::prefill_chunked_workspace(N);
    case GDN_PREFILL_SPLIT: return gdn::prefill_split_workspace(T, N, HV);
    default:
      return auto_uses_split(T, N, HV) ? gdn::prefill_split_workspace(T, N, HV)
                                       : gdn::prefill_chunked_workspace(N);
  }
}
}  // namespace

extern "C" size_t gdn_prefill_workspace_size_variant(int variant, int total_tokens, int num_seqs,
                                                     int num_q_heads, int num_v_heads,
                                                     int head_size) {
  (void)num_q_heads;
  (void)head_size;
  return variant_workspace(variant, total_tokens, num_seqs, num_v_heads);
}

extern "C" size_t gdn_prefill_workspace_size_ext(int variant, int total_tokens, int num_seqs,
                                                 int num_q_heads, int num_v_heads, int head_size,
                                                 int use_qk_l2norm, int gate_mode,
                                                 int checkpoint_every_n_tokens) {
  (void)num_q_heads;
  (void)head_size;
  const bool ext = gate_mode != 0 || checkpoint_every_n_tokens > 0;
  return variant_workspace(variant, total_tokens, num_seqs, num_v_heads,
                           ext_needs_split(use_qk_l2norm != 0, ext));
}

extern "C" size_t gdn_prefill_workspace_size(int total_tokens, int num_seqs, int num_q_heads,
                                             int num_v_heads, int head_size) {
  return gdn_prefill_workspace_size_variant(GDN_PREFILL_AUTO, total_tokens, num_seqs,
                                            num_q_heads, num_v_heads, head_size);
}

namespace {
struct PrefillExt {
  bool gates_pre = false;
  const float* g_alpha = nullptr;
  const float* g_beta = nullptr;
  float* ckpt = nullptr;
  const long long* ckpt_starts = nullptr;
  long long ckpt_capacity = 0;
  int ckpt_every = 0;
};

int prefill_entry(int variant, const void* q, const void* k, const void* v, const float* state,
                  const float* A_log, const void* a, const float* dt_bias, const void* b,
                  const void* cu_seqlens, int cu_seqlens_int64, float scale, void* output,
                  float* new_state, int total_tokens, int num_seqs, int num_q_heads,
                  int num_k_heads, int num_v_heads, int head_size, int use_qk_l2norm,
                  void* workspace, size_t workspace_bytes, void* stream,
                  const PrefillExt& ext = PrefillExt{}, const gdn::RowStrides* strides = nullptr) {
  using namespace gdn;
  if (variant < GDN_PREFILL_AUTO || variant > GDN_PREFILL_SPLIT) return GDN_ERR_INVALID_ARGUMENT;
  if (total_tokens < 0 || num_seqs < 0 || num_q_heads <= 0 || num_k_heads <= 0 ||
      num_v_heads <= 0)
    return GDN_ERR_INVALID_ARGUMENT;
  if (head_size != kHeadDim || num_k_heads != num_q_heads || num_v_heads % num_q_heads != 0)
    return GDN_ERR_UNSUPPORTED;
  if (num_seqs == 0) return GDN_OK;
  if (!cu_seqlens || !new_state) return GDN_ERR_INVALID_ARGUMENT;
  if (!ext.gates_pre && (!A_log || !dt_bias)) return GDN_ERR_INVALID_ARGUMENT;
  if (total_tokens > 0 && (!q || !k || !v || !output || (!ext.gates_pre && (!a || !b))))
    return GDN_ERR_INVALID_ARGUMENT;
  if (ext.ckpt_every < 0 || (ext.ckpt_every > 0 && (ext.ckpt_every % 64 != 0 || !ext.ckpt ||
                                                    !ext.ckpt_starts || ext.ckpt_capacity < 0)))
    return GDN_ERR_INVALID_ARGUMENT;
  if ((ext.g_alpha && misaligned(ext.g_alpha, 4)) || (ext.g_beta && misaligned(ext.g_beta, 4)) ||
      (ext.ckpt && misaligned(ext.ckpt, 16)) || (ext.ckpt_starts && misaligned(ext.ckpt_starts, 8)))
    return GDN_ERR_INVALID_ARGUMENT;
  const bool has_ext = ext.gates_pre || ext.ckpt_every > 0;
  const bool need_split = ext_needs_split(use_qk_l2norm != 0, has_ext);
  if (need_split && variant == GDN_PREFILL_FUSED) return GDN_ERR_UNSUPPORTED;
  if (misaligned(q, 8) || misaligned(k, 8) || misaligned(new_state, 16) ||
      (state && misaligned(state, 16)) || misaligned(cu_seqlens, cu_seqlens_int64 ? 8 : 4))
    return GDN_ERR_INVALID_ARGUMENT;
  if ((long long)num_seqs * num_v_heads * 8 > 0x7fffffffLL) return GDN_ERR_INVALID_ARGUMENT;
  const RowStrides rs = strides ? *strides : dense_rows(num_q_heads, num_v_heads);
  {  // token rows of one tensor never overlap; q/k rows keep their 8-byte alignment
    const long long qk_row = (long long)num_q_heads * kHeadDim;
    const long long v_row = (long long)num_v_heads * kHeadDim;
    if (rs.q < qk_row || rs.k < qk_row || rs.v < v_row || rs.o < v_row ||
        rs.a < num_v_heads || rs.b < num_v_heads || rs.q % 4 != 0 || rs.k % 4 != 0)
      return GDN_ERR_INVALID_ARGUMENT;
  }
  const size_t need = variant_workspace(variant, total_tokens, num_seqs, num_v_heads, need_split);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need)) return GDN_ERR_WORKSPACE;
  if (need > 0 && misaligned(workspace, 16)) return GDN_ERR_INVALID_ARGUMENT;  // 16-byte records

  PrefillArgs p{q,        k,     v,      state,      A_log,        a,           dt_bias,
                b,        cu_seqlens, cu_seqlens_int64 != 0, scale, output, new_state,
                (long long)total_tokens, num_seqs, num_q_heads, num_v_heads,
                use_qk_l2norm != 0, workspace, workspace_bytes};
  p.rs = rs;
  p.gates_pre = ext.gates_pre;
  p.g_alpha = ext.g_alpha;
  p.g_beta = ext.g_beta;
  if (ext.ckpt_every > 0) {
    p.ckpt = ext.ckpt;
    p.ckpt_starts = ext.ckpt_starts;
    p.ckpt_capacity = ext.ckpt_capacity;
    p.ckpt_every = ext.ckpt_every;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool chunked_ok = total_tokens > 0 && prefill_chunked_supported(p);
  int kind = variant;
  if (kind == GDN_PREFILL_AUTO)
    kind = !chunked_ok ? GDN_PREFILL_RECURRENT
                       : ((need_split || auto_uses_split(total_tokens, num_seqs, num_v_heads))
                              ? GDN_PREFILL_SPLIT
                              : GDN_PREFILL_FUSED);
  if ((kind == GDN_PREFILL_FUSED || kind == GDN_PREFILL_SPLIT) && !chunked_ok) {
    if (total_tokens > 0) return GDN_ERR_UNSUPPORTED;
    kind = GDN_PREFILL_RECURRENT;  // no tokens: only the zero final states to write
  }
  cudaError_t err;
  if (kind == GDN_PREFILL_SPLIT)
    err = launch_prefill_split(p, st);
  else if (kind == GDN_PREFILL_FUSED)
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
  return prefill_entry(GDN_PREFILL_AUTO, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
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
  return prefill_entry(GDN_PREFILL_RECURRENT, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                       cu_seqlens_int64, scale, output, new_state, total_tokens, num_seqs,
                       num_q_heads, num_k_heads, num_v_heads, head_size, use_qk_l2norm, workspace,
                       workspace_bytes, stream);
}

extern "C" int gdn_prefill_launch_variant(
    int variant, const void* q, const void* k, const void* v, const float* state,
    const float* A_log, const void* a, const float* dt_bias, const void* b,
    const void* cu_seqlens, int cu_seqlens_int64, float scale, void* output, float* new_state,
    int total_tokens, int num_seqs, int num_q_heads, int num_k_heads, int num_v_heads,
    int head_size, int use_qk_l2norm, void* workspace, size_t workspace_bytes, void* stream) {
  return prefill_entry(variant, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                       cu_seqlens_int64, scale, output, new_state, total_tokens, num_seqs,
                       num_q_heads, num_k_heads, num_v_heads, head_size, use_qk_l2norm, workspace,
                       workspace_bytes, stream);
}

extern "C" int gdn_prefill_launch_ext(
    int variant, const void* q, const void* k, const void* v, const float* state, int gate_mode,
    const float* A_log, const void* a, const float* dt_bias, const void* b, const float* g,
    const float* beta, const void* cu_seqlens, int cu_seqlens_int64, float scale, void* output,
    float* new_state, float* state_checkpoints, const long long* checkpoint_cu_starts,
    long long checkpoint_capacity, int checkpoint_every_n_tokens, int total_tokens, int num_seqs,
    int num_q_heads, int num_k_heads, int num_v_heads, int head_size, int use_qk_l2norm,
    void* workspace, size_t workspace_bytes, void* stream) {
  if (gate_mode != 0 && gate_mode != 1) return GDN_ERR_INVALID_ARGUMENT;
  PrefillExt ext;
  ext.gates_pre = gate_mode == 1;
  ext.g_alpha = g;
  ext.g_beta = beta;
  ext.ckpt = state_checkpoints;
  ext.ckpt_starts = checkpoint_cu_starts;
  ext.ckpt_capacity = checkpoint_capacity;
  ext.ckpt_every = checkpoint_every_n_tokens;
  return prefill_entry(variant, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                       cu_seqlens_int64, scale, output, new_state, total_tokens, num_seqs,
                       num_q_heads, num_k_heads, num_v_heads, head_size, use_qk_l2norm, workspace,
                       workspace_bytes, stream, ext);
}

extern "C" int gdn_device_error(int clear) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  const unsigned a = gdn::read_device_error(clear != 0);
  const unsigned b = gdn::read_split_device_error(clear != 0);
  const unsigned d = gdn::read_decode_device_error(clear != 0);
  const unsigned e = gdn::read_segment_device_error(clear != 0);
  const unsigned t = gdn::read_selftest_device_error(clear != 0);
  if (a == ~0u || b == ~0u || d == ~0u || e == ~0u || t == ~0u) return -1;
  return (int)(a | b | d | e | t);
}

extern "C" int gdn_prefill_launch_strided(
    int variant, const void* q, const void* k, const void* v, const float* state,
    const float* A_log, const void* a, const float* dt_bias, const void* b,
    const void* cu_seqlens, int cu_seqlens_int64, float scale, void* output, float* new_state,
    int total_tokens, int num_seqs, int num_q_heads, int num_k_heads, int num_v_heads,
    int head_size, int use_qk_l2norm, long long q_stride, long long k_stride,
    long long v_stride, long long a_stride, long long b_stride, long long output_stride,
    void* workspace, size_t workspace_bytes, void* stream) {
  const gdn::RowStrides rs{q_stride, k_stride, v_stride, a_stride, b_stride, output_stride};
  return prefill_entry(variant, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                       cu_seqlens_int64, scale, output, new_state, total_tokens, num_seqs,
                       num_q_heads, num_k_heads, num_v_heads, head_size, use_qk_l2norm, workspace,
                       workspace_bytes, stream, PrefillExt{}, &rs);
}
