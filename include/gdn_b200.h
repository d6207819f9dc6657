/*
 * gdn_b200.h -- C ABI of the B200 (sm_100a) Gated DeltaNet decode / prefill kernels.
 *
 * These entry points replace the two solution entry points of the reference
 * repository (flashinfer-bench "destination passing style" callables):
 *
 *   gdn_decode_launch   <- gdn_decode(q, k, v, state, A_log, a, dt_bias, b, scale,
 *                                      output, new_state)
 *                          gdn_decode/solution/triton/kernel.py:221-272
 *                          (entry point named in gdn_decode/config.toml:8)
 *   gdn_prefill_launch  <- gdn_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
 *                                       scale, output, new_state)
 *                          gdn_prefill/solution/triton/kernel.py:253-337
 *                          (entry point named in gdn_prefill/config.toml:8)
 *
 * and fill the empty CUDA template the reference ships for that purpose
 * (gdn_decode/solution/cuda/kernel.cu:13-20, binding.py:14-25).
 *
 * Conventions (all entry points):
 *   - Every tensor pointer is a DEVICE pointer to a dense, contiguous
 *     (row-major) buffer on the device that is current for the calling thread.
 *     bf16 tensors are passed as `const void*` / `void*` (IEEE bfloat16, 2 bytes).
 *   - head_size must be 128; num_q_heads == num_k_heads; num_v_heads is a
 *     multiple of num_q_heads (GVA: v-head h reads q/k head h / (HV/HQ)).
 *   - `state` may be NULL, meaning an all-zero initial state.
 *   - `scale` <= 0 (or NaN) means 1/sqrt(head_size), matching the reference's
 *     "scale is None or scale == 0.0" default.
 *   - `use_qk_l2norm` != 0 normalises q and k over head_dim in fp32,
 *     x * rsqrt(sum(x^2) + 1e-6), before use.  0 reproduces the reference
 *     (which does not normalise).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Launches are
 *     asynchronous; no entry point synchronises, allocates, or reads device
 *     memory on the host.
 *   - Return value: GDN_OK (0) or a negative GDN_ERR_* code.  Nothing is
 *     launched when an argument check fails.  No entry point aborts the process.
 *   - new_state may alias state (in-place update is supported); outputs must
 *     not otherwise overlap inputs.
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_OK 0
#define GDN_ERR_INVALID_ARGUMENT (-1) /* null pointer, bad size, misalignment     */
#define GDN_ERR_UNSUPPORTED (-2)      /* head_size != 128, bad head ratio, ...    */
#define GDN_ERR_LAUNCH (-3)           /* the CUDA launch itself reported an error */
#define GDN_ERR_WORKSPACE (-4)        /* workspace missing or too small           */
#define GDN_ERR_TOO_LARGE (-5)        /* beyond a fixed capacity (no-alloc entry) */

/* Library version, e.g. 100 for 0.1.0. */
int gdn_b200_version(void);

/* Human-readable name of a GDN_* status code (static storage). */
const char* gdn_status_string(int status);

/*
 * One decode step (seq_len == 1) for `batch` sequences.
 *   q       bf16 [batch, 1, num_q_heads, 128]
 *   k       bf16 [batch, 1, num_k_heads, 128]
 *   v       bf16 [batch, 1, num_v_heads, 128]
 *   state   fp32 [batch, num_v_heads, 128 (v), 128 (k)]  (k-last) or NULL
 *   A_log   fp32 [num_v_heads];  dt_bias fp32 [num_v_heads]
 *   a, b    bf16 [batch, 1, num_v_heads]
 *   output  bf16 [batch, 1, num_v_heads, 128]                       (written)
 *   new_state fp32 [batch, num_v_heads, 128, 128]                   (written)
 * Replaces gdn_decode_kernel (gdn_decode/solution/triton/kernel.py:71-218).
 * batch == 0 is a no-op that returns GDN_OK.
 */
int gdn_decode_launch(const void* q, const void* k, const void* v, const float* state,
                      const float* A_log, const void* a, const float* dt_bias, const void* b,
                      float scale, void* output, float* new_state, int batch,
                      int num_q_heads, int num_k_heads, int num_v_heads, int head_size,
                      int use_qk_l2norm, void* stream);

/*
 * gdn_decode_launch for q, k, v, a, b and output whose batch rows are strided, as the
 * reference's wrapper allows by handing every stride to its kernel
 * (gdn_decode/solution/triton/kernel.py:255-264): slices of a fused projection, say.
 * Each *_stride is the number of elements between consecutive batch rows of that
 * tensor; within a row the heads stay dense (head stride 128 for q, k, v and output,
 * 1 for a and b).  Rows of one tensor must not overlap (q/k/v/output strides >= heads *
 * 128, a/b strides >= num_v_heads) and q/k strides must be multiples of 4 (8-byte
 * rows); else GDN_ERR_INVALID_ARGUMENT.  Strides that keep every row 16-byte aligned
 * (multiples of 8) keep the fastest kernels available.  state and new_state stay dense.
 * The dense strides reproduce gdn_decode_launch exactly.
 */
int gdn_decode_launch_strided(const void* q, const void* k, const void* v, const float* state,
                              const float* A_log, const void* a, const float* dt_bias,
                              const void* b, float scale, void* output, float* new_state,
                              int batch, int num_q_heads, int num_k_heads, int num_v_heads,
                              int head_size, int use_qk_l2norm, long long q_stride,
                              long long k_stride, long long v_stride, long long a_stride,
                              long long b_stride, long long output_stride, void* stream);

/*
 * Multi-token decode (speculative-decoding verification): `seq_len` tokens per batch
 * row applied in order to the row's state in a pool, as the flashinfer-bench
 * definition `_gdn_mtp_reference` does (flashinfer/trace/templates/gdn.py:379-466;
 * FlashInfer's GPU API gated_delta_rule_mtp, flashinfer/gdn_decode.py:557).
 *   q, k          bf16 [batch, seq_len, num_q_heads, 128]
 *   v             bf16 [batch, seq_len, num_v_heads, 128]
 *   initial_state fp32 [pool_size, num_v_heads, 128 (v), 128 (k)] (k-last pool)
 *   state_indices int32 (state_indices_int64 == 0) or int64 [batch]: pool slot of each
 *                 row; a slot outside [0, pool_size) marks a padding row (zero
 *                 output, no state read or written)
 *   A_log, dt_bias fp32 [num_v_heads];  a, b bf16 [batch, seq_len, num_v_heads]
 *   output        bf16 [batch, seq_len, num_v_heads, 128]                 (written)
 *   final_state   fp32 [pool_size, num_v_heads, 128, 128]: slot state_indices[i]
 *                 receives row i's state after the last token; other slots are not
 *                 touched.  May be initial_state (in-place pool update).
 *   intermediate_states  fp32 [pool_size, seq_len, num_v_heads, 128, 128] or NULL:
 *                 slot state_indices[i], token t receives the state after token t
 * Rows must reference distinct slots (rows sharing a slot race on its final state).
 * Each slot is read once and written once; q/k/v/gates are read once.
 */
int gdn_mtp_launch(const void* q, const void* k, const void* v, const float* initial_state,
                   const void* state_indices, int state_indices_int64, const float* A_log,
                   const void* a, const float* dt_bias, const void* b, float scale,
                   void* output, float* final_state, float* intermediate_states, int batch,
                   int seq_len, int pool_size, int num_q_heads, int num_k_heads,
                   int num_v_heads, int head_size, int use_qk_l2norm, void* stream);

/*
 * bf16 state storage (the bf16-state backend of FlashInfer's decode,
 * flashinfer/gdn_decode.py:146-149): same contracts as gdn_decode_launch and
 * gdn_mtp_launch with state, new_state, the pool and the rollback buffer as bf16
 * (same shapes, 16-byte aligned).  The state is widened to fp32 on load, updated in
 * fp32 (across all tokens of a multi-token call) and rounded to nearest bf16 on every
 * store; the state traffic is half that of the fp32 entry points.  Decode calls with
 * at least 592 (batch x v-head) pairs, a non-NULL state and 16-byte aligned q, k, v
 * run a persistent streaming kernel (bulk copies into shared memory); its results are
 * bitwise those of the one-shot kernel used otherwise.  Its first call on a device sets
 * the kernel's shared-memory attribute (make it before any stream capture).
 */
int gdn_decode_launch_bf16state(const void* q, const void* k, const void* v, const void* state,
                                const float* A_log, const void* a, const float* dt_bias,
                                const void* b, float scale, void* output, void* new_state,
                                int batch, int num_q_heads, int num_k_heads, int num_v_heads,
                                int head_size, int use_qk_l2norm, void* stream);
int gdn_mtp_launch_bf16state(const void* q, const void* k, const void* v,
                             const void* initial_state, const void* state_indices,
                             int state_indices_int64, const float* A_log, const void* a,
                             const float* dt_bias, const void* b, float scale, void* output,
                             void* final_state, void* intermediate_states, int batch,
                             int seq_len, int pool_size, int num_q_heads, int num_k_heads,
                             int num_v_heads, int head_size, int use_qk_l2norm, void* stream);

/*
 * Bytes of device workspace gdn_prefill_launch needs for this problem (may be 0).
 */
size_t gdn_prefill_workspace_size(int total_tokens, int num_seqs, int num_q_heads,
                                  int num_v_heads, int head_size);

/*
 * Variable-length prefill over `num_seqs` packed sequences.
 *   q        bf16 [total_tokens, num_q_heads, 128]
 *   k        bf16 [total_tokens, num_k_heads, 128]
 *   v        bf16 [total_tokens, num_v_heads, 128]
 *   state    fp32 [num_seqs, num_v_heads, 128, 128] (k-last) or NULL
 *   A_log    fp32 [num_v_heads];  dt_bias fp32 [num_v_heads]
 *   a, b     bf16 [total_tokens, num_v_heads]
 *   cu_seqlens int32 (cu_seqlens_int64 == 0) or int64 [num_seqs + 1], on the device,
 *            non-decreasing, cu_seqlens[0] == 0, cu_seqlens[num_seqs] == total_tokens
 *   output   bf16 [total_tokens, max(num_q_heads, num_v_heads), 128]  (written)
 *   new_state fp32 [num_seqs, max(num_q_heads, num_v_heads), 128, 128] (written)
 *   workspace  device buffer of >= gdn_prefill_workspace_size(...) bytes, 16-byte
 *              aligned (cudaMalloc's alignment is more than enough)
 *              (may be NULL when that size is 0).  Scratch only: it holds the
 *              longest-first order in which the sequences are scheduled and,
 *              for the split kernels, the per-chunk records (33,808 bytes per
 *              64-token chunk and v-head); it is rewritten by every call and
 *              must not be shared by calls that overlap on the GPU.
 * A sequence of length 0 gets an all-zero new_state slice (as the
 * flashinfer-bench definition reference does).
 * One long sequence over few v-heads (split kernels, at least 64 chunks, SMs left idle by
 * the state kernel) runs in two pieces, the second piece's preparation on a library-owned
 * side stream overlapping the first piece's state kernel; `stream` waits for it before the
 * call's last kernel (event fork / join).  The first such call on a device creates that
 * side stream and two events: make it before capturing the stream into a CUDA graph.
 * Replaces gdn_prefill_chunk_kernel (gdn_prefill/solution/triton/kernel.py:28-250)
 * and its host wrapper's zero-fill / state copy passes (:281-299).
 */
int gdn_prefill_launch(const void* q, const void* k, const void* v, const float* state,
                       const float* A_log, const void* a, const float* dt_bias, const void* b,
                       const void* cu_seqlens, int cu_seqlens_int64, float scale,
                       void* output, float* new_state, int total_tokens, int num_seqs,
                       int num_q_heads, int num_k_heads, int num_v_heads, int head_size,
                       int use_qk_l2norm, void* workspace, size_t workspace_bytes,
                       void* stream);

/*
 * Same contract as gdn_prefill_launch, but always runs the token-serial
 * recurrent CUDA-core kernel (the definition's per-token recurrence, exact to
 * fp32 rounding) instead of the chunked tensor-core kernel.  For validation
 * and for callers whose buffers do not meet the chunked kernel's 16-byte
 * alignment.  `workspace` is ignored.  Same reference interface as
 * gdn_prefill_launch.
 */
int gdn_prefill_launch_recurrent(const void* q, const void* k, const void* v, const float* state,
                                 const float* A_log, const void* a, const float* dt_bias,
                                 const void* b, const void* cu_seqlens, int cu_seqlens_int64,
                                 float scale, void* output, float* new_state, int total_tokens,
                                 int num_seqs, int num_q_heads, int num_k_heads, int num_v_heads,
                                 int head_size, int use_qk_l2norm, void* workspace,
                                 size_t workspace_bytes, void* stream);

/*
 * Prefill kernel selection (no counterpart in the reference), for validation
 * and benchmarking of the individual kernels:
 *   GDN_PREFILL_AUTO       what gdn_prefill_launch runs for these sizes
 *   GDN_PREFILL_RECURRENT  token-serial CUDA-core kernel (same as
 *                          gdn_prefill_launch_recurrent; no workspace)
 *   GDN_PREFILL_FUSED      chunked tensor-core kernel, one CTA per
 *                          (sequence, v-head) for the whole scan
 *   GDN_PREFILL_SPLIT      chunk-parallel preparation kernel + sequential
 *                          state kernel per (sequence, v-head, 64-row v-block)
 * FUSED and SPLIT need 16-byte aligned q, k, v and output (else
 * GDN_ERR_UNSUPPORTED); AUTO falls back to RECURRENT in that case.
 */
#define GDN_PREFILL_AUTO 0
#define GDN_PREFILL_RECURRENT 1
#define GDN_PREFILL_FUSED 2
#define GDN_PREFILL_SPLIT 3

/* Workspace bytes of gdn_prefill_launch_variant(variant, ...) for this problem. */
size_t gdn_prefill_workspace_size_variant(int variant, int total_tokens, int num_seqs,
                                          int num_q_heads, int num_v_heads, int head_size);

/* gdn_prefill_launch with an explicit kernel choice (GDN_PREFILL_*). */
int gdn_prefill_launch_variant(int variant, const void* q, const void* k, const void* v,
                               const float* state, const float* A_log, const void* a,
                               const float* dt_bias, const void* b, const void* cu_seqlens,
                               int cu_seqlens_int64, float scale, void* output,
                               float* new_state, int total_tokens, int num_seqs,
                               int num_q_heads, int num_k_heads, int num_v_heads, int head_size,
                               int use_qk_l2norm, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * Prefill with the options of FlashInfer's chunk_gated_delta_rule
 * (flashinfer/gdn_prefill.py:99-185), otherwise the gdn_prefill_launch_variant
 * contract:
 *   gate_mode 0: gates from A_log, a, dt_bias, b as in gdn_prefill_launch (g, beta
 *                ignored);
 *   gate_mode 1: precomputed fp32 [total_tokens, num_v_heads] decay g (alpha in [0, 1],
 *                the forget gate itself) and beta; NULL means all ones; A_log, a,
 *                dt_bias, b are ignored (may be NULL).
 *   checkpoint_every_n_tokens = N > 0 (a multiple of 64): the state after every N tokens
 *                of sequence i goes to state_checkpoints[checkpoint_cu_starts[i] + j]
 *                (fp32 [num_v_heads, 128, 128] each, j < len_i / N); entries at or beyond
 *                checkpoint_capacity are not written.  N = 0: no checkpoints (the three
 *                checkpoint pointers may be NULL).
 * With raw (un-normalised) q/k and either option, GDN_PREFILL_AUTO runs the split
 * kernels and GDN_PREFILL_FUSED returns GDN_ERR_UNSUPPORTED.
 */
size_t gdn_prefill_workspace_size_ext(int variant, int total_tokens, int num_seqs,
                                      int num_q_heads, int num_v_heads, int head_size,
                                      int use_qk_l2norm, int gate_mode,
                                      int checkpoint_every_n_tokens);
int gdn_prefill_launch_ext(int variant, const void* q, const void* k, const void* v,
                           const float* state, int gate_mode, const float* A_log, const void* a,
                           const float* dt_bias, const void* b, const float* g,
                           const float* beta, const void* cu_seqlens, int cu_seqlens_int64,
                           float scale, void* output, float* new_state, float* state_checkpoints,
                           const long long* checkpoint_cu_starts, long long checkpoint_capacity,
                           int checkpoint_every_n_tokens, int total_tokens, int num_seqs,
                           int num_q_heads, int num_k_heads, int num_v_heads, int head_size,
                           int use_qk_l2norm, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * gdn_prefill_launch_variant for q, k, v, a, b and output whose token rows are
 * strided, as the reference's wrapper allows by handing every stride to its kernel
 * (gdn_prefill/solution/triton/kernel.py:318-325): slices of a fused QKV projection,
 * say.  Each *_stride is the number of elements between consecutive tokens of that
 * tensor; within a token the heads stay dense (head stride 128 for q, k, v and output,
 * 1 for a and b).  Rows of one tensor must not overlap (q/k/v/output strides >= heads *
 * 128, a/b strides >= num_v_heads) and q/k strides must be multiples of 4; else
 * GDN_ERR_INVALID_ARGUMENT.  The tensor-core kernels (GDN_PREFILL_FUSED / _SPLIT) also
 * need q/k/v/output strides that are multiples of 8 (16-byte rows): otherwise they
 * return GDN_ERR_UNSUPPORTED and GDN_PREFILL_AUTO runs the token-serial kernel.  The
 * dense strides reproduce gdn_prefill_launch_variant exactly.
 */
int gdn_prefill_launch_strided(int variant, const void* q, const void* k, const void* v,
                               const float* state, const float* A_log, const void* a,
                               const float* dt_bias, const void* b, const void* cu_seqlens,
                               int cu_seqlens_int64, float scale, void* output,
                               float* new_state, int total_tokens, int num_seqs,
                               int num_q_heads, int num_k_heads, int num_v_heads, int head_size,
                               int use_qk_l2norm, long long q_stride, long long k_stride,
                               long long v_stride, long long a_stride, long long b_stride,
                               long long output_stride, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * Allocation-free variant of gdn_prefill_launch (no counterpart in the
 * reference).  For callers that cannot allocate device memory where they
 * launch -- inside an allocator or memory-pool callback, under a runtime
 * whose device memory is fully pre-reserved, or in a plugin host that hands
 * the kernel only its inputs and outputs -- it takes no workspace and uses a
 * 16 KiB scratch array compiled into the library instead.
 *   - Same arguments and results as gdn_prefill_launch, minus the workspace.
 *   - num_seqs is limited to 4096; larger requests return GDN_ERR_TOO_LARGE
 *     and launch nothing.
 *   - The first call on each device looks up the scratch array's device
 *     address (cudaGetSymbolAddress); make that first call before capturing
 *     a stream.  No call allocates or frees memory.
 *   - All calls on a device share the scratch array: calls that overlap on
 *     the GPU (e.g. on two streams) race and must not be issued that way.
 */
int gdn_prefill_launch_noalloc(const void* q, const void* k, const void* v, const float* state,
                               const float* A_log, const void* a, const float* dt_bias,
                               const void* b, const void* cu_seqlens, int cu_seqlens_int64,
                               float scale, void* output, float* new_state, int total_tokens,
                               int num_seqs, int num_q_heads, int num_k_heads, int num_v_heads,
                               int head_size, int use_qk_l2norm, void* stream);

/*
 * Segment-scan output assembly (multi-GPU prefill of one long sequence split
 * into token segments; no counterpart in the reference, whose prefill walks a
 * sequence on one device).  Over a segment the outputs are affine in the
 * segment's start state S: o_t = S o^I_t + o^0_t, with o^I the segment's
 * output from the identity state with v = 0 and o^0 its output from a zero
 * state (both from ordinary prefill calls).  This forms, on `stream`,
 *   output[t][h][v] = bf16( sum_j start_state[h][v][j] o_identity[t][h][j]
 *                           + o_zero[t][h][v] )
 * for t < num_tokens, h < num_v_heads.  Layouts: o_identity, o_zero, output
 * [num_tokens, num_v_heads, head_size] bf16, 16-byte aligned;
 * start_state [num_v_heads, head_size, head_size] fp32 (k-last), 16-byte
 * aligned.  start_state is split into bf16 hi + lo in the kernel, so the sum
 * carries fp32-level precision in S.  head_size must be 128.
 */
int gdn_segment_outputs_launch(const void* o_identity, const void* o_zero,
                               const float* start_state, void* output, int num_tokens,
                               int num_v_heads, int head_size, void* stream);

/*
 * Segment-scan state chain (same multi-GPU scan; no counterpart in the
 * reference).  maps holds every segment's state map as all-gathered,
 * [num_maps][2][num_v_heads][head_size][head_size] fp32 (A_m then B_m; a
 * segment maps S to S A_m + B_m, and segment 0's entry is (unused, its final
 * state)).  For segment `rank` (1 <= rank < num_maps) this writes, on
 * `stream`, its start state S = (..(B_0 A_1 + B_1) A_2 + ..) A_{rank-1} +
 * B_{rank-1} and its final state S A_rank + B_rank, both
 * [num_v_heads][head_size][head_size] fp32, in fp32 arithmetic.  All pointers
 * 16-byte aligned; head_size must be 128.
 */
int gdn_segment_chain_launch(const float* maps, int num_maps, int rank, float* start_state,
                             float* final_state, int num_v_heads, int head_size,
                             void* stream);

/*
 * The same chain for every segment in one pass (no counterpart in the reference): with
 * maps as for gdn_segment_chain_launch, writes start_states[s - 1] = the start state of
 * segment s for s = 1 .. num_maps - 1 ([num_maps - 1][num_v_heads][head_size][head_size]
 * fp32) and final_state = the last segment's final state, in num_maps - 1 steps instead
 * of one chain per segment.  Used when every segment of a sequence is assembled on one
 * GPU (the segments of one call run side by side).  num_maps >= 2; all pointers 16-byte
 * aligned; head_size must be 128.
 */
int gdn_segment_chain_all_launch(const float* maps, int num_maps, float* start_states,
                                 float* final_state, int num_v_heads, int head_size,
                                 void* stream);

/*
 * Prefill of ONE sequence as token segments that run side by side (no counterpart in the
 * reference, whose prefill walks each sequence's chunks in order,
 * gdn_prefill/solution/triton/kernel.py:122-247).  For a sequence whose v-heads alone
 * leave most SMs idle (one sequence of a model sharded by q/k-head group over GPUs), the
 * total_tokens tokens are cut into S segments on 64-token chunk boundaries; one launch of
 * the split kernels runs segment 0 from `state` and every later segment twice (from zero,
 * and from the identity with v = 0), reading the tokens in place; the state-map chain and
 * the output kernel (see gdn_segment_chain_launch / gdn_segment_outputs_launch) then give
 * every segment's start state, the outputs o = S_start o^I + o^0 and the final state.
 * Same arguments and meaning as gdn_prefill_launch_strided for one sequence
 * (cu_seqlens = [0, total_tokens]): q, k [total_tokens, num_q_heads, 128], v
 * [total_tokens, num_v_heads, 128], a, b [total_tokens, num_v_heads] bf16 with the given
 * token strides (elements; q / k / v rows 16-byte aligned), state / new_state
 * [1, num_v_heads, 128, 128] fp32 (state may be NULL = zero, and may equal new_state),
 * output [total_tokens, num_v_heads, 128] bf16 dense and 16-byte aligned.  segments > 0
 * cuts S equal segments (capped at the number of chunks and at 64); segments = 0 takes
 * the plan of gdn_prefill_segment_plan for the current device; segment_bounds (host
 * memory, may be NULL) gives the bounds of segments = S > 0 segments instead: S + 1 token
 * offsets, 0 first, total_tokens last, strictly increasing, interior ones multiples of 64
 * (else GDN_ERR_INVALID_ARGUMENT; the workspace size function takes the same pair and
 * returns 0 for invalid bounds).  S = 1 is an ordinary split-kernel prefill.  The outputs of later segments carry one more
 * bf16 rounding (of o^I); the final state is fp32 throughout.  workspace (1024-byte
 * aligned) of gdn_prefill_segmented_workspace_size bytes; asynchronous on `stream`.
 */
int gdn_prefill_segments_auto(int total_tokens, int num_v_heads);
/*
 * The segment bounds gdn_prefill_segmented_launch uses: returns S and writes
 * bounds[0..S] (token offsets, bounds[0] = 0, bounds[S] = total_tokens; up to `capacity`
 * entries).  segments > 0: S equal shares of the 64-token chunks (capped at the chunks and
 * at 64).  segments = 0: the plan of a cost model of the kernels on num_sms SMs (<= 0: the
 * current device's): segment 0 of x chunks and S - 1 equal later segments, S <= 16 and x
 * chosen to minimise the modelled time; one segment unless that saves at least 5 %.
 */
int gdn_prefill_segment_plan(int total_tokens, int num_v_heads, int segments, int num_sms,
                             int* bounds, int capacity);
size_t gdn_prefill_segmented_workspace_size(int total_tokens, int num_v_heads, int segments,
                                            const int* segment_bounds);
int gdn_prefill_segmented_launch(const void* q, const void* k, const void* v, const float* state,
                                 const float* A_log, const void* a, const float* dt_bias,
                                 const void* b, float scale, void* output, float* new_state,
                                 int total_tokens, int num_q_heads, int num_k_heads,
                                 int num_v_heads, int head_size, int use_qk_l2norm, int segments,
                                 const int* segment_bounds, long long q_stride,
                                 long long k_stride, long long v_stride,
                                 long long a_stride, long long b_stride, void* workspace,
                                 size_t workspace_bytes, void* stream);

/*
 * Diagnostics: synchronises the current device and returns the device-side
 * error bits recorded by the kernels since the last call (0 = none; 1 = a TMA
 * or bulk-copy wait ran out, 2 = a tensor-core wait ran out, 8 = a shared-memory
 * stage of the streaming decode kernel was never released, 16 = the wait of
 * gdn_selftest_bounded_wait ran out; -1 = the device reported an error).  Every wait inside the kernels is bounded; a wait that runs out sets
 * a bit, the kernel releases its resources and returns instead of hanging.
 * The bits are cleared when `clear` != 0.  No counterpart in the reference.
 */
int gdn_device_error(int clear);

/*
 * Self-test of the bounded-wait path (no counterpart in the reference): one CTA waits,
 * with the same iteration-limited mbarrier wait every kernel of this library uses, on a
 * barrier that expects one arrival.  arrive != 0: the waiting thread arrives first and
 * the wait succeeds.  arrive == 0: nothing ever arrives, the wait gives up after `limit`
 * polls (1 <= limit <= 2^24), bit 16 of gdn_device_error is set and the kernel returns
 * normally -- the context stays usable.  `result` (device int, may be NULL) receives 1
 * when the wait succeeded, 0 when it ran out.  Asynchronous on `stream`.
 */
int gdn_selftest_bounded_wait(unsigned int limit, int arrive, int* result, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* GDN_B200_H_ */
