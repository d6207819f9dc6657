// Internal interface between the prefill C-ABI entry point and its kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

#include <climits>

#include "gdn_common.cuh"

namespace gdn {

struct PrefillArgs {
  const void* q;
  const void* k;
  const void* v;
  const float* state;  // may be null (zero initial state)
  const float* A_log;
  const void* a;
  const float* dt_bias;
  const void* b;
  const void* cu;  // int32 or int64 [N+1]
  bool cu_int64;
  float scale;
  void* out;
  float* new_state;
  long long T;
  int N;
  int HQ;
  int HV;
  bool l2norm;
  void* workspace;
  size_t workspace_bytes;
  // precomputed gates instead of (A_log, a, b, dt_bias): fp32 [T, HV] decay alpha = g
  // and beta, a null pointer meaning all ones
  bool gates_pre = false;
  const float* g_alpha = nullptr;
  const float* g_beta = nullptr;
  // state after every ckpt_every tokens of each sequence (0 = off) into
  // ckpt[ckpt_starts[n] + i] (fp32 [HV, 128, 128] each), i < len_n / ckpt_every;
  // indices outside [0, ckpt_capacity) are not written
  float* ckpt = nullptr;
  const long long* ckpt_starts = nullptr;
  long long ckpt_capacity = 0;
  int ckpt_every = 0;
  // token strides of q, k, v, a, b and the output (elements); dense when not set by the
  // caller (the entry point fills them in)
  RowStrides rs{};
  // segmented call of one sequence (split kernels only; gdn_prefill_segmented_launch): the
  // runs' token rows are virtual, T of them, over src_rows rows of q, k, v, a, b.  Rows
  // r >= vsplit belong to the identity runs: they read input row r - vsplit + vsrc, take
  // v = 0, start from the identity state and write their outputs to out_alt row
  // r - vsplit.  Only runs n < state_runs start from `state`; the others from zero.
  long long src_rows = 0;
  long long vsplit = LLONG_MAX;
  long long vsrc = 0;
  void* out_alt = nullptr;
  int state_runs = INT_MAX;
  // Only runs n < prep_runs get their per-chunk records prepared; an identity run reads
  // the records of run n - rec_alias (it covers the same tokens as that run).
  int prep_runs = INT_MAX;
  int rec_alias = 0;
  // Chunk offsets [N + 1] and longest-first sequence order [N] already written to device
  // memory by the caller on the same stream (null: computed on the device from cu).
  const int* ready_base = nullptr;
  const int* ready_order = nullptr;
};

// Token-serial recurrent kernel over sequences [seq_offset, seq_offset + nseq).
cudaError_t launch_prefill_recurrent(const PrefillArgs& p, int seq_offset, int nseq,
                                     cudaStream_t st);

// Chunked tcgen05 kernel (all sequences).  Needs T > 0, 16-byte aligned q/k/v/out
// and the driver's tensor-map encoder.
bool prefill_chunked_supported(const PrefillArgs& p);
// Scratch bytes the chunked path uses for its longest-first sequence order.
size_t prefill_chunked_workspace(int num_seqs);
cudaError_t launch_prefill_chunked(const PrefillArgs& p, cudaStream_t st);

// TMA descriptor of a [rows][heads * 128] bf16 matrix whose rows are `row_stride`
// elements apart (a multiple of 8), with 64 x 64 boxes and the 128-byte swizzle (false if
// the driver's encoder is unavailable or refuses it).
bool make_tile_map(CUtensorMap* m, const void* base, int heads, long long rows,
                   long long row_stride);
// Same with `box_x` (<= 64) columns per box, 128-byte swizzle or none.
bool make_tile_map_box(CUtensorMap* m, const void* base, int heads, long long rows,
                       long long row_stride, int box_x, bool swizzle128);

// Split path: a chunk-parallel preparation kernel and a sequential state kernel
// split over v-blocks.  Same requirements as the chunked kernel; the workspace
// holds the per-chunk records.
size_t prefill_split_workspace(long long T, int num_seqs, int HV);
cudaError_t launch_prefill_split(const PrefillArgs& p, cudaStream_t st);
unsigned read_split_device_error(bool clear);

// Segment-scan kernels (gdn_segment.cu).  The state-map chain over maps A_m =
// maps[a0 + m as], B_m = maps[b0 + m bs] (matrices of HV heads): segment `rank`'s start
// and final states, and with starts_all every segment s's start state at starts_all[s - 1].
cudaError_t launch_segment_chain(const float* maps, int a0, int as, int b0, int bs, int rank,
                                 int HV, float* start_out, float* final_out, float* starts_all,
                                 cudaStream_t s);
// Outputs of nseg segments in one launch (segment s: rows [off[s], off[s] + len[s]) of o^I,
// o^0 and the output, start state start_states[s]); o_zero may be the output itself.
cudaError_t launch_segment_outputs(const void* o_identity, long long rows_id, const void* o_zero,
                                   long long rows_zero, const float* start_states, void* output,
                                   int nseg, const int* off, const int* len, int HV,
                                   cudaStream_t s);

// Device-side error flag set by a bounded wait that ran out (0 = none).
unsigned read_device_error(bool clear);
// Same for the streaming decode kernel.
unsigned read_decode_device_error(bool clear);
unsigned read_segment_device_error(bool clear);
// Same for the bounded-wait self-test kernel (gdn_selftest_bounded_wait).
unsigned read_selftest_device_error(bool clear);

}  // namespace gdn
