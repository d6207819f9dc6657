// Allocation-free prefill entry point.
//
// gdn_prefill_launch needs a small device scratch buffer (the longest-first
// order in which sequences are scheduled), which its callers allocate and
// pass in.  Some callers cannot allocate device memory at the point where
// they launch: code running inside a custom allocator or memory-pool
// callback, runtimes whose device memory is fully pre-reserved by another
// allocator, and plugin hosts that hand a kernel only its input and output
// buffers.  For them, gdn_prefill_launch_noalloc takes no workspace argument
// and uses a fixed scratch array compiled into this library instead.
//
// The scratch is the file-scope array below: kNoAllocMaxSeqs ints (16 KiB),
// held by every GPU that loads the library until the process exits.  Host
// code cannot use the array's name as a device address, so the first call on
// each device looks the address up with cudaGetSymbolAddress (with that
// device current) and caches it; make that first call before capturing a
// stream.  No call allocates or frees memory.
//
// Every call on a device shares the one array and leaves its last contents
// behind.  Each call rewrites all entries it reads before reading them, so
// nothing has to start at zero, but two calls that overlap on the GPU (for
// example on two streams) race on the array and must not be issued that way.
#include <cuda_runtime.h>

#include "gdn_b200.h"

namespace {

constexpr int kNoAllocMaxSeqs = 4096;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) int g_noalloc_scratch[kNoAllocMaxSeqs];

// Device address of g_noalloc_scratch on the current device (looked up once
// per device), or nullptr if the lookup failed.
void* noalloc_scratch_address() {
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace

extern "C" int gdn_prefill_launch_noalloc(const void* q, const void* k, const void* v,
                                          const float* state, const float* A_log, const void* a,
                                          const float* dt_bias, const void* b,
                                          const void* cu_seqlens, int cu_seqlens_int64,
                                          float scale, void* output, float* new_state,
                                          int total_tokens, int num_seqs, int num_q_heads,
                                          int num_k_heads, int num_v_heads, int head_size,
                                          int use_qk_l2norm, void* stream) {
  if (num_seqs > kNoAllocMaxSeqs) return GDN_ERR_TOO_LARGE;
  // the fused chunked kernel: its only scratch is the sequence order (4 bytes each)
  const size_t need = gdn_prefill_workspace_size_variant(GDN_PREFILL_FUSED, total_tokens,
                                                         num_seqs, num_q_heads, num_v_heads,
                                                         head_size);
  if (need > sizeof(int) * (size_t)kNoAllocMaxSeqs) return GDN_ERR_TOO_LARGE;
  void* scratch = nullptr;
  if (need > 0) {
    scratch = noalloc_scratch_address();
    if (scratch == nullptr) return GDN_ERR_LAUNCH;
  }
  const size_t bytes = scratch ? sizeof(int) * (size_t)kNoAllocMaxSeqs : 0;
  const int rc = gdn_prefill_launch_variant(
      GDN_PREFILL_FUSED, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, cu_seqlens_int64,
      scale, output, new_state, total_tokens, num_seqs, num_q_heads, num_k_heads, num_v_heads,
      head_size, use_qk_l2norm, scratch, bytes, stream);
  if (rc != GDN_ERR_UNSUPPORTED) return rc;
  // buffers the chunked kernel cannot take (alignment): the token-serial kernel
  return gdn_prefill_launch_variant(GDN_PREFILL_RECURRENT, q, k, v, state, A_log, a, dt_bias, b,
                                    cu_seqlens, cu_seqlens_int64, scale, output, new_state,
                                    total_tokens, num_seqs, num_q_heads, num_k_heads, num_v_heads,
                                    head_size, use_qk_l2norm, nullptr, 0, stream);
}
