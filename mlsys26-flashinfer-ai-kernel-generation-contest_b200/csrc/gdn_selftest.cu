// Self-test of the bounded-wait path (no counterpart in the reference).
//
// Every wait inside this library's kernels (TMA and bulk-copy completions, tensor-core
// commits, stage hand-offs) is an mbarrier poll with an iteration limit: when the limit
// runs out the kernel records a bit in a device-side error word, releases what it holds
// and returns, so a lost arrival can never hang the GPU.  gdn_selftest_bounded_wait runs
// that path on purpose, without any fault: one CTA waits, with the same bounded wait
// (sm100::mbar_wait), on an mbarrier that expects one arrival.  With `arrive` != 0 the
// waiting thread arrives first and the wait succeeds; with `arrive` == 0 nothing ever
// arrives, the wait gives up after `limit` polls, bit 16 of gdn_device_error is set and
// the kernel returns normally (the CUDA context stays usable).
#include <cuda_runtime.h>

#include "gdn_b200.h"
#include "gdn_prefill.cuh"
#include "sm100.cuh"

namespace gdn {
namespace {

__device__ unsigned int g_selftest_error = 0;
constexpr unsigned kErrSelfTestTimeout = 16u;

__global__ void selftest_wait_kernel(uint32_t limit, int arrive, int* result) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (arrive) sm100::mbar_arrive(&bar);
    const bool ok = sm100::mbar_wait(&bar, 0, limit);
    if (!ok) atomicOr(&g_selftest_error, kErrSelfTestTimeout);
    if (result != nullptr) *result = ok ? 1 : 0;
  }
}

}  // namespace

unsigned read_selftest_device_error(bool clear) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_selftest_error, sizeof(v)) != cudaSuccess) return ~0u;
  if (clear && v != 0) {
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_selftest_error, &zero, sizeof(zero)) != cudaSuccess) return ~0u;
  }
  return v;
}

}  // namespace gdn

extern "C" int gdn_selftest_bounded_wait(unsigned int limit, int arrive, int* result,
                                         void* stream) {
  if (limit == 0 || limit > (1u << 24)) return GDN_ERR_INVALID_ARGUMENT;
  if (result != nullptr && (reinterpret_cast<uintptr_t>(result) & 3u) != 0)
    return GDN_ERR_INVALID_ARGUMENT;
  gdn::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit, arrive,
                                                                           result);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
