// Longest-first (LPT) ordering of the sequences of a packed batch, on the device.
#pragma once

#include <stdint.h>

namespace gdn {
namespace {  // one instantiation per translation unit

// CTAs are scheduled roughly in blockIdx order and one CTA fills an SM, so
// handing out the longest sequences first (longest-processing-time) keeps the
// last wave short.  One CTA bitonic-sorts (length desc, index asc) keys in
// shared memory and writes the permutation.
constexpr int kLptMaxSeqs = 8192;

template <typename CuT>
__global__ void __launch_bounds__(1024) lpt_order_kernel(const CuT* __restrict__ cu, int N,
                                                         long long T, int* __restrict__ order) {
  extern __shared__ unsigned long long keys[];
  int P = 1;
  while (P < N) P <<= 1;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    unsigned long long key = 0ull;  // padding sorts last
    if (i < N) {
      const long long a = min(max((long long)cu[i], 0LL), T);
      const long long b = min(max((long long)cu[i + 1], 0LL), T);
      const unsigned long long len = (unsigned long long)max(b - a, 0LL);
      key = (len << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)i);
    }
    keys[i] = key;
  }
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long x = keys[i], y = keys[l];
          const bool desc = (i & k) == 0;  // descending overall
          if (desc ? (x < y) : (x > y)) {
            keys[i] = y;
            keys[l] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < N; i += blockDim.x)
    order[i] = (int)(0xFFFFFFFFu - (unsigned)(keys[i] & 0xFFFFFFFFull));
}

}  // namespace
}  // namespace gdn
