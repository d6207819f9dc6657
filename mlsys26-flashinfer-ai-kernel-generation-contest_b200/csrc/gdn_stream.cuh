// Shared-memory side of the streaming decode kernels: a state row or a bf16 vector
// staged in shared memory by a bulk copy, read into registers with the column ownership
// of RowSlice (the same columns, in the same order, as the one-shot kernels read from
// global memory, so that both give identical results).
#pragma once

#include "gdn_common.cuh"
#include "sm100.cuh"

namespace gdn {

// 16 columns of a state row held in shared memory (same column set as RowSlice)
template <typename ST>
__device__ __forceinline__ void load_row_smem(uint32_t row_addr, int j, float (&x)[16]) {
  using RS = RowSlice<ST>;
#pragma unroll
  for (int m = 0; m < RS::kChunks; ++m) {
    const uint4 u = sm100::ld_shared_v4(row_addr + (uint32_t)(RS::col(j, m) * sizeof(ST)));
    if constexpr (sizeof(ST) == 4) {
      x[4 * m] = __uint_as_float(u.x);
      x[4 * m + 1] = __uint_as_float(u.y);
      x[4 * m + 2] = __uint_as_float(u.z);
      x[4 * m + 3] = __uint_as_float(u.w);
    } else {
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = bf2x2_to_f2(w[e]);
        x[8 * m + 2 * e] = f.x;
        x[8 * m + 2 * e + 1] = f.y;
      }
    }
  }
}
// the lane's 16 columns of a bf16 vector in shared memory
template <typename ST>
__device__ __forceinline__ void load_vec_smem(uint32_t vec_addr, int j, float (&x)[16]) {
  using RS = RowSlice<ST>;
#pragma unroll
  for (int m = 0; m < RS::kChunks; ++m) {
    const uint32_t a = vec_addr + 2u * (uint32_t)RS::col(j, m);
    if constexpr (RS::kVec == 4) {
      uint32_t w0, w1;
      asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(w0), "=r"(w1) : "r"(a));
      const float2 f0 = bf2x2_to_f2(w0), f1 = bf2x2_to_f2(w1);
      x[4 * m] = f0.x; x[4 * m + 1] = f0.y; x[4 * m + 2] = f1.x; x[4 * m + 3] = f1.y;
    } else {
      const uint4 u = sm100::ld_shared_v4(a);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = bf2x2_to_f2(w[e]);
        x[8 * m + 2 * e] = f.x;
        x[8 * m + 2 * e + 1] = f.y;
      }
    }
  }
}

}  // namespace gdn
