// Shared device helpers for the GDN sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn_b200.h"

namespace gdn {

constexpr int kHeadDim = 128;
constexpr float kL2NormEps = 1e-6f;

// Elements between consecutive rows (tokens in prefill, batch rows in decode) of the
// token-indexed tensors; within a row the heads are dense (head stride 128 for q, k, v
// and the output, 1 for a and b).  Dense tensors have q = HQ * 128, a = HV, ...
struct RowStrides {
  long long q, k, v, a, b, o;
};
inline RowStrides dense_rows(int HQ, int HV) {
  return RowStrides{(long long)HQ * kHeadDim, (long long)HQ * kHeadDim, (long long)HV * kHeadDim,
                    (long long)HV,            (long long)HV,            (long long)HV * kHeadDim};
}

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }

// Two packed bf16 (low half first in memory) -> two floats.
__device__ __forceinline__ float2 bf2x2_to_f2(uint32_t u) {
  float2 r;
  r.x = __uint_as_float(u << 16);
  r.y = __uint_as_float(u & 0xffff0000u);
  return r;
}

// Per-token gates, fp32, as the definition reference computes them:
//   g = exp(-exp(A_log) * softplus(a + dt_bias)),  softplus(x) = x for x > 20
//   beta = sigmoid(b)
// (flashinfer/trace/templates/gdn.py:51-53; reference decode kernel.py:122-131)
__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float gate_log_g(float A_log, float a, float dt_bias) {
  return -expf(A_log) * softplus_f(a + dt_bias);
}
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }
// log of a precomputed decay alpha in [0, 1]; alpha = 0 (full forget) maps to
// log(1e-38) ~ -87.5, whose exponential is 0 in fp32
__device__ __forceinline__ float log_alpha(float alpha) { return logf(fmaxf(alpha, 1e-38f)); }

// Slot of the checkpoint after `tokens` tokens of sequence n (every `every` tokens),
// or -1 when none is due or it falls outside [0, capacity).
__device__ __forceinline__ long long checkpoint_slot(const long long* starts, int n,
                                                     long long tokens, int every,
                                                     long long capacity) {
  if (every <= 0 || tokens <= 0 || tokens % every != 0) return -1;
  const long long ci = starts[n] + tokens / every - 1;
  return (ci >= 0 && ci < capacity) ? ci : -1;
}

// Streaming 128-bit global accesses: the state is touched exactly once.
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
  asm volatile("st.global.L1::no_allocate.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// The 16 columns one of the 8 lanes of a state row owns, accessed 16 bytes at a time
// so that every warp-wide access covers whole 128-byte segments: kVec = 4 fp32 or 8 bf16
// columns per access at col(m) = kVec*j + 8*kVec*m (m < kChunks), element e of access m
// held in x[kVec*m + e].  q and k are read with the same column set.
template <typename ST>
struct RowSlice {
  static constexpr int kVec = 16 / (int)sizeof(ST);
  static constexpr int kChunks = 16 / kVec;
  __device__ static __forceinline__ int col(int j, int m) { return kVec * j + 8 * kVec * m; }
  __device__ static __forceinline__ void load(const ST* row, int j, float (&x)[16]);
  __device__ static __forceinline__ void store(ST* row, int j, const float (&x)[16]);
  // columns of a bf16 vector (q or k), widened
  __device__ static __forceinline__ void load_bf16(const __nv_bfloat16* vec, int j,
                                                   float (&x)[16]) {
#pragma unroll
    for (int m = 0; m < kChunks; ++m) {
      const __nv_bfloat16* p = vec + col(j, m);
      if constexpr (kVec == 4) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
        const float2 a = bf2x2_to_f2(u.x), b = bf2x2_to_f2(u.y);
        x[4 * m] = a.x; x[4 * m + 1] = a.y; x[4 * m + 2] = b.x; x[4 * m + 3] = b.y;
      } else {  // two 8-byte loads: q and k rows need only 8-byte alignment
        const uint2 u0 = __ldg(reinterpret_cast<const uint2*>(p));
        const uint2 u1 = __ldg(reinterpret_cast<const uint2*>(p + 4));
        const uint32_t w[4] = {u0.x, u0.y, u1.x, u1.y};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = bf2x2_to_f2(w[e]);
          x[8 * m + 2 * e] = f.x;
          x[8 * m + 2 * e + 1] = f.y;
        }
      }
    }
  }
};
template <>
__device__ __forceinline__ void RowSlice<float>::load(const float* row, int j, float (&x)[16]) {
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float4 v = ld_stream_f4(row + col(j, m));
    x[4 * m] = v.x; x[4 * m + 1] = v.y; x[4 * m + 2] = v.z; x[4 * m + 3] = v.w;
  }
}
template <>
__device__ __forceinline__ void RowSlice<float>::store(float* row, int j, const float (&x)[16]) {
#pragma unroll
  for (int m = 0; m < 4; ++m)
    st_stream_f4(row + col(j, m), make_float4(x[4 * m], x[4 * m + 1], x[4 * m + 2], x[4 * m + 3]));
}
template <>
__device__ __forceinline__ void RowSlice<__nv_bfloat16>::load(const __nv_bfloat16* row, int j,
                                                              float (&x)[16]) {
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    uint32_t w[4];
    asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                 : "l"(row + col(j, m)));
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = bf2x2_to_f2(w[e]);
      x[8 * m + 2 * e] = f.x;
      x[8 * m + 2 * e + 1] = f.y;
    }
  }
}
template <>
__device__ __forceinline__ void RowSlice<__nv_bfloat16>::store(__nv_bfloat16* row, int j,
                                                               const float (&x)[16]) {
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(x[8 * m + 2 * e], x[8 * m + 2 * e + 1]);
      w[e] = *reinterpret_cast<uint32_t*>(&b2);
    }
    asm volatile("st.global.L1::no_allocate.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(row + col(j, m)),
                 "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                 : "memory");
  }
}

__device__ __forceinline__ float xor_sum8(float x) {
  // Sum over the 8 lanes of an aligned 8-lane group.
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  return x;
}

__host__ __device__ inline float default_scale(float scale) {
  // scale <= 0 or NaN -> 1/sqrt(128)
  return (scale > 0.f) ? scale : 0.08838834764831845f;
}

}  // namespace gdn
