// Shared device helpers for the GDN sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn_b200.h"

namespace gdn {

constexpr int kHeadDim = 128;
constexpr float kL2NormEps = 1e-6f;

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

// Four consecutive state values as fp32 from an fp32 state (one float4) or a bf16
// state (8 bytes, widened exactly); stores round to nearest bf16 for a bf16 state.
__device__ __forceinline__ float4 ld_state4(const float* p) { return ld_stream_f4(p); }
__device__ __forceinline__ float4 ld_state4(const __nv_bfloat16* p) {
  uint32_t x, y;
  asm volatile("ld.global.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(x), "=r"(y) : "l"(p));
  const float2 lo = bf2x2_to_f2(x), hi = bf2x2_to_f2(y);
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ void st_state4(float* p, float4 v) { st_stream_f4(p, v); }
__device__ __forceinline__ void st_state4(__nv_bfloat16* p, float4 v) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y);
  __nv_bfloat162 hi = __floats2bfloat162_rn(v.z, v.w);
  asm volatile("st.global.L1::no_allocate.v2.u32 [%0], {%1,%2};" ::"l"(p),
               "r"(*reinterpret_cast<uint32_t*>(&lo)), "r"(*reinterpret_cast<uint32_t*>(&hi))
               : "memory");
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
