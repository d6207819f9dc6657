// Output assembly of the segment-level scan (one long sequence split into token segments,
// one per GPU).  Over a segment the outputs are affine in the segment's start state S
// (k-last [v][j] per v-head): o_t = S o^I_t + o^0_t, where o^I is the output of the segment
// run from the identity state with v = 0 and o^0 its output from a zero state.  Once the
// start state is known (after the exchange of the segments' state maps), this kernel forms
//     out[t][h][v] = bf16( sum_j S[h][v][j] o^I[t][h][j] + o^0[t][h][v] )
// in one pass over o^I and o^0.
//
// One CTA per (128-token tile, v-head), 8 warps of 16 tokens each.  S[h] is split once per
// CTA into bf16 hi + lo (S = hi + lo to ~2^-17 relative) in shared memory; o^I is bf16
// already, so the products run as bf16 tensor-core fragments (m16n8k16, fp32 accumulate),
// two per output tile (hi and lo).  Rows are padded to 136 elements so that the fragment
// reads of the 32 lanes fall into 32 distinct banks.  The kernel moves
// 3 x T x HV x 128 x 2 bytes (o^I and o^0 in, out) and is HBM-bound.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn_b200.h"

namespace {

constexpr int kD = 128;
constexpr int kTile = 128;               // tokens per CTA
constexpr int kWarps = kTile / 16;
constexpr int kThreads = 32 * kWarps;
constexpr int kLd = kD + 8;              // padded row (bf16 elements)
constexpr size_t kSmem = (size_t)(2 * kD + kTile) * kLd * sizeof(__nv_bfloat16);

__device__ __forceinline__ uint32_t lds32(const __nv_bfloat16* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kThreads, 2)
    segment_outputs_kernel(const __nv_bfloat16* __restrict__ o_id,
                           const __nv_bfloat16* __restrict__ o_zero,
                           const float* __restrict__ start, __nv_bfloat16* __restrict__ out,
                           int L, int HV) {
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* shi = reinterpret_cast<__nv_bfloat16*>(smem);  // [v][j]
  __nv_bfloat16* slo = shi + kD * kLd;
  __nv_bfloat16* oit = slo + kD * kLd;                           // [t][j]
  const int h = blockIdx.y;
  const int t0 = blockIdx.x * kTile;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // S[h] -> hi | lo (fp32 rows of 128, four elements per load)
  const float4* s4 = reinterpret_cast<const float4*>(start + (size_t)h * kD * kD);
  for (int i = tid; i < kD * kD / 4; i += kThreads) {
    const float4 x = __ldg(s4 + i);
    const int v = i >> 5, j = (i & 31) * 4;
    const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(xs[e]);
      shi[v * kLd + j + e] = hi;
      slo[v * kLd + j + e] = __float2bfloat16_rn(xs[e] - __bfloat162float(hi));
    }
  }
  // o^I tile: 128 rows of 256 bytes (16 x 16-byte pieces); rows past L are zero
  for (int i = tid; i < kTile * 16; i += kThreads) {
    const int r = i >> 4, p = i & 15;
    const int t = t0 + r;
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (t < L) w = __ldg(reinterpret_cast<const uint4*>(o_id + ((size_t)t * HV + h) * kD) + p);
    *reinterpret_cast<uint4*>(oit + r * kLd + 8 * p) = w;
  }
  __syncthreads();

  const int g = lane >> 2, c = lane & 3;
  const int r0 = 16 * warp;  // this warp's rows in the tile
  float acc[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < kD / 16; ++ks) {
    const int k0 = 16 * ks + 2 * c;
    uint32_t a[4];
    a[0] = lds32(oit + (r0 + g) * kLd + k0);
    a[1] = lds32(oit + (r0 + g + 8) * kLd + k0);
    a[2] = lds32(oit + (r0 + g) * kLd + k0 + 8);
    a[3] = lds32(oit + (r0 + g + 8) * kLd + k0 + 8);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int vrow = (8 * nt + g) * kLd + k0;  // B[k = j][n = v] = S[v][j]
      mma_bf16_16816(acc[nt], a, lds32(shi + vrow), lds32(shi + vrow + 8));
      mma_bf16_16816(acc[nt], a, lds32(slo + vrow), lds32(slo + vrow + 8));
    }
  }
  // + o^0, bf16 out (two adjacent v per store)
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int t = t0 + r0 + g + 8 * half;
    if (t >= L) continue;
    const size_t row = ((size_t)t * HV + h) * kD;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int v = 8 * nt + 2 * c;
      const __nv_bfloat162 z = *reinterpret_cast<const __nv_bfloat162*>(o_zero + row + v);
      const float2 zf = __bfloat1622float2(z);
      *reinterpret_cast<__nv_bfloat162*>(out + row + v) =
          __floats2bfloat162_rn(acc[nt][2 * half] + zf.x, acc[nt][2 * half + 1] + zf.y);
    }
  }
}

bool misaligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; }

}  // namespace

extern "C" int gdn_segment_outputs_launch(const void* o_identity, const void* o_zero,
                                          const float* start_state, void* output,
                                          int num_tokens, int num_v_heads, int head_size,
                                          void* stream) {
  if (num_tokens < 0 || num_v_heads <= 0 || num_v_heads > 65535) return GDN_ERR_INVALID_ARGUMENT;
  if (head_size != kD) return GDN_ERR_UNSUPPORTED;
  if (num_tokens == 0) return GDN_OK;
  if (o_identity == nullptr || o_zero == nullptr || start_state == nullptr || output == nullptr)
    return GDN_ERR_INVALID_ARGUMENT;
  if (misaligned(o_identity, 16) || misaligned(start_state, 16) || misaligned(o_zero, 4) ||
      misaligned(output, 4))
    return GDN_ERR_INVALID_ARGUMENT;
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_LAUNCH;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(segment_outputs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmem) != cudaSuccess)
      return GDN_ERR_LAUNCH;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const dim3 grid((unsigned)((num_tokens + kTile - 1) / kTile), (unsigned)num_v_heads);
  segment_outputs_kernel<<<grid, kThreads, kSmem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(o_identity), static_cast<const __nv_bfloat16*>(o_zero),
      start_state, static_cast<__nv_bfloat16*>(output), num_tokens, num_v_heads);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
