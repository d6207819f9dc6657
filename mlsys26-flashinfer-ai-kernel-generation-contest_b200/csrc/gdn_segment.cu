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

// Four 8 x 8 bf16 matrices from shared memory; lane l gives the row address of matrix l / 8.
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const __nv_bfloat16* row) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
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

  // o^I tile: 128 rows of 256 bytes (16 x 16-byte pieces); rows past L are zero.  All of a
  // thread's loads are issued before the first store (the loads are independent).
  {
    constexpr int kPer = kTile * 16 / kThreads;
    uint4 w[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = tid + k * kThreads, r = i >> 4, p = i & 15, t = t0 + r;
      w[k] = t < L ? __ldg(reinterpret_cast<const uint4*>(o_id + ((size_t)t * HV + h) * kD) + p)
                   : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = tid + k * kThreads;
      *reinterpret_cast<uint4*>(oit + (i >> 4) * kLd + 8 * (i & 15)) = w[k];
    }
  }
  // S[h] -> hi | lo (fp32 rows of 128, four elements per load), in two batches of loads
  const float4* s4 = reinterpret_cast<const float4*>(start + (size_t)h * kD * kD);
#pragma unroll
  for (int b = 0; b < 2; ++b) {
    constexpr int kPer = kD * kD / 4 / kThreads / 2;
    float4 x[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) x[k] = __ldg(s4 + tid + (b * kPer + k) * kThreads);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = tid + (b * kPer + k) * kThreads;
      const int v = i >> 5, j = (i & 31) * 4;
      const __nv_bfloat162 h01 = __floats2bfloat162_rn(x[k].x, x[k].y);
      const __nv_bfloat162 h23 = __floats2bfloat162_rn(x[k].z, x[k].w);
      const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
      const __nv_bfloat162 l01 = __floats2bfloat162_rn(x[k].x - f01.x, x[k].y - f01.y);
      const __nv_bfloat162 l23 = __floats2bfloat162_rn(x[k].z - f23.x, x[k].w - f23.y);
      uint2 hv, lv;
      hv.x = *reinterpret_cast<const uint32_t*>(&h01);
      hv.y = *reinterpret_cast<const uint32_t*>(&h23);
      lv.x = *reinterpret_cast<const uint32_t*>(&l01);
      lv.y = *reinterpret_cast<const uint32_t*>(&l23);
      *reinterpret_cast<uint2*>(shi + v * kLd + j) = hv;
      *reinterpret_cast<uint2*>(slo + v * kLd + j) = lv;
    }
  }
  __syncthreads();

  const int g = lane >> 2, c = lane & 3;
  const int r0 = 16 * warp;  // this warp's rows in the tile
  float acc[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
  // ldmatrix row addresses: A matrices (rows 0-7 | 8-15) x (k 0-7 | 8-15) of the warp's
  // 16 rows; B matrices (n-tile nt: v 0-7, nt + 1: v 8-15) x (k 0-7 | 8-15), B[k][n] = S[v][j]
  const int lr = lane & 7, lm = lane >> 3;
  const __nv_bfloat16* a_row = oit + (r0 + lr + 8 * (lm & 1)) * kLd + 8 * (lm >> 1);
  const int b_off = (lr + 8 * (lm >> 1)) * kLd + 8 * (lm & 1);
#pragma unroll
  for (int ks = 0; ks < kD / 16; ++ks) {
    uint32_t a[4];
    ldmatrix_x4(a, a_row + 16 * ks);
#pragma unroll
    for (int np = 0; np < 8; ++np) {  // pairs of n-tiles
      uint32_t bh[4], bl[4];
      ldmatrix_x4(bh, shi + (16 * np) * kLd + b_off + 16 * ks);
      ldmatrix_x4(bl, slo + (16 * np) * kLd + b_off + 16 * ks);
      mma_bf16_16816(acc[2 * np], a, bh[0], bh[1]);
      mma_bf16_16816(acc[2 * np], a, bl[0], bl[1]);
      mma_bf16_16816(acc[2 * np + 1], a, bh[2], bh[3]);
      mma_bf16_16816(acc[2 * np + 1], a, bl[2], bl[3]);
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

// Start state and final state of segment `rank` from every segment's state map
// maps[m] = (A_m, B_m), each [HV][128][128] fp32:
//   S = B_0;  S <- S A_m + B_m for m = 1 .. rank-1;  start = S;  final = S A_rank + B_rank.
// Rows of S evolve independently (row i of S A depends on row i of S only), so each CTA
// carries 32 rows of one v-head through the whole chain with no exchange between CTAs.
// 128 threads, each 4 rows x 8 columns (32 FMAs per 8 A values read), fp32 FMAs.  A_m is
// staged in shared memory, the next map's A copied in (cp.async) while a step computes.
constexpr int kChainRows = 32;
constexpr int kChainThreads = 128;
constexpr int kSLd = kD + 4;  // padded S rows
constexpr int kAPer = kD * kD / 4 / kChainThreads;  // 16-byte pieces of A per thread
constexpr size_t kChainSmem = (size_t)(2 * kD * kD + kChainRows * kSLd) * sizeof(float);

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(kChainThreads, 1)
    segment_chain_kernel(const float* __restrict__ maps, int rank, int HV,
                         float* __restrict__ start_out, float* __restrict__ final_out) {
  extern __shared__ __align__(16) float csm[];
  float* S = csm + 2 * kD * kD;  // [row][kSLd]
  const int h = blockIdx.y, r0 = kChainRows * blockIdx.x;
  const int tid = threadIdx.x, rq = tid >> 4, cb = tid & 15;
  const size_t mat = (size_t)kD * kD;
  auto A = [&](int m) { return maps + ((size_t)(2 * m) * HV + h) * mat; };
  auto B = [&](int m) { return maps + ((size_t)(2 * m + 1) * HV + h) * mat; };
  auto prefetch = [&](int m, float* dst) {
    const float* src = A(m);
#pragma unroll 8
    for (int k = 0; k < kAPer; ++k) {
      const int i = tid + k * kChainThreads;
      cp_async16(dst + 4 * i, src + 4 * i);
    }
    cp_async_commit();
  };
  prefetch(1, csm);
  // S = B_0 (this CTA's rows)
  for (int i = tid; i < kChainRows * kD / 4; i += kChainThreads) {
    const int r = i >> 5, c4 = i & 31;
    *reinterpret_cast<float4*>(S + r * kSLd + 4 * c4) =
        __ldg(reinterpret_cast<const float4*>(B(0) + (size_t)(r0 + r) * kD) + c4);
  }
  for (int m = 1; m <= rank; ++m) {
    const float* As = csm + ((m - 1) & 1) * kD * kD;
    cp_async_wait_all();
    __syncthreads();  // A_m and S in place; the other A buffer is no longer read
    if (m < rank) prefetch(m + 1, csm + (m & 1) * kD * kD);
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4* b4 =
          reinterpret_cast<const float4*>(B(m) + (size_t)(r0 + 4 * rq + i) * kD + 8 * cb);
      const float4 x = __ldg(b4), y = __ldg(b4 + 1);
      acc[i][0] = x.x; acc[i][1] = x.y; acc[i][2] = x.z; acc[i][3] = x.w;
      acc[i][4] = y.x; acc[i][5] = y.y; acc[i][6] = y.z; acc[i][7] = y.w;
    }
    const float* srow = S + (4 * rq) * kSLd;
#pragma unroll 4
    for (int j = 0; j < kD; ++j) {
      const float4 x = *reinterpret_cast<const float4*>(As + j * kD + 8 * cb);
      const float4 y = *reinterpret_cast<const float4*>(As + j * kD + 8 * cb + 4);
      const float av[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float si = srow[i * kSLd + j];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i][e] = fmaf(si, av[e], acc[i][e]);
      }
    }
    if (m == rank) {  // the segment's own map: its final state; S holds its start state
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float* dst = final_out + ((size_t)h * kD + r0 + 4 * rq + i) * kD + 8 * cb;
        reinterpret_cast<float4*>(dst)[0] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
      }
      break;
    }
    __syncthreads();  // every read of S done
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float* d = S + (4 * rq + i) * kSLd + 8 * cb;
      reinterpret_cast<float4*>(d)[0] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      reinterpret_cast<float4*>(d)[1] = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
    }
  }
  // start state = S (rows of this CTA)
  for (int i = tid; i < kChainRows * kD / 4; i += kChainThreads) {
    const int r = i >> 5, c4 = i & 31;
    reinterpret_cast<float4*>(start_out + ((size_t)h * kD + r0 + r) * kD)[c4] =
        *reinterpret_cast<const float4*>(S + r * kSLd + 4 * c4);
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

extern "C" int gdn_segment_chain_launch(const float* maps, int num_maps, int rank,
                                        float* start_state, float* final_state,
                                        int num_v_heads, int head_size, void* stream) {
  if (num_v_heads <= 0 || num_v_heads > 65535 || rank < 1 || rank >= num_maps)
    return GDN_ERR_INVALID_ARGUMENT;
  if (head_size != kD) return GDN_ERR_UNSUPPORTED;
  if (maps == nullptr || start_state == nullptr || final_state == nullptr)
    return GDN_ERR_INVALID_ARGUMENT;
  if (misaligned(maps, 16) || misaligned(start_state, 16) || misaligned(final_state, 16))
    return GDN_ERR_INVALID_ARGUMENT;
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_LAUNCH;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(segment_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kChainSmem) != cudaSuccess)
      return GDN_ERR_LAUNCH;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const dim3 grid(kD / kChainRows, (unsigned)num_v_heads);
  segment_chain_kernel<<<grid, kChainThreads, kChainSmem, static_cast<cudaStream_t>(stream)>>>(
      maps, rank, num_v_heads, start_state, final_state);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
