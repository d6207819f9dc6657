// Shared device helpers of the chunked prefill kernels: bf16 hi/lo splits done
// with integer operations, TMEM column loads, and the 64 x 64 unit lower
// triangular inverse (CUDA cores + warp-level 3xTF32 tensor-core merges).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "sm100.cuh"

namespace gdn {
namespace cm {
using namespace sm100;

constexpr int kLd = 68;                // row stride (floats) of the in-place A / T matrix
constexpr int kLdE3 = 20, kLdE4 = 36;  // scratch strides of the merges (2-way conflicts at most)

// bf16 conversions with integer operations (ALU pipe) rather than cvt (which
// shares the XU pipe with exp/rsqrt and was the kernel's busiest pipe).
// Round-to-nearest-even of a finite fp32 bit pattern to bf16, kept in the high half.
__device__ __forceinline__ uint32_t rn_bf16_bits(uint32_t xb) {
  return (xb + 0x7FFFu + ((xb >> 16) & 1u)) & 0xFFFF0000u;
}
// Two bf16 values held in the high halves of a and b -> one packed word (a low, b high).
__device__ __forceinline__ uint32_t pack_hi16(uint32_t a, uint32_t b) {
  return __byte_perm(a, b, 0x7632);
}
// 8 floats -> (hi, lo) bf16 chunks with x ~= hi + lo: hi is x truncated to bf16
// (exact residual x - hi, |x - hi| < 2^-7 |x|) and lo that residual truncated, so
// hi + lo keeps ~15 significant bits (relative error < 2^-15) for three ALU
// operations per element (mask, subtract, byte-permute).
__device__ __forceinline__ void split8(const float* x, uint4& hi, uint4& lo) {
  uint32_t xb[8], lb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    xb[i] = __float_as_uint(x[i]);
    lb[i] = __float_as_uint(x[i] - __uint_as_float(xb[i] & 0xFFFF0000u));
  }
  hi = make_uint4(pack_hi16(xb[0], xb[1]), pack_hi16(xb[2], xb[3]), pack_hi16(xb[4], xb[5]),
                  pack_hi16(xb[6], xb[7]));
  lo = make_uint4(pack_hi16(lb[0], lb[1]), pack_hi16(lb[2], lb[3]), pack_hi16(lb[4], lb[5]),
                  pack_hi16(lb[6], lb[7]));
}
// Round-to-nearest bf16 pair (one cvt per two elements), low element first.
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo_elem, float hi_elem) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo_elem, hi_elem);
  return *reinterpret_cast<uint32_t*>(&v);
}
// 16 consecutive fp32 TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 8 consecutive fp32 TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// 8 consecutive 32-bit TMEM columns of this thread's lane <- registers (warp-collective).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(
                   taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
               : "memory");
}
__device__ __forceinline__ void st_v4(uint32_t addr, uint4 v) {
  st_shared_v4(addr, v.x, v.y, v.z, v.w);
}

// ---- warp-level tensor-core products for the inverse's block merges ----
// D(16x8) = X(16xK) * Y(Kx8), fp32 operands as 3xTF32 (hi.hi + hi.lo + lo.hi;
// hi = the top 10 mantissa bits, lo = the exact residual), so the result carries
// ~21 significant bits.  The three terms accumulate separately (three independent
// mma.sync chains instead of one, which matters where tcgen05 MMAs of the same CTA
// keep the tensor pipe busy) and are summed at the end.  Fragment layout of mma.m16n8k8 (tf32): g = lane/4,
// t = lane%4; A: (g, t) (g+8, t) (g, t+4) (g+8, t+4); B: (t, g) (t+4, g);
// C: (g, 2t) (g, 2t+1) (g+8, 2t) (g+8, 2t+1).

__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4],
                                         const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ void mma_tile_tf32x3(const float* X, int ldx, const float* Y, int ldy,
                                                int K, float (&c)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float c1[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
  c[0] = c[1] = c[2] = c[3] = 0.f;
  for (int k0 = 0; k0 < K; k0 += 8) {
    const float af[4] = {X[g * ldx + k0 + t], X[(g + 8) * ldx + k0 + t],
                         X[g * ldx + k0 + t + 4], X[(g + 8) * ldx + k0 + t + 4]};
    const float bf[2] = {Y[(k0 + t) * ldy + g], Y[(k0 + t + 4) * ldy + g]};
    uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      ah[i] = __float_as_uint(af[i]) & 0xFFFFE000u;
      al[i] = __float_as_uint(af[i] - __uint_as_float(ah[i]));
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      bh[i] = __float_as_uint(bf[i]) & 0xFFFFE000u;
      bl[i] = __float_as_uint(bf[i] - __uint_as_float(bh[i]));
    }
    mma_tf32(c1, al, bh);
    mma_tf32(c2, ah, bl);
    mma_tf32(c, ah, bh);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] += c1[i] + c2[i];
}
__device__ __forceinline__ void store_tile(float* D, int ldd, const float (&c)[4], float sgn) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  D[g * ldd + 2 * t] = sgn * c[0];
  D[g * ldd + 2 * t + 1] = sgn * c[1];
  D[(g + 8) * ldd + 2 * t] = sgn * c[2];
  D[(g + 8) * ldd + 2 * t + 1] = sgn * c[3];
}

// In-place T = (I + A)^-1 for the strictly lower triangular A in M[64][kLd], by
// 256 threads (local index u, named barrier kBar among them): 8x8 diagonal blocks by
// forward substitution, then 8->16 (CUDA cores), 16->32 and 32->64 (warp-level
// tensor cores, 3xTF32) block merges T21 = -T22 (A21 T11), each A21 block
// overwritten by T21 once it has been read.
template <uint32_t kBar>
__device__ __forceinline__ void invert_in_place(float* __restrict__ M, float* __restrict__ Es,
                                                int u) {
  if (u < 64) {
    const int o = 8 * (u >> 3), col = u & 7;
    float a[8][8];
#pragma unroll
    for (int r = 1; r < 8; ++r)
#pragma unroll
      for (int j = 0; j < r; ++j) a[r][j] = M[(o + r) * kLd + o + j];
    __syncwarp();  // the block's 8 threads share this warp: all reads before any write
    float x[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < r; ++j) acc = fmaf(a[r][j], x[j], acc);
      x[r] = (r < col) ? 0.f : ((r == col) ? 1.f : -acc);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) M[(o + r) * kLd + o + col] = x[r];
  }
  group_sync(kBar, 256);
  {  // 8 -> 16: pairs p = 0..3, rows bi = 16p + 8, cols bj = 16p
    const int p = u >> 6, r = (u >> 3) & 7, c = u & 7;
    const int bi = 16 * p + 8, bj = 16 * p;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc = fmaf(M[(bi + r) * kLd + bj + k], M[(bj + k) * kLd + bj + c], acc);
    Es[p * 64 + r * 8 + c] = acc;
    group_sync(kBar, 256);
    acc = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc = fmaf(M[(bi + r) * kLd + bi + k], Es[p * 64 + k * 8 + c], acc);
    M[(bi + r) * kLd + bj + c] = -acc;
  }
  group_sync(kBar, 256);
  const int wg = u >> 5;  // warp within the group
  {  // 16 -> 32 on the tensor cores: pairs p = 0..1 (rows bi = 32p+16, cols bj = 32p),
     // two 8-wide column tiles each -> warps 0..3
    if (wg < 4) {
      const int pr = wg >> 1, nt = wg & 1;
      const int bi = 32 * pr + 16, bj = 32 * pr;
      float c[4];
      mma_tile_tf32x3(M + bi * kLd + bj, kLd, M + bj * kLd + bj + 8 * nt, kLd, 16, c);
      store_tile(Es + pr * 16 * kLdE3 + 8 * nt, kLdE3, c, 1.f);
    }
    group_sync(kBar, 256);
    if (wg < 4) {
      const int pr = wg >> 1, nt = wg & 1;
      const int bi = 32 * pr + 16, bj = 32 * pr;
      float c[4];
      mma_tile_tf32x3(M + bi * kLd + bi, kLd, Es + pr * 16 * kLdE3 + 8 * nt, kLdE3, 16, c);
      store_tile(M + bi * kLd + bj + 8 * nt, kLd, c, -1.f);
    }
  }
  group_sync(kBar, 256);
  {  // 32 -> 64 on the tensor cores: rows 32..63 x cols 0..31 = 2 x 4 tiles of 16 x 8
    const int mt = wg >> 2, nt = wg & 3;
    float c[4];
    mma_tile_tf32x3(M + (32 + 16 * mt) * kLd, kLd, M + 8 * nt, kLd, 32, c);
    store_tile(Es + 16 * mt * kLdE4 + 8 * nt, kLdE4, c, 1.f);
    group_sync(kBar, 256);
    mma_tile_tf32x3(M + (32 + 16 * mt) * kLd + 32, kLd, Es + 8 * nt, kLdE4, 32, c);
    store_tile(M + (32 + 16 * mt) * kLd + 8 * nt, kLd, c, -1.f);
  }
  group_sync(kBar, 256);
}
}  // namespace cm
}  // namespace gdn
