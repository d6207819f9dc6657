// Segment-level scan of one long sequence split into token segments, one per GPU: the
// state-map chain and the output assembly.  Over a segment the outputs are affine in the
// segment's start state S (k-last [v][j] per v-head): o_t = S o^I_t + o^0_t, where o^I is
// the output of the segment run from the identity state with v = 0 and o^0 its output
// from a zero state.  Once the start state is known (after the exchange of the segments'
// state maps, chained below), the output kernel forms
//     out[t][h][v] = bf16( sum_j S[h][v][j] o^I[t][h][j] + o^0[t][h][v] )
// in one pass over o^I and o^0.
//
// Output kernel: one CTA of 4 warps per (v-head, group of 128-token tiles), one CTA per SM.
// S[h], split into bf16 hi + lo (S = hi + lo to 2^-15 relative), is written once to shared
// memory in the 128-byte-swizzled K-major layout; the o^I and o^0 tiles arrive by TMA in
// the same layout, two tiles in flight; per tile one thread issues the 16 tcgen05 MMAs
// (M = 128 tokens, N = 128 v, K = 128 j; hi then lo) into an fp32 TMEM accumulator, and the
// epilogue reads its TMEM lane, adds o^0 and rounds once to bf16.  It moves
// 3 x T x HV x 128 x 2 bytes (o^I and o^0 in, out) and is HBM-bound.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "gdn_b200.h"
#include "gdn_chunk_math.cuh"
#include "gdn_prefill.cuh"
#include "sm100.cuh"

namespace {

using namespace gdn::sm100;

constexpr int kD = 128;
constexpr int kTile = 128;    // tokens per tile (the MMA's M)
constexpr int kThreads = 128;
// shared memory (1024-aligned): S hi | S lo images, then two buffers of [o^I | o^0] tile
// images (each 32 KB: two 64-column halves of 128 rows, 128-byte swizzle), then barriers
constexpr uint32_t kSH = 0, kSL = 32768, kBuf0 = 65536, kBufBytes = 65536, kOZ = 32768;
constexpr uint32_t kBarOff = kBuf0 + 2 * kBufBytes;
constexpr size_t kSmem = kBarOff + 64 + 1024;  // + slack to align the base to 1024 bytes
constexpr unsigned kErrTmaTimeout = 1u, kErrMmaTimeout = 2u;
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ unsigned g_segment_device_error;

// Row r (128 bf16 = two 64-element halves) of a K-major SW128 image: the 16-byte piece `ch`
// (8 elements) sits in half ch / 8, swizzled chunk ch % 8.
__device__ __forceinline__ uint32_t img_off(uint32_t r, uint32_t ch) {
  return (ch >> 3) * 16384u + sw128(r, ch & 7u);
}

// o^I and o^0 of the tile starting at row `row0` -> buffer at `buf` (four 64 x 64 boxes
// each; rows past the end of the tensors arrive as zeros), completion counted on `bar`.
__device__ __forceinline__ void load_tile(uint8_t* buf, const CUtensorMap* m_id,
                                          const CUtensorMap* m_zero, uint64_t* bar, int h,
                                          int row0) {
  mbar_arrive_expect_tx(bar, kBufBytes);
#pragma unroll
  for (int half = 0; half < 2; ++half)
#pragma unroll
    for (int rb = 0; rb < 2; ++rb) {
      const int x = h * kD + 64 * half, y = row0 + 64 * rb;
      const uint32_t off = 16384u * half + 8192u * rb;
      tma_load_2d(buf + off, m_id, bar, x, y);
      tma_load_2d(buf + kOZ + off, m_zero, bar, x, y);
    }
}

// Segments of one launch: segment s covers rows [off[s], off[s] + len[s]) of o^I, o^0 and
// the output, and starts from start[s].
constexpr int kMaxSegs = 64;
struct OutSegs {
  int n;
  int off[kMaxSegs];
  int len[kMaxSegs];
};

// One CTA per (segment, v-head, group of token tiles): S[h] is split once and stays in
// shared memory; the tiles of the group stream through two buffers (the next tile's TMA
// loads run while the current tile's MMAs and epilogue do).  A tile's rows past its
// segment's end may belong to the next segment: they are read (and discarded), never
// written, so o^0 may live in the output itself (each row is read by its own tile's copy
// before that tile writes it).
__global__ void __launch_bounds__(kThreads, 1)
    segment_outputs_kernel(const __grid_constant__ CUtensorMap m_id,
                           const __grid_constant__ CUtensorMap m_zero,
                           const float* __restrict__ start, __nv_bfloat16* out,
                           const __grid_constant__ OutSegs segs, int HV) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(smem);
  uint64_t* bar_in = reinterpret_cast<uint64_t*>(smem + kBarOff);  // [2]
  uint64_t* bar_mma = bar_in + 2;
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + kBarOff + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kBarOff + 28);
  const int h = blockIdx.y, group = blockIdx.x, groups = gridDim.x, seg = blockIdx.z;
  const int L = segs.len[seg], y0 = segs.off[seg];
  const int ntiles = (L + kTile - 1) / kTile;
  const int mine = ntiles > group ? (ntiles - group + groups - 1) / groups : 0;  // tiles g, g+G, ..
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (mine == 0) return;
  if (warp == 0) {
    tmem_alloc(slot, 128);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(&bar_in[0], 1);
    mbar_init(&bar_in[1], 1);
    mbar_init(bar_mma, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  int issued = 0;  // tiles whose loads were issued (thread 0)
  if (tid == 0) {
    tma_prefetch_desc(&m_id);
    tma_prefetch_desc(&m_zero);
    for (; issued < 2 && issued < mine; ++issued)
      load_tile(smem + kBuf0 + issued * kBufBytes, &m_id, &m_zero, &bar_in[issued], h,
                y0 + (group + issued * groups) * kTile);
  }
  // S[h] rows v -> hi | lo images (8 fp32 per piece)
  const float* sh = start + ((size_t)seg * HV + h) * kD * kD;
#pragma unroll 4
  for (int k = 0; k < 16; ++k) {
    const int i = tid + k * kThreads, v = i >> 4, p = i & 15;
    const float4 x = __ldg(reinterpret_cast<const float4*>(sh + v * kD + 8 * p));
    const float4 y = __ldg(reinterpret_cast<const float4*>(sh + v * kD + 8 * p + 4));
    const float f[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
    uint4 hi, lo;
    gdn::cm::split8(f, hi, lo);
    st_shared_v4(sb + kSH + img_off(v, p), hi.x, hi.y, hi.z, hi.w);
    st_shared_v4(sb + kSL + img_off(v, p), lo.x, lo.y, lo.z, lo.w);
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const uint32_t idesc = umma_idesc_bf16(128, 128, false, false);
  const int r = 32 * warp + lane;  // this thread's token row in a tile (its TMEM lane)
  bool ok = true, mma_pending = false;
  uint32_t mma_par = 0;  // phase of bar_mma that the pending MMA group completes
  for (int i = 0; i < mine && ok; ++i) {
    const int b = i & 1;
    const uint32_t par = (i >> 1) & 1;
    const uint32_t buf = sb + kBuf0 + b * kBufBytes;
    if (!mbar_wait(&bar_in[b], par, kWaitLimit)) {
      atomicOr(&g_segment_device_error, kErrTmaTimeout);
      ok = false;
    }
    if (!__syncthreads_and(ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (tid == 0) {  // D[t][v] = sum_j oI[t][j] (S_hi[v][j] + S_lo[v][j])
#pragma unroll
      for (int term = 0; term < 2; ++term)
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = 16384u * (ks >> 2) + 32u * (ks & 3);
          umma_bf16(tmem, umma_desc_k(buf + off), umma_desc_k(sb + (term ? kSL : kSH) + off),
                    idesc, (term | ks) != 0);
        }
      umma_commit(bar_mma);
    }
    mma_pending = true;
    mma_par = i & 1;
    if (!mbar_wait(bar_mma, mma_par, kWaitLimit)) {
      if (lane == 0) atomicOr(&g_segment_device_error, kErrMmaTimeout);
      ok = false;
    }
    if (!__syncthreads_and(ok)) {
      ok = false;
      break;
    }
    mma_pending = false;
    tc_fence_after();
    const int t = (group + i * groups) * kTile + r;
    const uint32_t tl = tmem + ((uint32_t)(32 * warp) << 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float d[32];
      tmem_ld32(tl + 32u * q, d);
      tmem_wait_ld();
      if (t < L) {
        uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)(y0 + t) * HV + h) * kD + 32 * q);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const uint4 zv = ld_shared_v4(buf + kOZ + img_off(r, 4 * q + p));
          const uint32_t zw[4] = {zv.x, zv.y, zv.z, zv.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 zf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zw[e]));
            const __nv_bfloat162 rr =
                __floats2bfloat162_rn(d[8 * p + 2 * e] + zf.x, d[8 * p + 2 * e + 1] + zf.y);
            o[e] = *reinterpret_cast<const uint32_t*>(&rr);
          }
          dst[p] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // buffer b and the accumulator are free
    if (tid == 0 && issued < mine) {
      load_tile(smem + kBuf0 + b * kBufBytes, &m_id, &m_zero, &bar_in[b], h,
                y0 + (group + issued * groups) * kTile);
      ++issued;
    }
  }
  if (!ok && tid == 0) {  // copies and MMAs still in flight land before the CTA exits
    if (mma_pending) mbar_wait(bar_mma, mma_par, kWaitLimit);
    for (int j = max(issued - 2, 0); j < issued; ++j) mbar_wait(&bar_in[j & 1], (j >> 1) & 1, kWaitLimit);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// Start state and final state of segment `rank` from every segment's state map
// (A_m, B_m), each [HV][128][128] fp32, A_m at maps[(a0 + m as) HV + h], B_m at
// maps[(b0 + m bs) HV + h] (matrices):
//   S = B_0;  S <- S A_m + B_m for m = 1 .. rank-1;  start = S;  final = S A_rank + B_rank.
// Rows of S evolve independently (row i of S A depends on row i of S only), so each CTA
// carries 8 RPT rows of one v-head through the whole chain with no exchange between CTAs.
// 256 threads, each RPT rows x 4 columns (4 RPT FMAs per 4 A values read; two warps per
// scheduler hide the shared-memory latency), fp32 FMAs in the same order for every RPT
// and thread layout (the results do not depend on them).  A_m is staged in shared
// memory, the next map's A copied in (one bulk copy) while a step computes.  RPT = 4 (32 rows,
// 4 CTAs per v-head) when there are enough v-heads to fill the SMs, 2 or 1 otherwise.
struct MapIndex {
  int a0, as, b0, bs;
};
constexpr int kChainThreads = 256;
constexpr int kSLd = kD + 4;  // padded S rows
constexpr size_t chain_smem(int rpt) { return (size_t)(2 * kD * kD + 8 * rpt * kSLd) * sizeof(float); }


template <int RPT>
__global__ void __launch_bounds__(kChainThreads, 1)
    segment_chain_kernel(const float* __restrict__ maps, const MapIndex mi, int rank, int HV,
                         float* __restrict__ start_out, float* __restrict__ final_out,
                         float* __restrict__ starts_all) {
  constexpr int kRows = 8 * RPT;
  extern __shared__ __align__(16) float csm[];
  float* S = csm + 2 * kD * kD;  // [row][kSLd]
  const int h = blockIdx.y, r0 = kRows * blockIdx.x;
  // warp rq owns rows RPT rq .. RPT rq + RPT - 1 of the CTA's rows, lane cb columns 4 cb ..
  // 4 cb + 3: a warp reads one 512-byte row of A per step (no bank conflicts) and one
  // broadcast element of S per row
  const int tid = threadIdx.x, rq = tid >> 5, cb = tid & 31;
  const int c0 = 4 * cb;
  const size_t mat = (size_t)kD * kD;
  auto A = [&](int m) { return maps + ((size_t)(mi.a0 + m * mi.as) * HV + h) * mat; };
  auto B = [&](int m) { return maps + ((size_t)(mi.b0 + m * mi.bs) * HV + h) * mat; };
  // A_m (64 KiB, contiguous) arrives in one bulk copy into buffer (m - 1) & 1, counted on
  // that buffer's mbarrier; buffer b completes its phase p at step m = 2 p + b + 1
  __shared__ __align__(8) uint64_t abar[2];
  if (tid == 0) {
    mbar_init(&abar[0], 1);
    mbar_init(&abar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto prefetch = [&](int m) {
    if (tid == 0) {
      fence_proxy_async();  // earlier reads of the buffer before the copy's writes
      uint64_t* bar = &abar[(m - 1) & 1];
      mbar_arrive_expect_tx(bar, (uint32_t)(mat * sizeof(float)));
      bulk_load(csm + ((m - 1) & 1) * kD * kD, A(m), (uint32_t)(mat * sizeof(float)), bar);
    }
  };
  int issued = 1;  // maps whose copies were issued (A_1 .. A_issued)
  prefetch(1);
  // S = B_0 (this CTA's rows): the start state of segment 1
  for (int i = tid; i < kRows * kD / 4; i += kChainThreads) {
    const int r = i >> 5, c4 = i & 31;
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(B(0) + (size_t)(r0 + r) * kD) + c4);
    *reinterpret_cast<float4*>(S + r * kSLd + 4 * c4) = b0;
    if (starts_all != nullptr)
      reinterpret_cast<float4*>(starts_all + ((size_t)h * kD + r0 + r) * kD)[c4] = b0;
  }
  for (int m = 1; m <= rank; ++m) {
    const float* As = csm + ((m - 1) & 1) * kD * kD;
    const bool landed = mbar_wait(&abar[(m - 1) & 1], ((m - 1) >> 1) & 1, kWaitLimit);
    if (__syncthreads_or(!landed)) {  // A_m and S in place; the other A buffer is free
      if (tid == 0) {  // let the copies in flight land before the CTA exits (bounded)
        atomicOr(&g_segment_device_error, kErrTmaTimeout);
        for (int q = max(m, issued - 1); q <= issued; ++q)
          mbar_wait(&abar[(q - 1) & 1], ((q - 1) >> 1) & 1, kWaitLimit);
      }
      return;
    }
    if (m < rank) {
      prefetch(m + 1);
      issued = m + 1;
    }
    // B_m rows: loaded now, added after the product (their latency hides behind it)
    float4 bq[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i)
      bq[i] = __ldg(reinterpret_cast<const float4*>(B(m) + (size_t)(r0 + RPT * rq + i) * kD + c0));
    float acc[RPT][4];
#pragma unroll
    for (int i = 0; i < RPT; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
    const float* srow = S + (RPT * rq) * kSLd;
    // software-pipelined: the shared-memory operands of step j + 1 are loaded while the
    // FMAs of step j issue
    float4 x = *reinterpret_cast<const float4*>(As + c0);
    float sv[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) sv[i] = srow[i * kSLd];
#pragma unroll 4
    for (int j = 0; j < kD; ++j) {
      const int jn = (j + 1) & (kD - 1);  // the last prefetch wraps to row 0 and is unused
      const float4 xn = *reinterpret_cast<const float4*>(As + jn * kD + c0);
      float svn[RPT];
#pragma unroll
      for (int i = 0; i < RPT; ++i) svn[i] = srow[i * kSLd + jn];
      const float av[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int i = 0; i < RPT; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][e] = fmaf(sv[i], av[e], acc[i][e]);
      x = xn;
#pragma unroll
      for (int i = 0; i < RPT; ++i) sv[i] = svn[i];
    }
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      acc[i][0] += bq[i].x; acc[i][1] += bq[i].y; acc[i][2] += bq[i].z; acc[i][3] += bq[i].w;
    }
    if (m == rank) {  // the segment's own map: its final state; S holds its start state
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        float* dst = final_out + ((size_t)h * kD + r0 + RPT * rq + i) * kD;
        *reinterpret_cast<float4*>(dst + c0) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      }
      break;
    }
    __syncthreads();  // every read of S done
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      float* d = S + (RPT * rq + i) * kSLd;
      *reinterpret_cast<float4*>(d + c0) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    }
    if (starts_all != nullptr) {  // S is now the start state of segment m + 1
      float* base = starts_all + (size_t)m * HV * kD * kD;
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        float* dst = base + ((size_t)h * kD + r0 + RPT * rq + i) * kD;
        *reinterpret_cast<float4*>(dst + c0) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      }
    }
  }
  // start state = S (rows of this CTA)
  for (int i = tid; i < kRows * kD / 4; i += kChainThreads) {
    const int r = i >> 5, c4 = i & 31;
    reinterpret_cast<float4*>(start_out + ((size_t)h * kD + r0 + r) * kD)[c4] =
        *reinterpret_cast<const float4*>(S + r * kSLd + 4 * c4);
  }
}

bool misaligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; }

struct DeviceInfo {
  bool ok = false;
  int sms = 0;
};

// Shared-memory opt-in of the segment kernels and the SM count, once per device.
const DeviceInfo* device_info() {
  static DeviceInfo info[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  DeviceInfo& d = info[dev];
  if (!d.ok) {
    if (cudaFuncSetAttribute(segment_outputs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmem) != cudaSuccess ||
        cudaFuncSetAttribute(segment_chain_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)chain_smem(1)) != cudaSuccess ||
        cudaFuncSetAttribute(segment_chain_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)chain_smem(2)) != cudaSuccess ||
        cudaFuncSetAttribute(segment_chain_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)chain_smem(4)) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return nullptr;
    d.ok = true;
  }
  return &d;
}

}  // namespace

namespace gdn {
unsigned read_segment_device_error(bool clear) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_segment_device_error, sizeof(v)) != cudaSuccess) return ~0u;
  if (clear) {
    const unsigned zero = 0;
    cudaMemcpyToSymbol(g_segment_device_error, &zero, sizeof(zero));
  }
  return v;
}

// The chain over maps A_m = maps[a0 + m as], B_m = maps[b0 + m bs] (matrices of HV heads):
// segment `rank`'s start state into start_out and final state into final_out, and, when
// starts_all is given, segment s's start state into starts_all[s - 1] for s = 1 .. rank.
// Rows per CTA: as few as keep every CTA resident (more CTAs shorten each step).
cudaError_t launch_segment_chain(const float* maps, int a0, int as, int b0, int bs, int rank,
                                 int HV, float* start_out, float* final_out, float* starts_all,
                                 cudaStream_t s) {
  const DeviceInfo* d = device_info();
  if (d == nullptr) return cudaErrorInvalidValue;
  const MapIndex mi{a0, as, b0, bs};
  const int rpt = 16 * HV <= d->sms ? 1 : (8 * HV <= d->sms ? 2 : 4);
  const dim3 grid((unsigned)(kD / (8 * rpt)), (unsigned)HV);
  if (rpt == 1)
    segment_chain_kernel<1><<<grid, kChainThreads, chain_smem(1), s>>>(maps, mi, rank, HV, start_out,
                                                                     final_out, starts_all);
  else if (rpt == 2)
    segment_chain_kernel<2><<<grid, kChainThreads, chain_smem(2), s>>>(maps, mi, rank, HV, start_out,
                                                                     final_out, starts_all);
  else
    segment_chain_kernel<4><<<grid, kChainThreads, chain_smem(4), s>>>(maps, mi, rank, HV, start_out,
                                                                     final_out, starts_all);
  return cudaGetLastError();
}

// Outputs of nseg segments in one launch: segment s covers rows [off[s], off[s] + len[s])
// of o^I (rows_id rows at o_identity), o^0 (rows_zero rows at o_zero) and the output, and
// starts from start_states[s].  o_zero may be the output itself.
cudaError_t launch_segment_outputs(const void* o_identity, long long rows_id, const void* o_zero,
                                   long long rows_zero, const float* start_states, void* output,
                                   int nseg, const int* off, const int* len, int HV,
                                   cudaStream_t s) {
  const DeviceInfo* d = device_info();
  if (d == nullptr || nseg <= 0 || nseg > kMaxSegs) return cudaErrorInvalidValue;
  OutSegs segs{};
  segs.n = nseg;
  int max_tiles = 0;
  for (int i = 0; i < nseg; ++i) {
    segs.off[i] = off[i];
    segs.len[i] = len[i];
    max_tiles = std::max(max_tiles, (len[i] + kTile - 1) / kTile);
  }
  if (max_tiles == 0) return cudaSuccess;
  CUtensorMap m_id, m_zero;
  const long long row = (long long)HV * kD;
  if (!make_tile_map(&m_id, o_identity, HV, rows_id, row) ||
      !make_tile_map(&m_zero, o_zero, HV, rows_zero, row))
    return cudaErrorInvalidValue;
  // about one CTA per SM: the SMs split over the (segment, v-head) pairs, each CTA a group
  // of token tiles
  const int groups = std::max(1, std::min(max_tiles, d->sms / (HV * nseg)));
  const dim3 grid((unsigned)groups, (unsigned)HV, (unsigned)nseg);
  segment_outputs_kernel<<<grid, kThreads, kSmem, s>>>(m_id, m_zero, start_states,
                                                       static_cast<__nv_bfloat16*>(output), segs, HV);
  return cudaGetLastError();
}
}  // namespace gdn

extern "C" int gdn_segment_outputs_launch(const void* o_identity, const void* o_zero,
                                          const float* start_state, void* output,
                                          int num_tokens, int num_v_heads, int head_size,
                                          void* stream) {
  if (num_tokens < 0 || num_v_heads <= 0 || num_v_heads > 65535) return GDN_ERR_INVALID_ARGUMENT;
  if (head_size != kD) return GDN_ERR_UNSUPPORTED;
  if (num_tokens == 0) return GDN_OK;
  if (o_identity == nullptr || o_zero == nullptr || start_state == nullptr || output == nullptr)
    return GDN_ERR_INVALID_ARGUMENT;
  if (misaligned(o_identity, 16) || misaligned(start_state, 16) || misaligned(o_zero, 16) ||
      misaligned(output, 16))
    return GDN_ERR_INVALID_ARGUMENT;
  const int off = 0;
  const cudaError_t e = gdn::launch_segment_outputs(o_identity, num_tokens, o_zero, num_tokens,
                                                    start_state, output, 1, &off, &num_tokens,
                                                    num_v_heads, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidValue) return GDN_ERR_UNSUPPORTED;
  return e == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
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
  // maps [num_maps][2][HV][128][128]: A_m = entry 2 m, B_m = entry 2 m + 1
  const cudaError_t e = gdn::launch_segment_chain(maps, 0, 2, 1, 2, rank, num_v_heads, start_state,
                                                  final_state, nullptr,
                                                  static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

extern "C" int gdn_segment_chain_all_launch(const float* maps, int num_maps, float* start_states,
                                            float* final_state, int num_v_heads, int head_size,
                                            void* stream) {
  if (num_v_heads <= 0 || num_v_heads > 65535 || num_maps < 2) return GDN_ERR_INVALID_ARGUMENT;
  if (head_size != kD) return GDN_ERR_UNSUPPORTED;
  if (maps == nullptr || start_states == nullptr || final_state == nullptr)
    return GDN_ERR_INVALID_ARGUMENT;
  if (misaligned(maps, 16) || misaligned(start_states, 16) || misaligned(final_state, 16))
    return GDN_ERR_INVALID_ARGUMENT;
  // one pass through every map: segment s's start state into start_states[s - 1] as the
  // chain reaches it, the last segment's final state into final_state
  const int rank = num_maps - 1;
  float* last_start = start_states + (size_t)(rank - 1) * num_v_heads * kD * kD;
  const cudaError_t e = gdn::launch_segment_chain(maps, 0, 2, 1, 2, rank, num_v_heads, last_start,
                                                  final_state, start_states,
                                                  static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
