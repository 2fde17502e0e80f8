// Device-side bucketing and staging helpers shared by the tile kernels:
// the one-CTA exclusive scan that turns bucket sizes into tile offsets,
// cp.async / zero-fill staging into 128B-swizzled shared memory, and the
// TMEM column visitor used by the epilogues.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace pisa {

// Counts one launch of this library (defined in timing.cu).
void count_launch();

namespace {

constexpr int kScanThreads = 1024;

// Exclusive scan of ceil(count / RT) over the buckets [blk*seg, (blk+1)*seg)
// of this CTA (RT a power of two; tile counts fit 31 bits): each warp owns a
// contiguous part (coalesced 32-wide chunks), warp totals are scanned in
// shared memory, then offsets are written in a second pass with four buckets
// per lane and step.  A single CTA also writes the total; with several CTAs
// the tile offset of each CTA's first bucket comes from `block_base`.
__global__ void __launch_bounds__(kScanThreads)
tile_scan_kernel(const int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                 int32_t* __restrict__ total_tiles, int64_t nb, int RT,
                 const int32_t* __restrict__ block_base, int64_t seg) {
  __shared__ int warp_base[kScanThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = kScanThreads / 32;
  const int lg = 31 - __clz(RT);
  const int64_t b0 = int64_t(blockIdx.x) * seg, b1 = min64(b0 + seg, nb);
  const int64_t wseg = ((b1 - b0 + warps - 1) / warps + 127) / 128 * 128;
  const int64_t s0 = min64(b0 + int64_t(warp) * wseg, b1), s1 = min64(s0 + wseg, b1);
  int sum = 0;
#pragma unroll 4
  for (int64_t i = s0 + lane; i < s1; i += 32) sum += (counts[i] + RT - 1) >> lg;
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
  if (lane == 0) warp_base[warp] = sum;
  __syncthreads();
  if (warp == 0) {
    const int v = warp_base[lane];
    int incl = v;
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += n;
    }
    warp_base[lane] = incl - v + (block_base ? block_base[blockIdx.x] : 0);
    if (lane == 31 && !block_base) *total_tiles = incl;
  }
  __syncthreads();
  // second pass: each lane takes four consecutive buckets per 128-bucket step
  int carry = warp_base[warp];
  for (int64_t base = s0; base < s1; base += 128) {
    const int64_t i0 = base + 4 * lane;
    int v[4], run = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[u] = i0 + u < s1 ? (counts[i0 + u] + RT - 1) >> lg : 0;
      run += v[u];
    }
    int incl = run;
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += n;
    }
    int off = carry + incl - run;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (i0 + u < s1) offsets[i0 + u] = off;
      off += v[u];
    }
    carry += __shfl_sync(kFull, incl, 31);
  }
}

// Tile totals of each CTA's bucket range (first phase of the multi-CTA scan).
__global__ void __launch_bounds__(kScanThreads)
tile_total_kernel(const int32_t* __restrict__ counts, int32_t* __restrict__ partials, int64_t nb, int RT,
                  int64_t seg) {
  __shared__ int warp_sum[kScanThreads / 32];
  const int lg = 31 - __clz(RT);
  const int64_t b0 = int64_t(blockIdx.x) * seg, b1 = min64(b0 + seg, nb);
  int sum = 0;
  for (int64_t i = b0 + threadIdx.x; i < b1; i += kScanThreads) sum += (counts[i] + RT - 1) >> lg;
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
  if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x < 32) {
    int v = warp_sum[threadIdx.x];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    if (threadIdx.x == 0) partials[blockIdx.x] = v;
  }
}

// Exclusive scan of at most 64 CTA totals in place, and the grand total.
__global__ void tile_bases_kernel(int32_t* __restrict__ partials, int n, int32_t* __restrict__ total_tiles) {
  const int lane = threadIdx.x;
  int v[2], run = 0;
#pragma unroll
  for (int u = 0; u < 2; ++u) { v[u] = 2 * lane + u < n ? partials[2 * lane + u] : 0; run += v[u]; }
  int incl = run;
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += x;
  }
  int off = incl - run;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    if (2 * lane + u < n) partials[2 * lane + u] = off;
    off += v[u];
  }
  if (lane == 31) *total_tiles = incl;
}


// Bucket sizes -> tile offsets and the tile total.  Up to 64K buckets one CTA
// does it; above, up to 60 CTAs (their totals kept in the 240 bytes after
// `total_tiles`, which sits at the start of a 256-byte workspace slot).
inline cudaError_t launch_tile_scan(const int32_t* counts, int32_t* offsets, int32_t* total_tiles, int64_t nb,
                                    int RT, cudaStream_t stream) {
  if (nb <= 65536) {
    tile_scan_kernel<<<1, kScanThreads, 0, stream>>>(counts, offsets, total_tiles, nb, RT, nullptr, nb);
    count_launch();
    return cudaGetLastError();
  }
  const int64_t seg = ((nb + 59) / 60 + 4095) / 4096 * 4096;
  const int nblk = int((nb + seg - 1) / seg);
  int32_t* partials = total_tiles + 4;
  tile_total_kernel<<<nblk, kScanThreads, 0, stream>>>(counts, partials, nb, RT, seg);
  tile_bases_kernel<<<1, 32, 0, stream>>>(partials, nblk, total_tiles);
  tile_scan_kernel<<<nblk, kScanThreads, 0, stream>>>(counts, offsets, total_tiles, nb, RT, partials, seg);
  count_launch();
  count_launch();
  count_launch();
  return cudaGetLastError();
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(dst), "l"(src) : "memory");
}
// 16 zero bytes at dst through the same asynchronous path (source size 0)
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* any_global) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, 0;" :: "r"(dst), "l"(any_global) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ void st_zero16(uint32_t dst) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" :: "r"(dst), "r"(0) : "memory");
}

// Visit the `n` accumulator columns of this thread's TMEM lane starting at
// `taddr` (n a multiple of 16): fn(column, value).  Warp-collective.
template <typename F>
__device__ __forceinline__ void for_columns(uint32_t taddr, int n, F&& fn) {
  int c = 0;
  for (; c + 32 <= n; c += 32) {
    float v[32];
    tc::tmem_ld32(taddr + c, v);
#pragma unroll
    for (int i = 0; i < 32; ++i) fn(c + i, v[i]);
  }
  if (c < n) {
    float v[16];
    tc::tmem_ld16(taddr + c, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) fn(c + i, v[i]);
  }
}

}  // namespace
}  // namespace pisa
