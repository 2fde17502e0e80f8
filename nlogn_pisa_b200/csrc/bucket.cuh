// Device-side bucketing and staging helpers shared by the tile kernels:
// the one-CTA exclusive scan that turns bucket sizes into tile offsets,
// cp.async / zero-fill staging into 128B-swizzled shared memory, and the
// TMEM column visitor used by the epilogues.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace pisa {
namespace {

constexpr int kScanThreads = 1024;

// Exclusive scan of ceil(count / RT) over all buckets in one CTA: each warp
// owns a contiguous segment (coalesced 32-wide chunks), warp totals are
// scanned in shared memory, then offsets are written in a second pass.
__global__ void __launch_bounds__(kScanThreads)
tile_scan_kernel(const int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                 int32_t* __restrict__ total_tiles, int64_t nb, int RT) {
  __shared__ int64_t warp_base[kScanThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = kScanThreads / 32;
  const int64_t seg = (nb + warps - 1) / warps;
  const int64_t s0 = min64(int64_t(warp) * seg, nb), s1 = min64(s0 + seg, nb);
  int64_t sum = 0;
  for (int64_t i = s0 + lane; i < s1; i += 32) sum += (counts[i] + RT - 1) / RT;
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
  if (lane == 0) warp_base[warp] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int w = 0; w < warps; ++w) { const int64_t v = warp_base[w]; warp_base[w] = acc; acc += v; }
    *total_tiles = int32_t(acc);
  }
  __syncthreads();
  int64_t carry = warp_base[warp];
  for (int64_t base = s0; base < s1; base += 32) {
    const int64_t i = base + lane;
    const int v = i < s1 ? (counts[i] + RT - 1) / RT : 0;
    int incl = v;
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += n;
    }
    if (i < s1) offsets[i] = int32_t(carry + incl - v);
    carry += __shfl_sync(kFull, incl, 31);
  }
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
