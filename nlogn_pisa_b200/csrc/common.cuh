// Shared device helpers for the PISA sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pisa_b200.h"

namespace pisa {

constexpr unsigned kFull = 0xffffffffu;

// Division of 31-bit unsigned numerators by a divisor fixed for a launch,
// by multiply-high and shift (Granlund and Montgomery, "Division by
// invariant integers using multiplication", 1994): with s = ceil(log2 d) and
// m = floor(2^32 * (2^s - d) / d) + 1, n / d = (umulhi(n, m) + n) >> s for
// n < 2^31.  Keeps integer division off the MUFU pipe, which the softmax
// exponentials of the tile kernels keep busy.
struct FastDiv {
  uint32_t d = 1, m = 1, s = 0;
  __host__ static FastDiv make(uint32_t divisor) {
    FastDiv f;
    f.d = divisor < 1 ? 1 : divisor;
    f.s = 0;
    while ((uint64_t(1) << f.s) < f.d) ++f.s;
    f.m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << f.s) - f.d)) / f.d + 1);
    return f;
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const { return (__umulhi(n, m) + n) >> s; }
  __device__ __forceinline__ uint32_t mod(uint32_t n) const { return n - div(n) * d; }
};
constexpr float kNegFill = -1.0e9f;  // invalid candidates (top_k_pyramid_torch.py:170)
constexpr float kPosFill = 1.0e9f;   // forced candidates (top_k_pyramid_torch.py:171)
constexpr int kMaxLevels = 32;

// ---------------------------------------------------------------------------
// element conversion
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Number of elements in one 16-byte vector.
template <typename T> struct Vec { static constexpr int N = 16 / sizeof(T); };

// Load one 16-byte vector of T as floats (read-only path).
template <typename T>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&out)[Vec<T>::N]) {
  uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  if constexpr (sizeof(T) == 4) {
    out[0] = __uint_as_float(raw.x); out[1] = __uint_as_float(raw.y);
    out[2] = __uint_as_float(raw.z); out[3] = __uint_as_float(raw.w);
  } else {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < Vec<T>::N; ++i) out[i] = to_f32<T>(e[i]);
  }
}

// Same as load_vec but through L2 only (data written earlier in this kernel by other CTAs).
template <typename T>
__device__ __forceinline__ void load_vec_cg(const T* p, float (&out)[Vec<T>::N]) {
  uint4 raw = __ldcg(reinterpret_cast<const uint4*>(p));
  if constexpr (sizeof(T) == 4) {
    out[0] = __uint_as_float(raw.x); out[1] = __uint_as_float(raw.y);
    out[2] = __uint_as_float(raw.z); out[3] = __uint_as_float(raw.w);
  } else {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < Vec<T>::N; ++i) out[i] = to_f32<T>(e[i]);
  }
}

template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float (&v)[Vec<T>::N]) {
  uint4 raw;
  if constexpr (sizeof(T) == 4) {
    raw.x = __float_as_uint(v[0]); raw.y = __float_as_uint(v[1]);
    raw.z = __float_as_uint(v[2]); raw.w = __float_as_uint(v[3]);
  } else {
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < Vec<T>::N; ++i) e[i] = from_f32<T>(v[i]);
  }
  *reinterpret_cast<uint4*>(p) = raw;
}

// ---------------------------------------------------------------------------
// warp reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// The descending bitonic comparison network of top_k_pyramid_torch.py:84-110,
// with its exact compare/exchange tie order.  Element i of the WP-wide network
// lives in lane (i % 32), slot (i / 32).  For WP < 32 only lanes < WP matter;
// lanes >= WP exchange among themselves (xor distances stay below WP).
//   pass (size, d): element i and i^d; "left" = (i & d) == 0;
//   descending = (size == WP) || (i & size);
//   exchange   = (left_score > right_score) != descending.
// Equal scores therefore exchange in descending groups and stay put in
// ascending ones, exactly as the reference.
// ---------------------------------------------------------------------------
template <int WP>
struct Network {
  static constexpr int E = WP >= 32 ? WP / 32 : 1;

  __device__ __forceinline__ static void sort(float (&s)[E], int (&id)[E], int lane) {
#pragma unroll
    for (int size = 2; size <= WP; size <<= 1) {
#pragma unroll
      for (int d = size >> 1; d > 0; d >>= 1) {
        if (d < 32) {
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const int i = e * 32 + lane;
            const float ps = __shfl_xor_sync(kFull, s[e], d);
            const int pid = __shfl_xor_sync(kFull, id[e], d);
            const bool desc = (size == WP) || (i & size);
            const bool left = (i & d) == 0;
            const float ls = left ? s[e] : ps;
            const float rs = left ? ps : s[e];
            const bool ex = (ls > rs) != desc;
            if (ex) { s[e] = ps; id[e] = pid; }
          }
        } else {
          constexpr int dummy = 0; (void)dummy;
          const int de = d / 32;
#pragma unroll
          for (int e = 0; e < E; ++e) {
            if ((e & de) == 0) {
              const int f = e | de;  // partner slot (same lane)
              const int i = e * 32 + lane;
              const bool desc = (size == WP) || (i & size);
              const bool ex = (s[e] > s[f]) != desc;  // e is the left element
              if (ex) {
                float ts = s[e]; s[e] = s[f]; s[f] = ts;
                int ti = id[e]; id[e] = id[f]; id[f] = ti;
              }
            }
          }
        }
      }
    }
  }
};

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

__host__ __device__ __forceinline__ int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

}  // namespace pisa
