// Per-candidate scores of the routing equations (top_k_pyramid_torch.py:48-80),
// SIMT forms shared by the per-item router (router.cu) and the standalone
// leaf scorer (leafscore.cu).  Scores are fp32 and summed over the G query
// heads of a KV head; `qs` holds the G query rows in fp32 ([G][D]).
#pragma once

#include "internal.h"

namespace pisa {

// acc[g] = row . q_g for the G query rows of `qs` ([G][D] fp32 in shared
// memory, read as broadcasts).  The row's 16-byte vectors are fetched eight
// at a time before any arithmetic, so a row costs one or two memory round
// trips instead of one per vector.
template <typename T, int GMAX>
__device__ __forceinline__ void row_dots(const T* __restrict__ row, const float* __restrict__ qs,
                                         int G, int D, float (&acc)[GMAX]) {
  constexpr int V = Vec<T>::N;
  constexpr int NB = 8;                      // vectors in flight
#pragma unroll
  for (int g = 0; g < GMAX; ++g) acc[g] = 0.f;
  for (int d0 = 0; d0 < D; d0 += NB * V) {
    uint4 raw[NB];
#pragma unroll
    for (int u = 0; u < NB; ++u)
      raw[u] = d0 + u * V < D ? __ldg(reinterpret_cast<const uint4*>(row + d0 + u * V)) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      if (d0 + u * V >= D) break;
      float x[V];
      if constexpr (sizeof(T) == 4) {
        x[0] = __uint_as_float(raw[u].x); x[1] = __uint_as_float(raw[u].y);
        x[2] = __uint_as_float(raw[u].z); x[3] = __uint_as_float(raw[u].w);
      } else {
        const T* e = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
        for (int i = 0; i < V; ++i) x[i] = to_f32<T>(e[i]);
      }
      const int d = d0 + u * V;
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        if (g < G) {
          const float* qg = qs + g * D + d;
#pragma unroll
          for (int i = 0; i < V; i += 4) {
            const float4 qv = *reinterpret_cast<const float4*>(qg + i);
            acc[g] = fmaf(qv.x, x[i + 0], acc[g]);
            acc[g] = fmaf(qv.y, x[i + 1], acc[g]);
            acc[g] = fmaf(qv.z, x[i + 2], acc[g]);
            acc[g] = fmaf(qv.w, x[i + 3], acc[g]);
          }
        }
      }
    }
  }
}

// Score of one coarse candidate (level >= 1) from its `br` child summaries,
// or of one node (pisa1, support 1).  Thread-local.
template <typename T, int GMAX>
__device__ float coarse_score(const RouteArgs& a, const T* level_base, int child_len, int id,
                              const float* qs) {
  const int64_t node_stride = int64_t(a.H) * a.D;
  float acc[GMAX];
  if (a.method == PISA_METHOD_PISA1) {
    row_dots<T, GMAX>(level_base + int64_t(id) * node_stride, qs, a.G, a.D, acc);
    float score = 0.f;
#pragma unroll
    for (int g = 0; g < GMAX; ++g)
      if (g < a.G) score += acc[g];
    return score;
  }
  // pisa: running max m / scaled sum s; pisa2 binary: z0, z1; pisa2 general:
  // sum of products s1 and of squares s2.
  float m[GMAX], s[GMAX], z0[GMAX], z1[GMAX], s1[GMAX], s2[GMAX];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    m[g] = -INFINITY; s[g] = 0.f; z0[g] = 0.f; z1[g] = 0.f; s1[g] = 0.f; s2[g] = 0.f;
  }
  int count = 0;
  const bool binary = a.br == 2;
  float score = 0.f;
  for (int j = 0; j < a.br; ++j) {
    const int c = id * a.br + j;
    if (c >= child_len) break;
    row_dots<T, GMAX>(level_base + int64_t(c) * node_stride, qs, a.G, a.D, acc);
    ++count;
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      if (g >= a.G) continue;
      if (a.method == PISA_METHOD_PISA) {
        const float z = acc[g] * a.scale;
        if (z > m[g]) { s[g] = s[g] * expf(m[g] - z) + 1.f; m[g] = z; }
        else { s[g] += expf(z - m[g]); }
      } else if (binary) {
        const float z = acc[g] * a.scale;
        if (j == 0) z0[g] = z; else z1[g] = z;
      } else {
        s1[g] += acc[g];
        s2[g] += acc[g] * acc[g];
      }
    }
  }
  const float cnt = float(count > 0 ? count : 1);
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    if (g >= a.G) continue;
    if (a.method == PISA_METHOD_PISA) {
      score += m[g] + logf(s[g]);
    } else if (binary) {
      const float total = z0[g] + z1[g];
      const float diff = z0[g] - z1[g];
      score += count == 2 ? 0.5f * total + 0.125f * diff * diff : total;
    } else {
      const float mean = s1[g] / cnt;
      const float second = s2[g] / cnt;
      const float var = fmaxf(second - mean * mean, 0.f);
      score += a.scale * mean + a.c2 * var;
    }
  }
  return score;
}

// Score of one leaf candidate from its C raw keys; executed by a whole warp.
template <typename T, int GMAX>
__device__ float leaf_score_warp(const RouteArgs& a, const T* key_base, int id, const float* qs,
                                 int lane) {
  float m[GMAX], s[GMAX], s2[GMAX], acc[GMAX];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) { m[g] = -INFINITY; s[g] = 0.f; s2[g] = 0.f; }
  int count = 0;
  const int64_t first = int64_t(id) * a.C;
  for (int kk = lane; kk < a.C; kk += 32) {
    const int64_t tok = first + kk;
    if (tok >= a.N) break;
    row_dots<T, GMAX>(key_base + tok * a.k_st, qs, a.G, a.D, acc);
    ++count;
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      if (g >= a.G) continue;
      if (a.method == PISA_METHOD_PISA) {
        const float z = acc[g] * a.scale;
        if (z > m[g]) { s[g] = s[g] * expf(m[g] - z) + 1.f; m[g] = z; }
        else { s[g] += expf(z - m[g]); }
      } else {
        s[g] += acc[g];
        s2[g] += acc[g] * acc[g];
      }
    }
  }
  float score = 0.f;
  if (a.method == PISA_METHOD_PISA) {
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      if (g >= a.G) continue;
      const float M = warp_max(m[g]);
      const float part = m[g] == -INFINITY ? 0.f : s[g] * expf(m[g] - M);
      const float S = warp_sum(part);
      score += M + logf(S);
    }
  } else {
    int total = count;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(kFull, total, o);
    const float cnt = float(total > 0 ? total : 1);
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      if (g >= a.G) continue;
      const float mean = warp_sum(s[g]) / cnt;
      const float second = warp_sum(s2[g]) / cnt;
      const float var = fmaxf(second - mean * mean, 0.f);
      score += a.scale * mean + a.c2 * var;
    }
  }
  return score;
}

}  // namespace pisa
