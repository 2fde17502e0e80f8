// K4 (gather form): attention over selected key blocks, forward and backward.
//
// Semantics of sparse_attention_torch (pisa/pisa/ops/flash_sparse_attn/
// sparse_attn/sparse_attn_torch.py:6-35): for query (b, t, head) the keys are
// the tokens id*C .. id*C+C-1 of every selected id (in slot order; duplicates
// count once per occurrence) that satisfy 0 <= token < N and, when causal,
// token <= position; one softmax over all of them with logits scale * q.k;
// rows without a visible key output 0 (lse = -inf).
//
// This form gives one CTA of four warps to one (b, t, KV head, group of up to
// four query heads): warps take slots round-robin, lanes own keys for the
// logits (q rows broadcast from shared memory) and own value columns for
// P.V, with a per-warp online softmax merged across warps at the end.  It is
// the decode path and the general fallback for any indices; prefill uses the
// block-bucketed tensor-core kernels.
#include "internal.h"

namespace pisa {

namespace {

constexpr int kWarps = 4;

template <typename T, int GC>
__device__ __forceinline__ void dots_gc(const T* __restrict__ row, const float* __restrict__ qs,
                                        int D, float (&acc)[GC]) {
  constexpr int V = Vec<T>::N;
#pragma unroll
  for (int g = 0; g < GC; ++g) acc[g] = 0.f;
  for (int d = 0; d < D; d += V) {
    float x[V];
    load_vec<T>(row + d, x);
#pragma unroll
    for (int g = 0; g < GC; ++g) {
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

__device__ __forceinline__ int64_t load_index(const void* p, int bytes, int64_t i) {
  return bytes == 4 ? int64_t(static_cast<const int32_t*>(p)[i]) : static_cast<const int64_t*>(p)[i];
}

// Key range [k0, k1) of a selected id, empty when the id contributes nothing.
__device__ __forceinline__ bool block_range(const AttnArgs& a, int64_t id, int64_t pos, int64_t& k0,
                                            int64_t& k1) {
  if (id < 0) return false;
  k0 = id * a.C;
  if (k0 >= a.N) return false;
  k1 = min64(k0 + a.C, a.N);
  if (a.causal) k1 = min64(k1, pos + 1);
  return k1 > k0;
}

template <typename T, int GC, int DPL>
__global__ void __launch_bounds__(kWarps * 32) attn_fwd_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                         // [GC][D]
  float* pw = qs + GC * a.D;              // [warps][GC][32]
  float* mw = pw + kWarps * GC * 32;      // [warps][GC]
  float* lw = mw + kWarps * GC;           // [warps][GC]
  float* ow = lw + kWarps * GC;           // [warps][GC][Dv]

  const int chunks = (a.G + GC - 1) / GC;
  const int chunk = blockIdx.x % chunks;
  const int64_t item = blockIdx.x / chunks;
  const int h = int(item % a.H);
  const int t = int((item / a.H) % a.T);
  const int b = int(item / (int64_t(a.H) * a.T));
  const int g0 = chunk * GC;
  const int gn = min(GC, a.G - g0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t pos = a.positions ? a.positions[int64_t(b) * a.T + t] : a.pos_offset + t;

  const T* qp = static_cast<const T*>(a.q) + b * a.q_sb + t * a.q_st + int64_t(h * a.G + g0) * a.q_sh;
  for (int e = tid; e < GC * a.D; e += blockDim.x) {
    const int g = e / a.D, d = e % a.D;
    qs[e] = g < gn ? to_f32<T>(qp[g * a.q_sh + d]) : 0.f;
  }
  __syncthreads();

  const T* kb = static_cast<const T*>(a.k) + b * a.k_sb + int64_t(h) * a.k_sh;
  const T* vb = static_cast<const T*>(a.v) + b * a.v_sb + int64_t(h) * a.v_sh;
  float m[GC], l[GC], o[GC][DPL];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) o[g][i] = 0.f;
  }
  float* pwarp = pw + warp * GC * 32;
  for (int s = warp; s < a.S; s += kWarps) {
    int64_t k0, k1;
    if (!block_range(a, load_index(a.indices, a.index_bytes, item * a.S + s), pos, k0, k1)) continue;
    for (int64_t base = k0; base < k1; base += 32) {
      const int64_t j = base + lane;
      const bool valid = j < k1;
      float z[GC];
      if (valid) {
        dots_gc<T, GC>(kb + j * a.k_st, qs, a.D, z);
#pragma unroll
        for (int g = 0; g < GC; ++g) z[g] *= a.scale;
      } else {
#pragma unroll
        for (int g = 0; g < GC; ++g) z[g] = -INFINITY;
      }
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        const float mnew = fmaxf(m[g], warp_max(z[g]));
        const float alpha = m[g] == -INFINITY ? 0.f : expf(m[g] - mnew);
        const float p = valid ? expf(z[g] - mnew) : 0.f;
        l[g] = l[g] * alpha + warp_sum(p);
        m[g] = mnew;
#pragma unroll
        for (int i = 0; i < DPL; ++i) o[g][i] *= alpha;
        pwarp[g * 32 + lane] = p;
      }
      __syncwarp();
      const int nk = int(min64(32, k1 - base));
      for (int jj = 0; jj < nk; ++jj) {
        const T* vrow = vb + (base + jj) * a.v_st;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const int d = lane + 32 * i;
          if (d < a.Dv) {
            const float vv = to_f32<T>(vrow[d]);
#pragma unroll
            for (int g = 0; g < GC; ++g) o[g][i] = fmaf(pwarp[g * 32 + jj], vv, o[g][i]);
          }
        }
      }
      __syncwarp();
    }
  }
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    if (lane == 0) { mw[warp * GC + g] = m[g]; lw[warp * GC + g] = l[g]; }
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = lane + 32 * i;
      if (d < a.Dv) ow[(warp * GC + g) * a.Dv + d] = o[g][i];
    }
  }
  __syncthreads();
  T* op = static_cast<T*>(a.out) + ((int64_t(b) * a.T + t) * a.Hq + h * a.G + g0) * a.Dv;
  for (int e = tid; e < gn * a.Dv; e += blockDim.x) {
    const int g = e / a.Dv, d = e % a.Dv;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mw[w * GC + g]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mwg = mw[w * GC + g];
        if (mwg == -INFINITY) continue;
        const float f = expf(mwg - M);
        L += lw[w * GC + g] * f;
        O += ow[(w * GC + g) * a.Dv + d] * f;
      }
    }
    op[e] = from_f32<T>(L > 0.f ? O / L : 0.f);
    if (d == 0 && a.lse) {
      a.lse[(int64_t(b) * a.T + t) * a.Hq + h * a.G + g0 + g] = L > 0.f ? M + logf(L) : -INFINITY;
    }
  }
}

// Forward for 16-bit inputs with D = Dv in {64, 128, 256} (E = D/16): logits
// with lane = key (the whole key row per lane, many loads in flight), online
// softmax with lane = key, then P.V with a half-warp per value row (16 lanes
// x 2E bytes, two rows per warp instruction, four instructions in flight),
// lanes owning E columns and the two halves summed at the end.
template <typename T, int GC, int E>
__global__ void __launch_bounds__(kWarps * 32) attn_fwd_coop_kernel(const AttnArgs a) {
  constexpr int D = 16 * E;
  __shared__ float zs[kWarps][GC][32];
  __shared__ float mw[kWarps][GC], lw[kWarps][GC];
  __shared__ float ow[kWarps][GC][D];

  const int chunks = (a.G + GC - 1) / GC;
  const int chunk = blockIdx.x % chunks;
  const int64_t item = blockIdx.x / chunks;
  const int h = int(item % a.H);
  const int t = int((item / a.H) % a.T);
  const int b = int(item / (int64_t(a.H) * a.T));
  const int g0 = chunk * GC;
  const int gn = min(GC, a.G - g0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int half = lane >> 4, l16 = lane & 15;
  const int64_t pos = a.positions ? a.positions[int64_t(b) * a.T + t] : a.pos_offset + t;

  // query heads (scaled) in shared memory, read as broadcasts by the logits
  __shared__ __align__(16) float qsm[GC * D];
  {
    const T* qp = static_cast<const T*>(a.q) + b * a.q_sb + t * a.q_st + int64_t(h * a.G + g0) * a.q_sh;
    for (int i = tid; i < GC * D; i += blockDim.x) {
      const int g = i / D, d = i % D;
      qsm[i] = g < gn ? to_f32<T>(qp[g * a.q_sh + d]) * a.scale : 0.f;
    }
  }
  __syncthreads();
  const T* kfull = static_cast<const T*>(a.k) + b * a.k_sb + int64_t(h) * a.k_sh;
  const T* vb = static_cast<const T*>(a.v) + b * a.v_sb + int64_t(h) * a.v_sh + l16 * E;
  float m[GC], l[GC], o[GC][E];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) o[g][e] = 0.f;
  }
  auto load_row = [&](const T* p, uint32_t (&w)[E / 2]) {
#pragma unroll
    for (int c = 0; c < E / 8; ++c) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + c);
      w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
    }
    if constexpr (E == 4) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
      w[0] = v.x; w[1] = v.y;
    }
  };
  for (int s = warp; s < a.S; s += kWarps) {
    int64_t k0, k1;
    if (!block_range(a, load_index(a.indices, a.index_bytes, item * a.S + s), pos, k0, k1)) continue;
    for (int64_t base = k0; base < k1; base += 32) {
      const int nk = int(min64(32, k1 - base));
      // logits with lane = key: each lane reads its whole key row (D/8
      // independent 16-byte loads in flight), q from shared memory
      {
        const int kk = lane;
        float z[GC];
        if (kk < nk) {
          dots_gc<T, GC>(kfull + (base + kk) * a.k_st, qsm, D, z);
        } else {
#pragma unroll
          for (int g = 0; g < GC; ++g) z[g] = -INFINITY;
        }
#pragma unroll
        for (int g = 0; g < GC; ++g) zs[warp][g][kk] = z[g];
      }
      __syncwarp();
      // online softmax with lane = key
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        const float zv = zs[warp][g][lane];
        const float mnew = fmaxf(m[g], warp_max(zv));
        const float alpha = m[g] == -INFINITY ? 0.f : expf(m[g] - mnew);
        const float pv = zv == -INFINITY ? 0.f : expf(zv - mnew);
        l[g] = l[g] * alpha + warp_sum(pv);
        m[g] = mnew;
#pragma unroll
        for (int e = 0; e < E; ++e) o[g][e] *= alpha;
        zs[warp][g][lane] = pv;
      }
      __syncwarp();
      // P.V: value rows base + jj + half
      for (int j0 = 0; j0 < nk; j0 += 8) {
        uint32_t w[4][E / 2];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int kk = j0 + 2 * u + half;
          if (kk < nk) load_row(vb + (base + kk) * a.v_st, w[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int kk = j0 + 2 * u + half;
          if (kk < nk) {
            const T* x = reinterpret_cast<const T*>(w[u]);
#pragma unroll
            for (int g = 0; g < GC; ++g) {
              const float pv = zs[warp][g][kk];
#pragma unroll
              for (int e = 0; e < E; ++e) o[g][e] = fmaf(pv, to_f32<T>(x[e]), o[g][e]);
            }
          }
        }
      }
      __syncwarp();
    }
  }
#pragma unroll
  for (int g = 0; g < GC; ++g) {
#pragma unroll
    for (int e = 0; e < E; ++e) o[g][e] += __shfl_xor_sync(kFull, o[g][e], 16);
    if (lane == 0) { mw[warp][g] = m[g]; lw[warp][g] = l[g]; }
    if (half == 0) {
#pragma unroll
      for (int e = 0; e < E; ++e) ow[warp][g][l16 * E + e] = o[g][e];
    }
  }
  __syncthreads();
  T* op = static_cast<T*>(a.out) + ((int64_t(b) * a.T + t) * a.Hq + h * a.G + g0) * D;
  for (int i = tid; i < gn * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mw[w][g]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (mw[w][g] == -INFINITY) continue;
        const float f = expf(mw[w][g] - M);
        L += lw[w][g] * f;
        O += ow[w][g][d] * f;
      }
    }
    op[i] = from_f32<T>(L > 0.f ? O / L : 0.f);
    if (d == 0 && a.lse) a.lse[(int64_t(b) * a.T + t) * a.Hq + h * a.G + g0 + g] = L > 0.f ? M + logf(L) : -INFINITY;
  }
}

template <typename T, int GC, int DPL>
__global__ void __launch_bounds__(kWarps * 32) attn_bwd_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                        // [GC][D]
  float* dos = qs + GC * a.D;            // [GC][Dv]
  float* lse_s = dos + GC * a.Dv;        // [GC]
  float* delta = lse_s + GC;             // [GC]
  float* pw = delta + GC;                // [warps][GC][32]
  float* dsw = pw + kWarps * GC * 32;    // [warps][GC][32]
  float* dqw = dsw + kWarps * GC * 32;   // [warps][GC][D]

  const int chunks = (a.G + GC - 1) / GC;
  const int chunk = blockIdx.x % chunks;
  const int64_t item = blockIdx.x / chunks;
  const int h = int(item % a.H);
  const int t = int((item / a.H) % a.T);
  const int b = int(item / (int64_t(a.H) * a.T));
  const int g0 = chunk * GC;
  const int gn = min(GC, a.G - g0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t pos = a.positions ? a.positions[int64_t(b) * a.T + t] : a.pos_offset + t;
  const int64_t row0 = (int64_t(b) * a.T + t) * a.Hq + h * a.G + g0;  // first query-head row

  const T* qp = static_cast<const T*>(a.q) + row0 * a.D;
  const T* dop = static_cast<const T*>(a.dout) + row0 * a.Dv;
  const T* opp = static_cast<const T*>(a.o) + row0 * a.Dv;
  for (int e = tid; e < GC * a.D; e += blockDim.x) qs[e] = e / a.D < gn ? to_f32<T>(qp[e]) : 0.f;
  for (int e = tid; e < GC * a.Dv; e += blockDim.x) dos[e] = e / a.Dv < gn ? to_f32<T>(dop[e]) : 0.f;
  // delta_g = sum_d dout . out  (one warp per head)
  for (int g = warp; g < GC; g += kWarps) {
    float acc = 0.f;
    if (g < gn)
      for (int d = lane; d < a.Dv; d += 32) acc += to_f32<T>(dop[g * a.Dv + d]) * to_f32<T>(opp[g * a.Dv + d]);
    acc = warp_sum(acc);
    if (lane == 0) {
      delta[g] = acc;
      lse_s[g] = g < gn ? a.lse_in[row0 + g] : -INFINITY;
    }
  }
  __syncthreads();

  const T* kb = static_cast<const T*>(a.k) + (int64_t(b) * a.N * a.H + h) * a.D;
  const T* vb = static_cast<const T*>(a.v) + (int64_t(b) * a.N * a.H + h) * a.Dv;
  float* dkb = a.dk_acc + (int64_t(b) * a.N * a.H + h) * a.D;
  float* dvb = a.dv_acc + (int64_t(b) * a.N * a.H + h) * a.Dv;
  const int64_t kst = int64_t(a.H) * a.D, vst = int64_t(a.H) * a.Dv;
  float dq[GC][DPL];
#pragma unroll
  for (int g = 0; g < GC; ++g)
#pragma unroll
    for (int i = 0; i < DPL; ++i) dq[g][i] = 0.f;
  float* pwarp = pw + warp * GC * 32;
  float* dswarp = dsw + warp * GC * 32;
  for (int s = warp; s < a.S; s += kWarps) {
    int64_t k0, k1;
    if (!block_range(a, load_index(a.indices, a.index_bytes, item * a.S + s), pos, k0, k1)) continue;
    for (int64_t base = k0; base < k1; base += 32) {
      const int64_t j = base + lane;
      const bool valid = j < k1;
      float z[GC], dp[GC];
      if (valid) {
        dots_gc<T, GC>(kb + j * kst, qs, a.D, z);
        dots_gc<T, GC>(vb + j * vst, dos, a.Dv, dp);
      }
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        const float L = lse_s[g];
        const float p = (valid && L != -INFINITY) ? expf(z[g] * a.scale - L) : 0.f;
        pwarp[g * 32 + lane] = p;
        dswarp[g * 32 + lane] = valid ? p * (dp[g] - delta[g]) : 0.f;
      }
      __syncwarp();
      const int nk = int(min64(32, k1 - base));
      for (int jj = 0; jj < nk; ++jj) {
        const int64_t key = base + jj;
        for (int d = lane; d < a.Dv; d += 32) {
          float acc = 0.f;
#pragma unroll
          for (int g = 0; g < GC; ++g) acc = fmaf(pwarp[g * 32 + jj], dos[g * a.Dv + d], acc);
          atomicAdd(dvb + key * vst + d, acc);
        }
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const int d = lane + 32 * i;
          if (d < a.D) {
            const float kv = to_f32<T>(kb[key * kst + d]);
            float acc = 0.f;
#pragma unroll
            for (int g = 0; g < GC; ++g) {
              const float ds = dswarp[g * 32 + jj];
              acc = fmaf(ds, qs[g * a.D + d], acc);
              dq[g][i] = fmaf(ds, kv, dq[g][i]);
            }
            atomicAdd(dkb + key * kst + d, acc * a.scale);
          }
        }
      }
      __syncwarp();
    }
  }
#pragma unroll
  for (int g = 0; g < GC; ++g)
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = lane + 32 * i;
      if (d < a.D) dqw[(warp * GC + g) * a.D + d] = dq[g][i];
    }
  __syncthreads();
  T* dqp = static_cast<T*>(a.dq) + row0 * a.D;
  for (int e = tid; e < gn * a.D; e += blockDim.x) {
    const int g = e / a.D, d = e % a.D;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) acc += dqw[(w * GC + g) * a.D + d];
    dqp[e] = from_f32<T>(acc * a.scale);
  }
}

template <typename T>
__global__ void convert_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    dst[i] = from_f32<T>(src[i]);
}

template <typename T, int GC, int DPL>
int launch_fwd(const AttnArgs& a, cudaStream_t stream) {
  const size_t smem = sizeof(float) * (GC * a.D + kWarps * GC * 32 + 2 * kWarps * GC + kWarps * GC * a.Dv);
  auto kernel = attn_fwd_kernel<T, GC, DPL>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return fail_cuda(e, "attention smem attribute");
  }
  const int64_t blocks = int64_t(a.B) * a.T * a.H * ((a.G + GC - 1) / GC);
  if (blocks == 0) return PISA_OK;
  kernel<<<unsigned(blocks), kWarps * 32, smem, stream>>>(a);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

template <typename T, int GC, int DPL>
int launch_bwd(const AttnArgs& a, cudaStream_t stream) {
  const size_t smem = sizeof(float) * (GC * a.D + GC * a.Dv + 2 * GC + 2 * kWarps * GC * 32 + kWarps * GC * a.D);
  auto kernel = attn_bwd_kernel<T, GC, DPL>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return fail_cuda(e, "attention bwd smem attribute");
  }
  const int64_t blocks = int64_t(a.B) * a.T * a.H * ((a.G + GC - 1) / GC);
  if (blocks == 0) return PISA_OK;
  kernel<<<unsigned(blocks), kWarps * 32, smem, stream>>>(a);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

template <typename T, int GC>
int fwd_dpl(const AttnArgs& a, cudaStream_t s) {
  const int d = max(a.D, a.Dv);
  if (d <= 32) return launch_fwd<T, GC, 1>(a, s);
  if (d <= 64) return launch_fwd<T, GC, 2>(a, s);
  if (d <= 128) return launch_fwd<T, GC, 4>(a, s);
  return launch_fwd<T, GC, 8>(a, s);
}

template <typename T, int GC>
int bwd_dpl(const AttnArgs& a, cudaStream_t s) {
  const int d = max(a.D, a.Dv);
  if (d <= 32) return launch_bwd<T, GC, 1>(a, s);
  if (d <= 64) return launch_bwd<T, GC, 2>(a, s);
  if (d <= 128) return launch_bwd<T, GC, 4>(a, s);
  return launch_bwd<T, GC, 8>(a, s);
}

template <typename T, int GC, int E>
int fwd_coop_launch(const AttnArgs& a, cudaStream_t stream) {
  auto kernel = attn_fwd_coop_kernel<T, GC, E>;
  const int64_t blocks = int64_t(a.B) * a.T * a.H * ((a.G + GC - 1) / GC);
  if (blocks == 0) return PISA_OK;
  kernel<<<unsigned(blocks), kWarps * 32, 0, stream>>>(a);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

template <typename T, int GC>
int fwd_coop(const AttnArgs& a, cudaStream_t s) {
  if (a.D == 64) return fwd_coop_launch<T, GC, 4>(a, s);
  if (a.D == 128) return fwd_coop_launch<T, GC, 8>(a, s);
  return fwd_coop_launch<T, GC, 16>(a, s);
}

template <typename T>
int fwd_t(const AttnArgs& a, cudaStream_t s) {
  if constexpr (sizeof(T) == 2) {
    // rows of 64, 128 or 256 16-bit elements, 16-byte aligned (checked by the caller)
    const bool coop = a.D == a.Dv && (a.D == 64 || a.D == 128 || a.D == 256) && a.k_st % 8 == 0 &&
                      a.v_st % 8 == 0 && a.k_sb % 8 == 0 && a.v_sb % 8 == 0 && a.k_sh % 8 == 0 && a.v_sh % 8 == 0;
    if (coop) {
      if (a.G == 1) return fwd_coop<T, 1>(a, s);
      if (a.G == 2) return fwd_coop<T, 2>(a, s);
      return fwd_coop<T, 4>(a, s);
    }
  }
  if (a.G == 1) return fwd_dpl<T, 1>(a, s);
  if (a.G == 2) return fwd_dpl<T, 2>(a, s);
  return fwd_dpl<T, 4>(a, s);
}

template <typename T>
int bwd_t(const AttnArgs& a, void* dk, void* dv, cudaStream_t s) {
  int rc;
  if (a.G == 1) rc = bwd_dpl<T, 1>(a, s);
  else if (a.G == 2) rc = bwd_dpl<T, 2>(a, s);
  else rc = bwd_dpl<T, 4>(a, s);
  if (rc != PISA_OK) return rc;
  const int64_t nk = int64_t(a.B) * a.N * a.H * a.D, nv = int64_t(a.B) * a.N * a.H * a.Dv;
  convert_kernel<T><<<1184, 256, 0, s>>>(a.dk_acc, static_cast<T*>(dk), nk);
  PISA_CHECK_LAUNCH();
  convert_kernel<T><<<1184, 256, 0, s>>>(a.dv_acc, static_cast<T*>(dv), nv);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

}  // namespace

int attn_fwd(const AttnArgs& a, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case PISA_F32: return fwd_t<float>(a, stream);
    case PISA_BF16: return fwd_t<__nv_bfloat16>(a, stream);
    case PISA_F16: return fwd_t<__half>(a, stream);
  }
  return fail(PISA_ERR_UNSUPPORTED, "unsupported dtype");
}

int attn_bwd(const AttnArgs& a, int dtype, void* dk, void* dv, cudaStream_t stream) {
  switch (dtype) {
    case PISA_F32: return bwd_t<float>(a, dk, dv, stream);
    case PISA_BF16: return bwd_t<__nv_bfloat16>(a, dk, dv, stream);
    case PISA_F16: return bwd_t<__half>(a, dk, dv, stream);
  }
  return fail(PISA_ERR_UNSUPPORTED, "unsupported dtype");
}

}  // namespace pisa
