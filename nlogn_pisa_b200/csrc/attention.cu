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
// the general fallback for any indices.  Decode (and any short query run)
// with 16-bit inputs, block size 64 and D = Dv in {64, 128} takes the
// ring-staged form (attn_fwd_ring_kernel) below; prefill uses the
// block-bucketed tensor-core kernels.
#include <type_traits>

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

// Forward for 16-bit inputs, D = Dv in {64, 128}, block size 64, G <= 8 (the
// decode gather): one CTA of eight warps per (b, t, KV head) with all G query
// heads (one CTA per SM at D = 128: the fragments and the output
// accumulators take about 160 registers a thread).  The visible selected
// blocks stream through a six-stage cp.async ring in shared memory (64 keys +
// 64 values per stage, 16-byte chunks XOR-swizzled by key row so the fragment
// loads are conflict-free) and are consumed in pairs, so four blocks' loads
// (128 KB at D = 128) are in flight while a pair is scored and the gather is
// bound by HBM, not by load latency.  The math runs on mma.sync fragments
// (a SIMT form of it was bound by instruction issue): warp w owns keys
// 8w..8w+7 of every block,
//   logits   S = Q K^T with m16n8k16 (rows = the G heads, padded to 16; the
//            q fragments stay in registers for the whole row), scaled into
//            the exp2 domain
//   softmax  every warp keeps its own running max and sum per head over
//            its keys (no exchange between the warps inside the loop)
//   P.V      the S accumulator fragment, exponentiated and rounded to the
//            input type, is the A fragment of an m16n8k8 MMA against the
//            warp's 8 value rows (ldmatrix.trans), accumulated in registers
// The warps' runs (max, sum, output) are merged through shared memory at the
// end.
// Semantics as attn_fwd_kernel (probabilities rounded to the input type
// before P.V, as in the tensor-core prefill kernels).
constexpr int kRingThreads = 256, kRingStages = 6, kRingC = 64;

__device__ __forceinline__ void ring_cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void ring_zero16(uint32_t dst, const void* any_global) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, 0;" :: "r"(dst), "l"(any_global) : "memory");
}
__device__ __forceinline__ void ring_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void ring_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}
// d = A B (m16n8k16, fp32 accumulate from zero); A rows 8-15 are zero
template <typename T>
__device__ __forceinline__ void mma_k16_top(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  const uint32_t z = 0u;
  const float f = 0.f;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%10,%10,%10,%10};"
                 : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
                 : "r"(a0), "r"(z), "r"(a2), "r"(z), "r"(b0), "r"(b1), "f"(f));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%10,%10,%10,%10};"
                 : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
                 : "r"(a0), "r"(z), "r"(a2), "r"(z), "r"(b0), "r"(b1), "f"(f));
  }
}
// (c0, c1) += A B (m16n8k8) for rows 0-7; rows 8-15 of A are zero and their
// outputs are dropped
template <typename T>
__device__ __forceinline__ void mma_k8_top(float& c0, float& c1, uint32_t a0, uint32_t b0) {
  const uint32_t z = 0u;
  float d2, d3;
  const float f = 0.f;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%7,%7};"
                 : "+f"(c0), "+f"(c1), "=f"(d2), "=f"(d3) : "r"(a0), "r"(z), "r"(b0), "f"(f));
  } else {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%7,%7};"
                 : "+f"(c0), "+f"(c1), "=f"(d2), "=f"(d3) : "r"(a0), "r"(z), "r"(b0), "f"(f));
  }
}
template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <int D>
constexpr size_t ring_smem_bytes(int G, int S) {
  return size_t(kRingStages) * 2 * kRingC * D * 2 + size_t(8) * (D + 8) * 2 + size_t(S) * 4;
}

template <typename T, int G, int D>
__global__ void __launch_bounds__(kRingThreads, D == 64 ? 2 : 1) attn_fwd_ring_kernel(const AttnArgs a) {
  constexpr int kRow = D * 2;              // bytes per key or value row
  constexpr int kTile = kRingC * kRow;     // one K or V tile
  constexpr int kChunks = D / 8;           // 16-byte chunks per row
  constexpr int kWarpsR = kRingThreads / 32;
  constexpr float kLog2e = 1.4426950408889634f;
  static_assert(kWarpsR * 8 == kRingC, "one warp per 8 keys of a block");
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* ring = smem;                                          // stages x (K tile, V tile)
  // q rows of the G heads, zero rows up to 8, rows padded by 16 bytes so the
  // eight row addresses of an ldmatrix fall in distinct banks
  constexpr int kQRow = D + 8;
  T* qs = reinterpret_cast<T*>(smem + kRingStages * 2 * kTile);  // [8][kQRow]
  int* slots = reinterpret_cast<int*>(qs + 8 * kQRow);           // visible block ids, slot order
  __shared__ float lsum[kWarpsR][8], wmax[kWarpsR][8];           // the warps' running sums and maxima
  __shared__ int nvis_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = lane >> 2, tig = lane & 3;                     // fragment row (head), thread in group
  const int64_t item = blockIdx.x;
  const int h = int(item % a.H);
  const int t = int((item / a.H) % a.T);
  const int b = int(item / (int64_t(a.H) * a.T));
  const int64_t pos = a.positions ? a.positions[int64_t(b) * a.T + t] : a.pos_offset + t;

  {
    const T* qp = static_cast<const T*>(a.q) + b * a.q_sb + t * a.q_st + int64_t(h * G) * a.q_sh;
    for (int i = tid; i < 8 * D; i += kRingThreads) {
      const int g = i / D, d = i % D;
      qs[g * kQRow + d] = g < G ? qp[g * a.q_sh + d] : from_f32<T>(0.f);
    }
  }
  if (warp == 0) {
    int n = 0;
    for (int s0 = 0; s0 < a.S; s0 += 32) {
      const int s = s0 + lane;
      int64_t k0 = 0, k1 = 0;
      const bool vis = s < a.S && block_range(a, load_index(a.indices, a.index_bytes, item * a.S + s), pos, k0, k1);
      const unsigned bal = __ballot_sync(kFull, vis);
      if (vis) slots[n + __popc(bal & ((1u << lane) - 1u))] = int(k0 / kRingC);
      n += __popc(bal);
    }
    if (lane == 0) nvis_s = n;
  }
  __syncthreads();
  const int nvis = nvis_s;
  const T* kbase = static_cast<const T*>(a.k) + b * a.k_sb + int64_t(h) * a.k_sh;
  const T* vbase = static_cast<const T*>(a.v) + b * a.v_sb + int64_t(h) * a.v_sh;
  auto valid_keys = [&](int j) {
    const int64_t k0 = int64_t(slots[j]) * kRingC;
    int64_t k1 = min64(k0 + kRingC, a.N);
    if (a.causal) k1 = min64(k1, pos + 1);
    return int(k1 - k0);
  };
  // byte offset of 16-byte chunk ch of key row `row` in a tile
  auto chunk_off = [](int row, int ch) { return uint32_t(row * kRow + ((ch ^ (row & 7)) << 4)); };
  // keys and values of visible block j into stage st (rows past the valid
  // keys are zero-filled, so masked keys contribute 0 * 0 to P.V)
  // this thread copies chunk lch of rows lrow0 + r * kRowStep of every tile
  constexpr int kRowStep = kRingThreads / kChunks;
  const int lrow0 = tid / kChunks, lch = tid % kChunks;
  const T* kthr = kbase + lrow0 * a.k_st + lch * 8;
  const T* vthr = vbase + lrow0 * a.v_st + lch * 8;
  const int64_t kstep = int64_t(kRowStep) * a.k_st, vstep = int64_t(kRowStep) * a.v_st;
  auto load = [&](int j, int st) {
    const int64_t k0 = int64_t(slots[j]) * kRingC;
    const int nk = valid_keys(j);
    const uint32_t kd = smem_addr(ring + st * 2 * kTile), vd = kd + kTile;
    const T* kp = kthr + k0 * a.k_st;
    const T* vp = vthr + k0 * a.v_st;
#pragma unroll
    for (int r = 0; r < kRingC / kRowStep; ++r) {
      const int row = lrow0 + r * kRowStep;
      const uint32_t off = chunk_off(row, lch);
      if (row < nk) {
        ring_cp16(kd + off, kp);
        ring_cp16(vd + off, vp);
      } else {
        ring_zero16(kd + off, kbase);
        ring_zero16(vd + off, vbase);
      }
      kp += kstep;
      vp += vstep;
    }
  };
  // blocks are consumed in pairs (one commit group per pair); pairs p + 1 and
  // p + 2 are in flight while pair p is scored
  static_assert(kRingStages == 6, "three pairs of stages");
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j < nvis) load(j, j);
    if (j & 1) ring_commit();
  }

  // q A fragments come from shared memory by ldmatrix (row = head): matrix i
  // of an x4 load is 16-byte chunk 4c + i of rows 0-7
  const uint32_t q_addr = smem_addr(qs) + uint32_t((lane & 7) * kQRow * 2 + (lane >> 3) * 16);
  const float sl = a.scale * kLog2e;
  const int my_key = warp * 8 + (lane & 7), my_chunk = lane >> 3;   // ldmatrix row address of this lane
  const int key0 = warp * 8 + 2 * tig;                              // this lane's two logit columns
  float o[D / 8][2];                    // output of row grp, dims 8n + 2tig, +1 (this warp's keys)
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;

  // logits of head grp against keys 8w + 2tig, +1 of the block in stage st
  auto logits = [&](int st, int nk, float (&s)[2]) {
    const uint32_t Kt = smem_addr(ring + st * 2 * kTile);
    s[0] = s[1] = 0.f;
#pragma unroll
    for (int c4 = 0; c4 < kChunks / 4; ++c4) {
      uint32_t kb[4], qa[4];
      ldsm_x4(Kt + chunk_off(my_key, 4 * c4 + my_chunk), kb);
      ldsm_x4(q_addr + c4 * 64, qa);
      float d[4];
      mma_k16_top<T>(d, qa[0], qa[1], kb[0], kb[1]);
      s[0] += d[0]; s[1] += d[1];
      mma_k16_top<T>(d, qa[2], qa[3], kb[2], kb[3]);
      s[0] += d[0]; s[1] += d[1];
    }
    s[0] = key0 < nk ? s[0] * sl : -INFINITY;
    s[1] = key0 + 1 < nk ? s[1] * sl : -INFINITY;
  };
  // o += P V for this warp's eight value rows of the block in stage st
  auto pv = [&](int st, uint32_t pa) {
    const uint32_t Vt = smem_addr(ring + st * 2 * kTile) + kTile;
#pragma unroll
    for (int c4 = 0; c4 < kChunks / 4; ++c4) {
      uint32_t vb[4];
      ldsm_x4_trans(Vt + chunk_off(my_key, 4 * c4 + my_chunk), vb);
#pragma unroll
      for (int i = 0; i < 4; ++i) mma_k8_top<T>(o[4 * c4 + i][0], o[4 * c4 + i][1], pa, vb[i]);
    }
  };

  for (int j = 0; j < nvis; j += 2) {
    ring_wait<1>();
    __syncthreads();
    if (j + 4 < nvis) load(j + 4, (j + 4) % kRingStages);
    if (j + 5 < nvis) load(j + 5, (j + 5) % kRingStages);
    ring_commit();
    const bool two = j + 1 < nvis;   // uniform over the CTA
    float s0[2], s1[2] = {-INFINITY, -INFINITY};
    logits(j % kRingStages, valid_keys(j), s0);
    if (two) logits((j + 1) % kRingStages, valid_keys(j + 1), s1);
    // this warp's running max of row grp over its own keys of the pair (the
    // warps' runs are merged at the end); all its keys can be masked
    float bm = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s1[0], s1[1]));
    bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 1));
    bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 2));
    const float mn = fmaxf(m_run, bm);
    const float alpha = mn == m_run ? 1.f : exp2f(m_run - mn);   // m_run = -inf gives 0
    m_run = mn;
    float p[4];
    p[0] = s0[0] == -INFINITY ? 0.f : exp2f(s0[0] - mn);
    p[1] = s0[1] == -INFINITY ? 0.f : exp2f(s0[1] - mn);
    p[2] = s1[0] == -INFINITY ? 0.f : exp2f(s1[0] - mn);
    p[3] = s1[1] == -INFINITY ? 0.f : exp2f(s1[1] - mn);
    l_run = l_run * alpha + ((p[0] + p[1]) + (p[2] + p[3]));
#pragma unroll
    for (int n = 0; n < D / 8; ++n) { o[n][0] *= alpha; o[n][1] *= alpha; }
    pv(j % kRingStages, pack_pair<T>(p[0], p[1]));
    if (two) pv((j + 1) % kRingStages, pack_pair<T>(p[2], p[3]));
  }
  // add the warps' outputs and sums through the (now idle) ring
  asm volatile("cp.async.wait_all;" ::: "memory");
  l_run += __shfl_xor_sync(kFull, l_run, 1);
  l_run += __shfl_xor_sync(kFull, l_run, 2);
  __syncthreads();
  float* red = reinterpret_cast<float*>(ring);   // [warp][head][D]
  if (grp < G) {
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
      *reinterpret_cast<float2*>(red + (warp * G + grp) * D + 8 * n + 2 * tig) = make_float2(o[n][0], o[n][1]);
    if (tig == 0) { lsum[warp][grp] = l_run; wmax[warp][grp] = m_run; }
  }
  __syncthreads();
  T* op = static_cast<T*>(a.out) + ((int64_t(b) * a.T + t) * a.Hq + h * G) * D;
  for (int i = tid; i < G * D; i += kRingThreads) {
    const int g = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarpsR; ++w) M = fmaxf(M, wmax[w][g]);
    float sum = 0.f, L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarpsR; ++w) {
        const float mw = wmax[w][g];
        if (mw == -INFINITY) continue;
        const float f = exp2f(mw - M);
        sum = fmaf(red[(w * G + g) * D + d], f, sum);
        L = fmaf(lsum[w][g], f, L);
      }
    }
    op[i] = from_f32<T>(L > 0.f ? sum / L : 0.f);
    if (d == 0 && a.lse)
      a.lse[(int64_t(b) * a.T + t) * a.Hq + h * G + g] = L > 0.f ? (M + log2f(L)) / kLog2e : -INFINITY;
  }
}

template <typename T, int G, int D>
int fwd_ring_launch(const AttnArgs& a, cudaStream_t stream) {
  auto kernel = attn_fwd_ring_kernel<T, G, D>;
  const size_t smem = ring_smem_bytes<D>(G, a.S);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return fail_cuda(e, "attention ring smem attribute");
  const int64_t blocks = int64_t(a.B) * a.T * a.H;
  if (blocks == 0) return PISA_OK;
  kernel<<<unsigned(blocks), kRingThreads, smem, stream>>>(a);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

template <typename T, int D>
int fwd_ring(const AttnArgs& a, cudaStream_t s) {
  switch (a.G) {
    case 1: return fwd_ring_launch<T, 1, D>(a, s);
    case 2: return fwd_ring_launch<T, 2, D>(a, s);
    case 4: return fwd_ring_launch<T, 4, D>(a, s);
    default: return fwd_ring_launch<T, 8, D>(a, s);
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
    // the ring-staged gather: block size 64, D = Dv in {64, 128}, up to 8
    // query heads per KV head, slot list within shared memory
    const bool ring = coop && a.C == kRingC && (a.D == 64 || a.D == 128) &&
                      (a.G == 1 || a.G == 2 || a.G == 4 || a.G == 8) && a.S <= 4096;
    if (ring) return a.D == 64 ? fwd_ring<T, 64>(a, s) : fwd_ring<T, 128>(a, s);
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
