// Flat BSA block selection: the comparator the reference benchmarks PISA
// against, on the same leaf means as the pyramid.
//
// Restates bsa_select (pisa/pisa/ops/flash_sparse_attn/bsa/bsa_torch.py:63-106)
// and its streaming comparison network (bsa_torch.py:9-60; the GPU form is
// bsa_triton.py:12-83).  For one query token and KV head:
//   q'         = round_to_dtype(q * D^-0.5) per query head (bsa_torch.py:83-84)
//   logit_j    = q' . mean_j over the leaf means of the KV head, fp32
//   normaliser = LSE of the logits of the complete blocks j < (pos+1)//C,
//                0 when there is none (:88-90)
//   p_j        = exp(logit_j - normaliser) for j < pos//C, else 0; required
//                blocks (first, the force_recent most recent) get 1 (:91-99)
//   score_j    = sum of p_j over the G query heads; id_j = j if j <= pos//C
//                else -1 (:100-101)
//   top-K      blocks in tiles of W = pow2(max(C, 2K)): each tile is sorted
//              into alternating runs, merged ascending, its lower half
//              replaced by the retained best half, then merged descending;
//              tiles without a valid id are skipped (:30-60).  Ties follow
//              the network (equal scores exchange in descending runs only).
//
// Layout of the work.  A warp owns 16 query rows: TPW = 16 / G consecutive
// tokens x G heads of one (batch, KV head).  The logits of 8 blocks at a time
// are one m16n8k16 MMA per 16 head dims (bf16/fp16 in, fp32 accumulate; the
// fragment map is the router's: lane c holds dims 32p+8c..32p+8c+7 of pair
// step p), or the same 16 x 8 tile by FMAs for fp32 inputs.  Pass 1 keeps a
// running max / sum per row for the normaliser; pass 2 recomputes the logits
// tile by tile, writes the per-row probabilities of a tile to shared memory,
// and the warp then runs each token's network over the tile with the head sum
// taken on the way in (element i of the W-wide network in lane i % 32, slot
// i / 32).  The retained lists live in shared memory.
#include <algorithm>
#include <cmath>
#include <type_traits>

#include "internal.h"

namespace pisa {

namespace {

constexpr int kRows = 16;      // query rows per warp (the MMA's M)
constexpr int kMaxWarps = 8;

template <typename T>
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

struct BsaArgs {
  const void* q;
  int64_t q_sb, q_st, q_sh;
  const void* means;      // [B, M, H, D], node stride H*D
  int64_t m_sb;
  const int64_t* positions;
  int64_t pos_offset;
  int B, T, H, G, D, M, C, K, TPW, force_first, force_recent;
  float scale;
  int64_t* out;           // [B, T, H, K]
};

// One pass of bitonic merging of runs of 2^STAGE over a W-wide network held
// as E = W/32 slots per lane (element i = e*32 + lane).  MODE < 0: run r
// descends when bit STAGE of its elements is set; 0: every run ascends; 1:
// every run descends.  A pair exchanges when (lower > upper) != descending.
template <int W, int STAGE, int MODE>
__device__ __forceinline__ void merge_pass(float (&s)[W >= 32 ? W / 32 : 1], int (&id)[W >= 32 ? W / 32 : 1],
                                           int lane) {
  constexpr int E = W >= 32 ? W / 32 : 1;
#pragma unroll
  for (int ex = STAGE - 1; ex >= 0; --ex) {
    const int d = 1 << ex;
    if (d < 32) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = e * 32 + lane;
        const float ps = __shfl_xor_sync(kFull, s[e], d);
        const int pid = __shfl_xor_sync(kFull, id[e], d);
        const bool desc = MODE < 0 ? ((i >> STAGE) & 1) != 0 : MODE == 1;
        const bool lower = (i & d) == 0;
        const float lo = lower ? s[e] : ps;
        const float hi = lower ? ps : s[e];
        if ((lo > hi) != desc) { s[e] = ps; id[e] = pid; }
      }
    } else {
      const int de = d / 32;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if ((e & de) == 0) {
          const int f = e | de;
          const int i = e * 32 + lane;
          const bool desc = MODE < 0 ? ((i >> STAGE) & 1) != 0 : MODE == 1;
          if ((s[e] > s[f]) != desc) {
            const float ts = s[e]; s[e] = s[f]; s[f] = ts;
            const int ti = id[e]; id[e] = id[f]; id[f] = ti;
          }
        }
      }
    }
  }
}

template <int W, int STAGE>
__device__ __forceinline__ void alternating_runs(float (&s)[W >= 32 ? W / 32 : 1], int (&id)[W >= 32 ? W / 32 : 1],
                                                 int lane) {
  if constexpr ((1 << STAGE) < W) {
    merge_pass<W, STAGE, -1>(s, id, lane);
    alternating_runs<W, STAGE + 1>(s, id, lane);
  }
}

template <int W>
constexpr int log2_of() { return W <= 1 ? 0 : 1 + log2_of<W / 2>(); }

// 16 bytes of a row (read-only path), zero when absent.
__device__ __forceinline__ uint4 ld16(const void* p, bool ok) {
  return ok ? __ldg(static_cast<const uint4*>(p)) : make_uint4(0u, 0u, 0u, 0u);
}

// Eight 16-bit values of a query row, scaled in fp32 and rounded back.
template <typename T>
__device__ __forceinline__ uint4 scale_round(uint4 raw, float scale) {
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(to_f32<T>(e[i]) * scale);
  return raw;
}

// Logits of the warp's 16 rows against 8 consecutive blocks j0 .. j0+7:
// c[0], c[1] = rows g, columns 2c, 2c+1; c[2], c[3] = row g+8 (g = lane/4,
// c = lane%4).  Blocks at or past M read as zero.
template <typename T, int KP>
struct Logits16 {
  uint4 q0[KP], q1[KP];

  __device__ void load(const BsaArgs& a, int b, int tok0, int h, int lane) {
    const int g = lane >> 2, c = lane & 3;
    const int r0 = g, r1 = g + 8;
    const int t0 = tok0 + r0 / a.G, t1 = tok0 + r1 / a.G;
    const bool ok0 = r0 < a.TPW * a.G && t0 < a.T, ok1 = r1 < a.TPW * a.G && t1 < a.T;
    const T* base = static_cast<const T*>(a.q) + int64_t(b) * a.q_sb;
    const T* p0 = base + int64_t(ok0 ? t0 : 0) * a.q_st + int64_t(h * a.G + r0 % a.G) * a.q_sh;
    const T* p1 = base + int64_t(ok1 ? t1 : 0) * a.q_st + int64_t(h * a.G + r1 % a.G) * a.q_sh;
#pragma unroll
    for (int p = 0; p < KP; ++p) {
      const int d = 32 * p + 8 * c;
      q0[p] = scale_round<T>(ld16(p0 + d, ok0 && d < a.D), a.scale);
      q1[p] = scale_round<T>(ld16(p1 + d, ok1 && d < a.D), a.scale);
    }
  }

  __device__ __forceinline__ void tile(const BsaArgs& a, const T* xbase, int j0, int lane, float (&acc)[4]) const {
    const int g = lane >> 2, c = lane & 3;
    const int j = j0 + g;
    const bool have = j < a.M;
    const T* xr = xbase + int64_t(have ? j : 0) * (int64_t(a.H) * a.D);
    uint4 xv[KP];
#pragma unroll
    for (int p = 0; p < KP; ++p) {
      const int d = 32 * p + 8 * c;
      xv[p] = ld16(xr + d, have && d < a.D);
    }
    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
#pragma unroll
    for (int p = 0; p < KP; ++p) {
      mma_16816<T>(acc, q0[p].x, q1[p].x, q0[p].y, q1[p].y, xv[p].x, xv[p].y);
      mma_16816<T>(acc, q0[p].z, q1[p].z, q0[p].w, q1[p].w, xv[p].z, xv[p].w);
    }
  }
};

// The same tile by fp32 FMAs (fp32 inputs); the warp's scaled query rows are
// staged in shared memory (qs: 16 rows of D + 4 floats).
struct LogitsF32 {
  float* qs;

  __device__ void load(const BsaArgs& a, int b, int tok0, int h, int lane, float* smem) {
    qs = smem;
    const int ld = a.D + 4;
    for (int r = 0; r < kRows; ++r) {
      const int t = tok0 + r / a.G;
      const bool ok = r < a.TPW * a.G && t < a.T;
      const float* row = static_cast<const float*>(a.q) + int64_t(b) * a.q_sb + int64_t(ok ? t : 0) * a.q_st +
                         int64_t(h * a.G + r % a.G) * a.q_sh;
      for (int d = lane; d < a.D; d += 32) qs[r * ld + d] = ok ? __ldg(row + d) * a.scale : 0.f;
    }
    __syncwarp();
  }

  __device__ __forceinline__ void tile(const BsaArgs& a, const float* xbase, int j0, int lane, float (&acc)[4]) const {
    const int g = lane >> 2, c = lane & 3;
    const int ld = a.D + 4;
    const int ja = j0 + 2 * c, jb = ja + 1;
    const float* xa = xbase + int64_t(ja < a.M ? ja : 0) * (int64_t(a.H) * a.D);
    const float* xb = xbase + int64_t(jb < a.M ? jb : 0) * (int64_t(a.H) * a.D);
    const float* q0 = qs + g * ld;
    const float* q1 = qs + (g + 8) * ld;
    float s00 = 0.f, s01 = 0.f, s10 = 0.f, s11 = 0.f;
    for (int d = 0; d < a.D; d += 4) {
      const float4 u = __ldg(reinterpret_cast<const float4*>(xa + d));
      const float4 v = __ldg(reinterpret_cast<const float4*>(xb + d));
      const float4 p = *reinterpret_cast<const float4*>(q0 + d);
      const float4 r = *reinterpret_cast<const float4*>(q1 + d);
      s00 = fmaf(p.x, u.x, s00); s00 = fmaf(p.y, u.y, s00); s00 = fmaf(p.z, u.z, s00); s00 = fmaf(p.w, u.w, s00);
      s01 = fmaf(p.x, v.x, s01); s01 = fmaf(p.y, v.y, s01); s01 = fmaf(p.z, v.z, s01); s01 = fmaf(p.w, v.w, s01);
      s10 = fmaf(r.x, u.x, s10); s10 = fmaf(r.y, u.y, s10); s10 = fmaf(r.z, u.z, s10); s10 = fmaf(r.w, u.w, s10);
      s11 = fmaf(r.x, v.x, s11); s11 = fmaf(r.y, v.y, s11); s11 = fmaf(r.z, v.z, s11); s11 = fmaf(r.w, v.w, s11);
    }
    acc[0] = ja < a.M ? s00 : 0.f;
    acc[1] = jb < a.M ? s01 : 0.f;
    acc[2] = ja < a.M ? s10 : 0.f;
    acc[3] = jb < a.M ? s11 : 0.f;
  }
};

__device__ __forceinline__ bool required_block(int j, int cur, int force_first, int force_recent) {
  return (force_first && j == 0) || (j <= cur && cur - j < force_recent);
}

// Shared memory of one warp: P [16][W + 8] floats, then the retained lists
// [TPW][W] scores and [TPW][W] ids, then (fp32) the staged query rows.
__host__ __device__ inline int warp_smem_floats(int W, int TPW, int D, bool f32) {
  return kRows * (W + 8) + 2 * TPW * W + (f32 ? kRows * (D + 4) : 0);
}

template <typename T, typename L, int W>
__global__ void __launch_bounds__(kMaxWarps * 32) bsa_select_kernel(const BsaArgs a) {
  constexpr int E = W >= 32 ? W / 32 : 1;
  constexpr int STAGES = log2_of<W>();
  constexpr bool kF32 = std::is_same<T, float>::value;
  extern __shared__ float smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const int bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int tok0 = (blockIdx.x * warps + warp) * a.TPW;
  if (tok0 >= a.T) return;  // warp-uniform; no block-wide barrier follows
  float* P = smem + warp * warp_smem_floats(W, a.TPW, a.D, kF32);
  const int ldp = W + 8;
  float* ret_s = P + kRows * ldp;
  int* ret_id = reinterpret_cast<int*>(ret_s + a.TPW * W);

  // positions of the warp's tokens (lane i < TPW holds token i's)
  const int ntok = min(a.TPW, a.T - tok0);
  int my_pos = 0;
  if (lane < ntok) {
    my_pos = a.positions ? int(a.positions[int64_t(b) * a.T + tok0 + lane])
                         : int(a.pos_offset + tok0 + lane);
  }
  // per lane: rows g and g+8
  const int g = lane >> 2, c = lane & 3;
  int cur[2], comp[2];
  bool rok[2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = g + 8 * rr;
    const int tok = r / a.G;
    rok[rr] = r < a.TPW * a.G && tok < ntok;
    const int pos = __shfl_sync(kFull, my_pos, rok[rr] ? tok : 0);
    cur[rr] = rok[rr] ? pos / a.C : -1;
    comp[rr] = rok[rr] ? (pos + 1) / a.C : 0;
  }
  const int cur_max = __reduce_max_sync(kFull, max(cur[0], cur[1]));
  const int comp_max = __reduce_max_sync(kFull, max(comp[0], comp[1]));

  const T* xbase = static_cast<const T*>(a.means) + int64_t(b) * a.m_sb + int64_t(h) * a.D;
  L lg;
  if constexpr (kF32) {
    lg.load(a, b, tok0, h, lane, ret_s + 2 * a.TPW * W);
  } else {
    lg.load(a, b, tok0, h, lane);
  }

  // pass 1: log-sum-exp of each row's logits over its complete blocks
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  for (int j0 = 0; j0 < comp_max; j0 += 8) {
    float acc[4];
    lg.tile(a, xbase, j0, lane, acc);
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int j = j0 + 2 * c + cc;
        if (j < comp[rr]) {
          const float x = acc[2 * rr + cc];
          const float mn = fmaxf(m[rr], x);
          l[rr] = l[rr] * expf(m[rr] - mn) + expf(x - mn);
          m[rr] = mn;
        }
      }
    }
  }
  float norm[2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      const float mo = __shfl_xor_sync(kFull, m[rr], o);
      const float lo = __shfl_xor_sync(kFull, l[rr], o);
      const float mn = fmaxf(m[rr], mo);
      if (mn == -INFINITY) continue;
      l[rr] = l[rr] * expf(m[rr] - mn) + lo * expf(mo - mn);
      m[rr] = mn;
    }
    norm[rr] = comp[rr] > 0 ? m[rr] + logf(l[rr]) : 0.f;
  }

  // pass 2: probabilities tile by tile, streamed through each token's network
  for (int t0 = 0; t0 <= cur_max; t0 += W) {
    for (int n0 = 0; n0 < W; n0 += 8) {
      const int j0 = t0 + n0;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (j0 < cur_max) lg.tile(a, xbase, j0, lane, acc);   // logits only matter below the current block
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        float p[2];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int j = j0 + 2 * c + cc;
          float v = j < cur[rr] ? expf(acc[2 * rr + cc] - norm[rr]) : 0.f;
          if (rok[rr] && required_block(j, cur[rr], a.force_first, a.force_recent)) v = 1.f;
          p[cc] = v;
        }
        *reinterpret_cast<float2*>(P + (g + 8 * rr) * ldp + n0 + 2 * c) = make_float2(p[0], p[1]);
      }
    }
    __syncwarp();
    for (int tok = 0; tok < ntok; ++tok) {
      const int pos = __shfl_sync(kFull, my_pos, tok);
      const int ct = pos / a.C;
      if (t0 > ct) continue;  // no valid id in this tile for this token
      float s[E];
      int id[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = e * 32 + lane;
        float v = 0.f;
        int jd = -1;
        if (i < W) {
          for (int hh = 0; hh < a.G; ++hh) v += P[(tok * a.G + hh) * ldp + i];
          const int j = t0 + i;
          jd = (j <= ct && j < a.M) ? j : -1;
        }
        s[e] = v;
        id[e] = jd;
      }
      alternating_runs<W, 1>(s, id, lane);
      float* rs = ret_s + tok * W;
      int* ri = ret_id + tok * W;
      if (t0 > 0) {
        merge_pass<W, STAGES, 0>(s, id, lane);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int i = e * 32 + lane;
          if (i < W / 2) { s[e] = rs[i]; id[e] = ri[i]; }
        }
      }
      merge_pass<W, STAGES, 1>(s, id, lane);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = e * 32 + lane;
        if (i < W) { rs[i] = s[e]; ri[i] = id[e]; }
      }
    }
    __syncwarp();
  }

  for (int tok = 0; tok < ntok; ++tok) {
    int64_t* o = a.out + ((int64_t(b) * a.T + tok0 + tok) * a.H + h) * a.K;
    for (int i = lane; i < a.K; i += 32) o[i] = ret_id[tok * W + i];
  }
}

template <typename T, typename L, int W>
int launch_w(const BsaArgs& a, cudaStream_t stream) {
  const bool f32 = std::is_same<T, float>::value;
  const int per_warp = warp_smem_floats(W, a.TPW, a.D, f32) * 4;
  const int warps_needed = (a.T + a.TPW - 1) / a.TPW;
  int warps = std::min(kMaxWarps, warps_needed);
  while (warps > 1 && warps * per_warp > 96 * 1024) --warps;
  const int bytes = warps * per_warp;
  if (bytes > 200 * 1024) return fail(PISA_ERR_UNSUPPORTED, "BSA selection tile does not fit in shared memory");
  auto kern = bsa_select_kernel<T, L, W>;
  if (bytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return fail_cuda(e, "bsa smem attribute");
  }
  const int tok_per_cta = warps * a.TPW;
  dim3 grid(unsigned((a.T + tok_per_cta - 1) / tok_per_cta), unsigned(a.B * a.H));
  TimedLaunch timed(PISA_KERNEL_BSA, stream);
  kern<<<grid, warps * 32, bytes, stream>>>(a);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

template <typename T, typename L>
int launch_l(const BsaArgs& a, int W, cudaStream_t stream) {
  switch (W) {
    case 16: return launch_w<T, L, 16>(a, stream);
    case 32: return launch_w<T, L, 32>(a, stream);
    case 64: return launch_w<T, L, 64>(a, stream);
    case 128: return launch_w<T, L, 128>(a, stream);
    case 256: return launch_w<T, L, 256>(a, stream);
  }
  return fail(PISA_ERR_UNSUPPORTED, "BSA comparison tile must be at most 256 blocks");
}

template <typename T>
int launch_t(const BsaArgs& a, int W, cudaStream_t stream) {
  if constexpr (std::is_same<T, float>::value) {
    return launch_l<T, LogitsF32>(a, W, stream);
  } else {
    const int kp = (a.D + 31) / 32;
    if (kp <= 1) return launch_l<T, Logits16<T, 1>>(a, W, stream);
    if (kp <= 2) return launch_l<T, Logits16<T, 2>>(a, W, stream);
    if (kp <= 4) return launch_l<T, Logits16<T, 4>>(a, W, stream);
    return launch_l<T, Logits16<T, 8>>(a, W, stream);
  }
}

bool aligned_rows(const void* p, int esz, int64_t sb, int64_t st, int64_t sh) {
  const int64_t v = 16 / esz;
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && sb % v == 0 && st % v == 0 && sh % v == 0;
}

int tile_width(int64_t C, int64_t K) {
  const int64_t want = std::max<int64_t>(C, 2 * K);
  int64_t w = 1;
  while (w < want) w <<= 1;
  return w > (1 << 20) ? (1 << 20) : int(w);
}

int64_t means_bytes(int64_t B, int64_t N, int64_t H, int64_t D, int dtype, int64_t C) {
  const int64_t M = (N + C - 1) / C;
  return (B * M * H * D * (dtype == PISA_F32 ? 4 : 2) + 255) / 256 * 256;
}

}  // namespace

}  // namespace pisa

using namespace pisa;

extern "C" {

int64_t pisa_bsa_workspace_bytes(int64_t B, int64_t N, int64_t H, int64_t D, int dtype, int64_t block_size,
                                 int have_means) {
  if (B <= 0 || N <= 0 || H <= 0 || D <= 0 || block_size < 1 || dtype < PISA_F32 || dtype > PISA_F16) return -1;
  return have_means ? 0 : means_bytes(B, N, H, D, dtype, block_size);
}

int pisa_bsa_select(const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh, const void* keys, int64_t key_sb,
                    int64_t key_st, int64_t key_sh, const void* leaf_means, int64_t means_sb,
                    const int64_t* positions, int64_t position_offset, int dtype, int64_t B, int64_t Tq,
                    int64_t Hq, int64_t H, int64_t D, int64_t N, int64_t block_size, int64_t topk,
                    int force_first, int64_t force_recent, int64_t* out_ids, void* workspace,
                    int64_t workspace_bytes, pisa_stream_t stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype < PISA_F32 || dtype > PISA_F16) return fail(PISA_ERR_UNSUPPORTED, "BSA routing supports FP16, BF16 and FP32");
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || D <= 0 || N <= 0) return fail(PISA_ERR_INVALID, "nonempty tensors are required");
  if (Hq % H) return fail(PISA_ERR_INVALID, "a whole number of query heads per KV head is required");
  if (block_size < 1 || topk < 1 || force_recent < 0)
    return fail(PISA_ERR_INVALID, "positive block_size/topk and nonnegative force_recent required");
  const int64_t G = Hq / H;
  if (G > kRows) return fail(PISA_ERR_UNSUPPORTED, "BSA routing supports at most 16 query heads per KV head");
  const int esz = dtype == PISA_F32 ? 4 : 2;
  if (D % (16 / esz) || D > 256) return fail(PISA_ERR_UNSUPPORTED, "head_dim must fill whole 16-byte vectors and be at most 256");
  const int W = tile_width(block_size, topk);
  if (W > 256) return fail(PISA_ERR_UNSUPPORTED, "BSA comparison tile max(block_size, 2*topk) must be at most 256");
  const int64_t M = (N + block_size - 1) / block_size;
  if (Tq > INT32_MAX / 2 || N > INT32_MAX / 2 || B * H > 65535)
    return fail(PISA_ERR_UNSUPPORTED, "sequence or batch too large for the BSA launch");
  if (!positions) {
    if (position_offset < 0 || position_offset + Tq > N)
      return fail(PISA_ERR_INVALID, "queries must refer to positions within their key sequence");
    // most required blocks over the rows (bsa_torch.py:94-95): the last row has the most
    const int64_t cur = (position_offset + Tq - 1) / block_size;
    const int64_t need = std::min<int64_t>(force_recent, cur + 1) + ((force_first && cur >= force_recent) ? 1 : 0);
    if (need > topk) return fail(PISA_ERR_INVALID, "topk is smaller than the number of required distinct blocks");
  }
  if (!out_ids) return fail(PISA_ERR_INVALID, "out_ids is required");
  if (!aligned_rows(q, esz, q_sb, q_st, q_sh) || !aligned_rows(keys, esz, key_sb, key_st, key_sh))
    return fail(PISA_ERR_UNSUPPORTED, "q and key rows must be 16-byte aligned");

  const void* means = leaf_means;
  int64_t m_sb = means_sb;
  if (means) {
    if (!aligned_rows(means, esz, means_sb, H * D, D)) return fail(PISA_ERR_UNSUPPORTED, "leaf mean rows must be 16-byte aligned");
  } else {
    const int64_t need = means_bytes(B, N, H, D, dtype, block_size);
    if (!workspace || workspace_bytes < need) return fail(PISA_ERR_INVALID, "workspace too small");
    const int64_t off = 0;
    int rc = build_pyramid(keys, dtype, B, N, H, D, key_sb, key_st, key_sh, block_size, 2, 1, workspace, M * H * D,
                           &off, 0, s);
    if (rc) return rc;
    means = workspace;
    m_sb = M * H * D;
  }

  BsaArgs a{};
  a.q = q; a.q_sb = q_sb; a.q_st = q_st; a.q_sh = q_sh;
  a.means = means; a.m_sb = m_sb;
  a.positions = positions; a.pos_offset = position_offset;
  a.B = int(B); a.T = int(Tq); a.H = int(H); a.G = int(G); a.D = int(D); a.M = int(M);
  a.C = int(block_size); a.K = int(topk);
  a.TPW = int(kRows / G);
  a.force_first = force_first ? 1 : 0;
  a.force_recent = int(std::min<int64_t>(force_recent, INT32_MAX));
  a.scale = float(1.0 / std::sqrt(double(D)));
  a.out = out_ids;
  switch (dtype) {
    case PISA_F32: return launch_t<float>(a, W, s);
    case PISA_BF16: return launch_t<__nv_bfloat16>(a, W, s);
    case PISA_F16: return launch_t<__half>(a, W, s);
  }
  return fail(PISA_ERR_UNSUPPORTED, "unsupported dtype");
}

}  // extern "C"
