// K2a: dense tensor-core scoring of whole coarse pyramid levels.
//
// At a coarse level l >= 1 a candidate node's score depends only on the query
// and the node's b children at level l-1 (block_scores, top_k_pyramid_torch.py:
// 48-80: LSE over the children for pisa, the binary 1/2-sum + 1/8-difference^2
// or mean + variance form for pisa2).  Which nodes a row ends up scoring
// depends on its descent, but the score of a node does not -- so every node of
// the level is scored for every row up front, as a GEMM: a tile of 128/G
// consecutive tokens x G query heads of one KV head (128 rows) against the
// level's child summaries, kChunk children per tcgen05 MMA (N=kChunk, K=head_dim),
// accumulators in TMEM.  The epilogue (thread = row) reduces each node's b
// child columns to its score, sums the G heads with shuffles and writes
// scores[b, t, h, node].  The router then reads scores instead of computing
// dot products.  Node chunks entirely past the tile's last position are
// skipped (causally invalid).  pisa1 scores nodes against themselves
// (support 1, scale 1): same kernel with children = the level's own nodes.
#include <algorithm>

#include "bucket.cuh"
#include "internal.h"
#include "tc.cuh"

namespace pisa {

namespace {

// two warps per TMEM lane quarter: warp w reads lanes 32*(w%4).. and the
// column half w/4 of every chunk, so eight warps share each chunk's epilogue
constexpr int kThreads = 256;
// children per MMA chunk: 64 TMEM columns and 8 KB of summaries per 64-dim
// chunk keep four CTAs resident per SM at D = 128, so some CTAs load while
// others run their epilogue, and the causal cut-off skips work in steps of 64
constexpr int kChunk = 64;
// child chunk buffers: the TMA runs kStages - 1 chunks ahead of the MMA.
// Two buffers (65 KB of shared memory at D = 128) keep three CTAs of eight
// warps per SM; four buffers (two CTAs) measured slower (31 ms against 23 ms
// for the dense levels of a 256K prefill): more resident CTAs beat a deeper
// prefetch here
constexpr int kStages = 2;

// MUFU base-2 logarithm (lg2.approx: relative error about 2^-22)
__device__ __forceinline__ float lg2_approx(float x) {
  float r;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// LSE of a node whose SUP (2 or 4) children all exist, base 2 as in the
// general path (y = v * scale * log2 e): the largest child contributes
// 2^0 = 1 exactly, so only the others take an exponential; a min/max network
// splits the values into the maximum and the rest.
template <int SUP>
__device__ __forceinline__ float lse_full_node(const float (&v)[32], int j, float k2) {
  const float ln2 = 0.6931471805599453f;
  if constexpr (SUP == 4) {
    const float h0 = fmaxf(v[j], v[j + 1]), l0 = fminf(v[j], v[j + 1]);
    const float h1 = fmaxf(v[j + 2], v[j + 3]), l1 = fminf(v[j + 2], v[j + 3]);
    const float m = fmaxf(h0, h1), o = fminf(h0, h1);
    const float my = m * k2;
    const float sum = 1.f + tc::ex2f(fmaf(l0, k2, -my)) + tc::ex2f(fmaf(l1, k2, -my)) + tc::ex2f(fmaf(o, k2, -my));
    return ln2 * (my + lg2_approx(sum));
  } else if constexpr (SUP == 2) {
    const float m = fmaxf(v[j], v[j + 1]), o = fminf(v[j], v[j + 1]);
    const float my = m * k2;
    return ln2 * (my + lg2_approx(1.f + tc::ex2f(fmaf(o, k2, -my))));
  } else {
    return v[j] * k2 * ln2;
  }
}

// Sums each node score of one 32-column half over the G = 2^LG query-head
// lanes of its token and stores it from one lane: a reduce-scatter by
// shuffles (lane bit k keeps the upper or lower half of the remaining nodes
// at stage k), so every head lane ends with NPT / G finished scores.  The
// additions associate as the shuffle butterfly ((h0+h1)+(h2+h3))+... .
template <int NPT, int LG>
__device__ __forceinline__ void head_sum_store(float (&s)[NPT], int g, float* dst, bool live) {
  int base = 0;
#pragma unroll
  for (int k = 0; k < LG; ++k) {
    const int half = NPT >> (k + 1);
    const bool hi = (g >> k) & 1;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float mine = hi ? s[half + i] : s[i];
      const float other = hi ? s[i] : s[half + i];
      s[i] = mine + __shfl_xor_sync(kFull, other, 1 << k);
    }
    base += hi ? half : 0;
  }
  if (live) {
#pragma unroll
    for (int i = 0; i < (NPT >> LG); ++i) dst[base + i] = s[i];
  }
}

// Per CTA: the tile's query rows stay in shared memory while the level's
// child chunks stream through a ring of kStages buffers: the TMA runs
// kStages - 1 chunks ahead and the MMA of chunk c+1 (into the other of two
// TMEM accumulators) runs while the warps reduce chunk c's columns to node
// scores.
template <typename T, int SUP>
__global__ void __launch_bounds__(kThreads) dense_level_kernel(const __grid_constant__ DenseArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int qch = a.Dp / 64;
  const int xbytes = qch * kChunk * 128;   // one child chunk: [qch][kChunk children][128 B]
  uint8_t* Qs = smem;                      // [qch][128 rows][128 B]
  uint8_t* Xs = smem + qch * 128 * 128;    // kStages child chunk buffers
  __shared__ uint64_t mma_bar[2], ld_bar[kStages];
  __shared__ uint32_t tmem_slot;
  __shared__ unsigned long long s_maxpos;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tt = 128 / a.G;                // tokens per tile
  const int t0 = a.t_begin + blockIdx.x * tt;
  const int t_end = a.t_begin + a.t_count;
  const int h = blockIdx.y, b = blockIdx.z;
  const int lgG = 31 - __clz(a.G);
  const int row = tid & 127, half = tid >> 7, r = row >> lgG, g = row & (a.G - 1);
  const int t = t0 + r;
  const bool live = t < t_end;
  const int64_t pos = live ? (a.positions ? a.positions[int64_t(b) * a.T + t] : a.pos_offset + t) : 0;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) tc::mbar_init(&mma_bar[i], 1);
    for (int i = 0; i < kStages; ++i) tc::mbar_init(&ld_bar[i], 1);
    s_maxpos = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, 2 * kChunk);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (live && half == 0) atomicMax(&s_maxpos, static_cast<unsigned long long>(pos));
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_base = (uint32_t(warp & 3) * 32) << 16;
  const uint32_t qs_addr = tc::smem_u32(Qs), xs_addr = tc::smem_u32(Xs);
  __syncthreads();
  // chunks up to the last one holding a node at or before the tile's last
  // position (later nodes are causally invalid for every row of the tile;
  // node 0 starts at token 0, so there is always at least one chunk)
  const int64_t maxpos = int64_t(s_maxpos);
  int nchunks = 0;
  for (int c0 = 0; c0 < a.n_child; c0 += kChunk) {
    if (int64_t(c0 / SUP) * a.span > maxpos) break;
    ++nchunks;
  }

  // chunk c of kChunk child summaries by TMA into buffer c % kStages (rows past the
  // storage read as zero; rows past the level are ignored by the epilogue);
  // the query rows (one box of G heads x 128/G tokens per 64-dim chunk) come
  // with chunk 0
  const uint32_t q_bytes = uint32_t(qch) * 128 * 128;
  auto load_chunk = [&](int c) {
    const int bi = c % kStages;
    tc::mbar_arrive_expect_tx(&ld_bar[bi], uint32_t(xbytes) + (c == 0 ? q_bytes : 0u));
    if (c == 0)
      for (int ch = 0; ch < qch; ++ch)
        tc::tma_load_4d(qs_addr + ch * 128 * 128, &a.tm_q, ch * 64, h * a.G, t0, b, &ld_bar[0]);
    for (int ch = 0; ch < qch; ++ch)
      tc::tma_load_4d(xs_addr + bi * xbytes + ch * kChunk * 128, &a.tm_x, ch * 64, h,
                      int(a.child_off) + c * kChunk, b, &ld_bar[bi]);
  };
  auto issue_mma = [&](int c) {
    const int ai = c & 1, bi = c % kStages;
    const int nc = min(kChunk, a.n_child - c * kChunk);
    const uint32_t idesc = tc::idesc_f16(128, (nc + 15) / 16 * 16, a.bf16);
    for (int ks = 0; ks < a.Dp / 16; ++ks) {
      const int ch = ks >> 2, off = (ks & 3) * 32;
      tc::mma_f16(tmem + ai * kChunk, tc::desc_sw128(qs_addr + ch * 128 * 128 + off),
                  tc::desc_sw128(xs_addr + bi * xbytes + ch * kChunk * 128 + off), idesc, ks > 0);
    }
    tc::mma_commit(&mma_bar[ai]);
  };
  bool ok = true;
  uint32_t ld_phase = 0u, mma_phase = 0u;   // bit i: parity of barrier i's next wait
  if (tid == 0)
    for (int c = 0; c < kStages && c < nchunks; ++c) load_chunk(c);
  if (!tc::mbar_wait(&ld_bar[0], ld_phase & 1u)) ok = false;
  ld_phase ^= 1u;
  tc::fence_after_sync();
  if (tid == 0) issue_mma(0);

  float* out = a.scores + ((int64_t(b) * a.t_count + (live ? t - a.t_begin : 0)) * a.H + h) * a.row_stride + a.out_off;
  const float k2 = a.scale * 1.4426950408889634f;   // scale * log2 e
  const float ln2 = 0.6931471805599453f;

  for (int c = 0; c < nchunks; ++c) {
    const int bi = c & 1;   // accumulator of chunk c
    // next chunk's MMA (its data landed; its accumulator was read out by the
    // previous iteration's epilogue, closed by the barrier below)
    if (c + 1 < nchunks) {
      const int sn = (c + 1) % kStages;
      if (!tc::mbar_wait(&ld_bar[sn], (ld_phase >> sn) & 1u)) ok = false;
      ld_phase ^= 1u << sn;
      tc::fence_after_sync();
      if (tid == 0) issue_mma(c + 1);
    }
    // this chunk's MMA done: its summary buffer takes chunk c + kStages
    if (!tc::mbar_wait(&mma_bar[bi], (mma_phase >> bi) & 1u)) ok = false;
    mma_phase ^= 1u << bi;
    tc::fence_after_sync();
    if (tid == 0 && c + kStages < nchunks) load_chunk(c + kStages);

    // nodes of this chunk: children [c0, c0 + nc) in groups of SUP columns
    const int c0 = c * kChunk;
    const int nc = min(kChunk, a.n_child - c0);
    for (int cc = 32 * half; cc < nc; cc += 64) {
      float v[32];
      tc::tmem_ld32(tmem + lane_base + bi * kChunk + cc, v);
      if constexpr (SUP >= 2) {
        // a complete half of LSE nodes with G in {2, 4, 8}: scores of every
        // node, then one reduce-scatter over the head lanes
        if (a.method == PISA_METHOD_PISA && cc + 32 <= nc && a.G >= 2 && a.G <= 8) {
          constexpr int NPT = 32 / SUP;
          float sc[NPT];
#pragma unroll
          for (int n = 0; n < NPT; ++n) sc[n] = lse_full_node<SUP>(v, n * SUP, k2);
          float* dst = out + (c0 + cc) / SUP;
          if (a.G == 2) head_sum_store<NPT, 1>(sc, g, dst, live);
          else if (a.G == 4) head_sum_store<NPT, 2>(sc, g, dst, live);
          else head_sum_store<NPT, 3>(sc, g, dst, live);
          continue;
        }
      }
#pragma unroll
      for (int j = 0; j < 32; j += SUP) {
        if (cc + j >= nc) break;                       // uniform across the warp
        const int child0 = c0 + cc + j;
        const int cnt = min(SUP, a.n_child - child0);
        float score;
        if (a.method == PISA_METHOD_PISA1) {
          score = v[j];
        } else if (a.method == PISA_METHOD_PISA && cnt == SUP && SUP >= 2) {
          score = lse_full_node<SUP>(v, j, k2);
        } else if (a.method == PISA_METHOD_PISA) {
          // base 2: LSE = ln2 * (max y + log2 sum 2^(y - max y)), y = v * scale * log2 e
          float m = v[j];
#pragma unroll
          for (int i = 1; i < SUP; ++i) if (i < cnt) m = fmaxf(m, v[j + i]);
          const float my = m * k2;
          float sum = 0.f;
#pragma unroll
          for (int i = 0; i < SUP; ++i) if (i < cnt) sum += tc::ex2f(fmaf(v[j + i], k2, -my));
          score = ln2 * (my + lg2_approx(sum));
        } else if (SUP == 2) {
          const float z0 = v[j] * a.scale, z1 = cnt == 2 ? v[j + 1] * a.scale : 0.f;
          const float total = z0 + z1, diff = z0 - z1;
          score = cnt == 2 ? 0.5f * total + 0.125f * diff * diff : total;
        } else {
          float s1 = 0.f, s2 = 0.f;
#pragma unroll
          for (int i = 0; i < SUP; ++i) if (i < cnt) { s1 += v[j + i]; s2 = fmaf(v[j + i], v[j + i], s2); }
          const float mean = s1 / cnt, var = fmaxf(s2 / cnt - mean * mean, 0.f);
          score = a.scale * mean + a.c2 * var;
        }
        for (int o = 1; o < a.G; o <<= 1) score += __shfl_xor_sync(kFull, score, o);
        if (live && g == 0) out[child0 / SUP] = score;
      }
    }
    // every thread's TMEM loads of accumulator bi are done before the MMA of
    // chunk c + 2 overwrites it
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }
  if (!ok && lane == 0) atomicExch(a.status, PISA_ERR_TIMEOUT);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_free(tmem, 2 * kChunk);
}

}  // namespace

int dense_level(const DenseArgs& a, int dtype, cudaStream_t stream) {
  const int qch = a.Dp / 64;
  // query rows + kStages chunks of child summaries
  const size_t smem = size_t(qch) * 128 * (128 + kStages * kChunk) + 1024;
  void (*kernel)(const DenseArgs);
  if (a.support == 1) kernel = dtype == PISA_BF16 ? dense_level_kernel<__nv_bfloat16, 1> : dense_level_kernel<__half, 1>;
  else if (a.support == 2) kernel = dtype == PISA_BF16 ? dense_level_kernel<__nv_bfloat16, 2> : dense_level_kernel<__half, 2>;
  else kernel = dtype == PISA_BF16 ? dense_level_kernel<__nv_bfloat16, 4> : dense_level_kernel<__half, 4>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return fail_cuda(e, "dense level smem attribute");
  const int tt = 128 / a.G;
  dim3 grid(unsigned((a.t_count + tt - 1) / tt), unsigned(a.H), unsigned(a.B));
  TimedLaunch timed(PISA_KERNEL_DENSE_LEVEL, stream);
  kernel<<<grid, kThreads, smem, stream>>>(a);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

}  // namespace pisa
