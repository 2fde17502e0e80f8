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

constexpr int kThreads = 128;
// children per MMA chunk: 64 TMEM columns and 8 KB of summaries per 64-dim
// chunk keep four CTAs resident per SM at D = 128, so some CTAs load while
// others run their epilogue, and the causal cut-off skips work in steps of 64
constexpr int kChunk = 64;

template <typename T, int SUP>
__global__ void __launch_bounds__(kThreads) dense_level_kernel(const __grid_constant__ DenseArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int qch = a.Dp / 64;
  uint8_t* Qs = smem;                      // [qch][128 rows][128 B]
  uint8_t* Xs = smem + qch * 128 * 128;    // [qch][kChunk children][128 B]
  __shared__ uint64_t mbar, ld_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ unsigned long long s_maxpos;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tt = 128 / a.G;                // tokens per tile
  const int t0 = a.t_begin + blockIdx.x * tt;
  const int t_end = a.t_begin + a.t_count;
  const int h = blockIdx.y, b = blockIdx.z;
  const int lgG = 31 - __clz(a.G);
  const int row = tid, r = row >> lgG, g = row & (a.G - 1);
  const int t = t0 + r;
  const bool live = t < t_end;
  const int64_t pos = live ? (a.positions ? a.positions[int64_t(b) * a.T + t] : a.pos_offset + t) : 0;

  if (tid == 0) {
    tc::mbar_init(&mbar, 1);
    tc::mbar_init(&ld_bar, 1);
    s_maxpos = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, kChunk);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (live) atomicMax(&s_maxpos, static_cast<unsigned long long>(pos));
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_base = (uint32_t(warp) * 32) << 16;
  const uint32_t qs_addr = tc::smem_u32(Qs), xs_addr = tc::smem_u32(Xs);

  // the tile's query rows (token t0 + r, head h*G + g) arrive by TMA together
  // with the first child chunk: one box of G heads x 128/G tokens per
  // 64-dim chunk (dims past D and tokens past the sequence read as zero)
  const uint32_t q_bytes = uint32_t(qch) * 128 * 128;
  if (tid == 0)
    for (int ch = 0; ch < qch; ++ch)
      tc::tma_load_4d(qs_addr + ch * 128 * 128, &a.tm_q, ch * 64, h * a.G, t0, b, &ld_bar);
  __syncthreads();
  const int64_t maxpos = int64_t(s_maxpos);
  uint32_t phase = 0, ld_phase = 0;
  bool ok = true;
  float* out = a.scores + ((int64_t(b) * a.t_count + (live ? t - a.t_begin : 0)) * a.H + h) * a.row_stride + a.out_off;
  const float l2e = 1.4426950408889634f;

  for (int c0 = 0; c0 < a.n_child; c0 += kChunk) {
    // every later node is past every position (never at c0 = 0: node 0 starts
    // at token 0, so the query load issued above is always awaited here)
    if (int64_t(c0 / SUP) * a.span > maxpos) break;
    const int nc = min(kChunk, a.n_child - c0);
    const int ncp = (nc + 15) / 16 * 16;
    // kChunk child summaries per 64-dim chunk by TMA (rows past the storage
    // read as zero; rows past the level are ignored by the epilogue)
    if (tid == 0) {
      tc::mbar_arrive_expect_tx(&ld_bar, uint32_t(qch) * kChunk * 128 + (c0 == 0 ? q_bytes : 0u));
      for (int ch = 0; ch < qch; ++ch)
        tc::tma_load_4d(xs_addr + ch * kChunk * 128, &a.tm_x, ch * 64, h, int(a.child_off) + c0, b, &ld_bar);
    }
    if (!tc::mbar_wait(&ld_bar, ld_phase)) ok = false;
    ld_phase ^= 1;
    tc::fence_after_sync();
    if (tid == 0) {
      const uint32_t idesc = tc::idesc_f16(128, ncp, a.bf16);
      for (int ks = 0; ks < a.Dp / 16; ++ks) {
        const int ch = ks >> 2, off = (ks & 3) * 32;
        tc::mma_f16(tmem, tc::desc_sw128(qs_addr + ch * 128 * 128 + off),
                    tc::desc_sw128(xs_addr + ch * kChunk * 128 + off), idesc, ks > 0);
      }
      tc::mma_commit(&mbar);
    }
    if (!tc::mbar_wait(&mbar, phase)) ok = false;
    phase ^= 1;
    tc::fence_after_sync();

    // nodes of this chunk: children [c0, c0 + nc) in groups of SUP columns
    for (int cc = 0; cc < nc; cc += 32) {
      float v[32];
      tc::tmem_ld32(tmem + lane_base + cc, v);
#pragma unroll
      for (int j = 0; j < 32; j += SUP) {
        if (cc + j >= nc) break;                       // uniform across the warp
        const int child0 = c0 + cc + j;
        const int cnt = min(SUP, a.n_child - child0);
        float score;
        if (a.method == PISA_METHOD_PISA1) {
          score = v[j];
        } else if (a.method == PISA_METHOD_PISA) {
          float m = v[j];
#pragma unroll
          for (int i = 1; i < SUP; ++i) if (i < cnt) m = fmaxf(m, v[j + i]);
          const float mz = m * a.scale;
          float sum = 0.f;
#pragma unroll
          for (int i = 0; i < SUP; ++i) if (i < cnt) sum += exp2f((v[j + i] * a.scale - mz) * l2e);
          score = mz + logf(sum);
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
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }
  if (!ok && lane == 0) atomicExch(a.status, PISA_ERR_TIMEOUT);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_free(tmem, kChunk);
}

}  // namespace

int dense_level(const DenseArgs& a, int dtype, cudaStream_t stream) {
  const int qch = a.Dp / 64;
  // query rows + one chunk of child summaries (49 KB at D = 128: four CTAs
  // per SM; TMEM, kChunk columns each, allows eight)
  const size_t smem = size_t(qch) * 128 * (128 + kChunk) + 1024;
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
