// Standalone leaf scoring of arbitrary candidate lists: grouped_leaf_scores
// (pisa/pisa/ops/flash_sparse_attn/top_k_pyramid/leaf_triton.py:144-232).
//
// Output: fp32 scores [B, Tq, Hkv, W] in candidate order.  A slot whose id is
// outside [0, blocks) gets -inf.  With query positions the reference's level-0
// masks apply as well (leaf_scoreable_mask, leaf_triton.py:23-60, with
// score_masks / required of top_k_pyramid_triton.py:14-24,105-122): ids past
// the query's causal edge, forced ids (first block, the force_recent most
// recent blocks) and, for pisa/pisa2, every id of a row whose valid ids all
// fit in top-K get -inf; the rest are scored.
//
// leaf_prepare_kernel writes the masks, int32 ids and the -inf fills; the
// scored slots then go through the grouped tensor-core pipeline (leaf.cu, one
// family per candidate block) or, for fp32 / pisa1 / shapes outside the
// tensor-core envelope, through leaf_scores_simt_kernel below.
#include "internal.h"
#include "score.cuh"

namespace pisa {

namespace {

__device__ __forceinline__ int64_t cand_at(const void* p, int bytes, int64_t i) {
  return bytes == 4 ? int64_t(static_cast<const int32_t*>(p)[i]) : static_cast<const int64_t*>(p)[i];
}

// One warp per (batch, token, KV head) row.
__global__ void __launch_bounds__(128) leaf_prepare_kernel(const LeafPrepArgs p) {
  const int64_t row = int64_t(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= int64_t(p.B) * p.T * p.H) return;
  const int64_t bt = row / p.H;                    // b * T + t
  const int64_t pos = p.positions ? p.positions[bt] : 0;
  const int64_t leaf = pos / p.C;
  const int64_t base = row * p.W;
  auto valid_of = [&](int64_t id) {
    return id >= 0 && id < p.blocks && (!p.positions || id * p.C <= pos);
  };
  // identity shortcut (pisa / pisa2 with masks): nothing is scored when every
  // valid id fits in top-K
  bool shortcut = false;
  if (p.positions && p.method != PISA_METHOD_PISA1) {
    int cnt = 0;
    for (int w0 = 0; w0 < p.W; w0 += 32) {
      const int w = w0 + lane;
      cnt += __popc(__ballot_sync(kFull, w < p.W && valid_of(cand_at(p.cand, p.cand_bytes, base + w))));
    }
    shortcut = cnt <= p.K;
  }
  for (int w = lane; w < p.W; w += 32) {
    const int64_t id = cand_at(p.cand, p.cand_bytes, base + w);
    const bool valid = valid_of(id);
    bool forced = false;
    if (valid && p.positions) {
      if (p.force_first && id == 0) forced = true;
      for (int r = 0; r < p.force_recent; ++r)
        if (leaf - r >= 0 && id == leaf - r) forced = true;
    }
    const bool scoreable = valid && !forced && !shortcut;
    p.cand_out[base + w] = valid ? int32_t(id) : -1;
    p.flags[base + w] = uint8_t((valid ? 1 : 0) | (forced ? 2 : 0) | (scoreable ? 4 : 0));
    if (!scoreable) p.scores[base + w] = -INFINITY;
  }
}

// One CTA per row: the row's G query rows staged in fp32, one warp per
// scoreable slot (lanes over the block's keys), or the first-order score
// q . leaf mean for pisa1.
template <typename T, int GMAX>
__global__ void __launch_bounds__(128) leaf_scores_simt_kernel(const RouteArgs a, const int32_t* cand,
                                                               const uint8_t* flags, int W, float* scores,
                                                               const void* means, int64_t means_sb) {
  extern __shared__ __align__(16) float qs[];   // [G][D]
  const int64_t row = blockIdx.x;               // (b * T + t) * H + h
  const int h = int(row % a.H);
  const int64_t bt = row / a.H;
  const int t = int(bt % a.T), b = int(bt / a.T);
  const T* qp = static_cast<const T*>(a.q) + b * a.q_sb + t * a.q_st + int64_t(h) * a.G * a.q_sh;
  for (int e = threadIdx.x; e < a.G * a.D; e += blockDim.x) {
    const int g = e / a.D, d = e % a.D;
    qs[e] = to_f32<T>(qp[g * a.q_sh + d]);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* key_base = static_cast<const T*>(a.keys) + b * a.k_sb + int64_t(h) * a.k_sh;
  const T* mean_base = static_cast<const T*>(means) + b * means_sb + int64_t(h) * a.D;
  for (int w = warp; w < W; w += blockDim.x / 32) {
    if (!(flags[row * W + w] & 4)) continue;
    const int id = cand[row * W + w];
    float v;
    if (a.method == PISA_METHOD_PISA1) {
      v = coarse_score<T, GMAX>(a, mean_base, a.levels.size[0], id, qs);
    } else {
      v = leaf_score_warp<T, GMAX>(a, key_base, id, qs, lane);
    }
    if (lane == 0) scores[row * W + w] = v;
  }
}

template <typename T, int GMAX>
int launch_simt(const RouteArgs& a, const int32_t* cand, const uint8_t* flags, int W, float* scores,
                const void* means, int64_t means_sb, cudaStream_t stream) {
  const size_t smem = size_t(a.G) * a.D * sizeof(float);
  auto kernel = leaf_scores_simt_kernel<T, GMAX>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return fail_cuda(e, "leaf score smem attribute");
  }
  const int64_t rows = int64_t(a.B) * a.T * a.H;
  kernel<<<unsigned(rows), 128, smem, stream>>>(a, cand, flags, W, scores, means, means_sb);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

template <typename T>
int simt_t(const RouteArgs& a, const int32_t* cand, const uint8_t* flags, int W, float* scores,
           const void* means, int64_t means_sb, cudaStream_t stream) {
  if (a.G <= 1) return launch_simt<T, 1>(a, cand, flags, W, scores, means, means_sb, stream);
  if (a.G <= 2) return launch_simt<T, 2>(a, cand, flags, W, scores, means, means_sb, stream);
  if (a.G <= 4) return launch_simt<T, 4>(a, cand, flags, W, scores, means, means_sb, stream);
  if (a.G <= 8) return launch_simt<T, 8>(a, cand, flags, W, scores, means, means_sb, stream);
  if (a.G <= 16) return launch_simt<T, 16>(a, cand, flags, W, scores, means, means_sb, stream);
  return launch_simt<T, 32>(a, cand, flags, W, scores, means, means_sb, stream);
}

}  // namespace

int leaf_prepare(const LeafPrepArgs& p, cudaStream_t stream) {
  const int64_t rows = int64_t(p.B) * p.T * p.H;
  if (rows == 0) return PISA_OK;
  leaf_prepare_kernel<<<unsigned((rows + 3) / 4), 128, 0, stream>>>(p);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

int leaf_scores_simt(const RouteArgs& a, const int32_t* cand, const uint8_t* flags, int W, float* scores,
                     const void* means, int64_t means_sb, int dtype, cudaStream_t stream) {
  if (int64_t(a.B) * a.T * a.H == 0) return PISA_OK;
  switch (dtype) {
    case PISA_F32: return simt_t<float>(a, cand, flags, W, scores, means, means_sb, stream);
    case PISA_BF16: return simt_t<__nv_bfloat16>(a, cand, flags, W, scores, means, means_sb, stream);
    case PISA_F16: return simt_t<__half>(a, cand, flags, W, scores, means, means_sb, stream);
  }
  return fail(PISA_ERR_UNSUPPORTED, "unsupported dtype");
}

}  // namespace pisa
