// K5: fused single-token decode step -- selection and attention in one launch.
//
// The reference decodes in two steps: select_blocks with the "fused" routing
// schedule (one Triton program per (token, KV head) scoring every level,
// leaf included, top_k_pyramid_triton.py:125-276 with FUSE_LEAF), then
// decode_attention over the selected blocks (decode/decode_triton.py:8-79).
// Here one CTA per (sequence, token, KV head) does both: the per-item router
// (router.cu route_kernel: coarse levels from the caller's pyramid, leaf
// scores over the C raw keys, the comparison-network top-K) keeps the final
// ids in shared memory and attends over them straight away (router.cu
// decode_attend), so a decode step is one launch and the ids never make a
// round trip through memory before the attention reads the blocks.  The ids
// are also written to out_ids, as select_blocks returns them.
#include <algorithm>
#include <cmath>

#include "internal.h"

namespace pisa {
namespace {

bool is_pow2_i(int64_t x) { return x > 0 && (x & (x - 1)) == 0; }

bool aligned_rows(const void* p, int dtype, int64_t sb, int64_t st, int64_t sh) {
  const int64_t v = dtype == PISA_F32 ? 4 : 8;   // elements per 16 bytes
  return p != nullptr && reinterpret_cast<uintptr_t>(p) % 16 == 0 && sb % v == 0 && st % v == 0 && sh % v == 0;
}

}  // namespace
}  // namespace pisa

using namespace pisa;

extern "C" int pisa_decode_select_attend(
    const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh, const void* keys, int64_t key_sb, int64_t key_st,
    int64_t key_sh, const void* values, int64_t value_sb, int64_t value_st, int64_t value_sh,
    const void* summary, int64_t summary_sb, const int64_t* level_offsets, const int64_t* level_sizes,
    int64_t num_levels, const int64_t* positions, int64_t position_offset, int dtype, int64_t B, int64_t Tq,
    int64_t Hq, int64_t H, int64_t D, int64_t Dv, int64_t N, int method, int64_t block_size,
    int64_t branching, int64_t topk, int force_first, int64_t force_recent, int64_t top,
    int64_t first_width, float scale, int64_t* out_ids, void* out, float* lse, pisa_stream_t stream) {
  if (dtype < PISA_F32 || dtype > PISA_F16) return fail(PISA_ERR_UNSUPPORTED, "GPU routing supports FP16, BF16 and FP32");
  if (method < PISA_METHOD_PISA1 || method > PISA_METHOD_PISA) return fail(PISA_ERR_INVALID, "method must be pisa1, pisa2 or pisa");
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || D <= 0 || Dv <= 0 || N <= 0)
    return fail(PISA_ERR_INVALID, "nonempty tensors are required");
  if (Hq % H) return fail(PISA_ERR_INVALID, "a whole number of query heads per KV head is required");
  const int64_t G = Hq / H;
  if (G > 32) return fail(PISA_ERR_UNSUPPORTED, "at most 32 query heads per KV head");
  if (D % 8 || D > 256) return fail(PISA_ERR_UNSUPPORTED, "head_dim must be a multiple of 8 and at most 256");
  if (Dv != 64 && Dv != 128 && Dv != 256) return fail(PISA_ERR_UNSUPPORTED, "fused decode needs a value head_dim of 64, 128 or 256");
  if (G > 16 || G * Dv > 2048) return fail(PISA_ERR_UNSUPPORTED, "fused decode needs G <= 16 and G * value head_dim <= 2048");
  if (!is_pow2_i(topk) || topk < 8 || topk > 64 || !is_pow2_i(block_size) || block_size < 16)
    return fail(PISA_ERR_UNSUPPORTED, "GPU routing requires power-of-two block_size >= 16 and topk in {8,16,32,64}");
  if (branching != 2 && branching != 4) return fail(PISA_ERR_UNSUPPORTED, "branching must be 2 or 4");
  if (force_recent < 1) return fail(PISA_ERR_INVALID, "causal pyramid routing requires force_recent >= 1");
  const int64_t blocks = (N + block_size - 1) / block_size;
  if (topk < std::min<int64_t>(blocks, force_recent + (force_first ? 1 : 0)))
    return fail(PISA_ERR_INVALID, "topk cannot hold all required blocks");
  if (top < 0 || top >= kMaxLevels) return fail(PISA_ERR_INVALID, "routing depth out of range");
  if (!is_pow2_i(first_width) || first_width < 16 || first_width > 256)
    return fail(PISA_ERR_UNSUPPORTED, "first network width must be a power of two in [16, 256]");
  if (topk * branching > 256) return fail(PISA_ERR_UNSUPPORTED, "topk * branching must be at most 256");
  if (!out_ids || !out) return fail(PISA_ERR_INVALID, "out_ids and out are required");
  if (!aligned_rows(q, dtype, q_sb, q_st, q_sh) || !aligned_rows(keys, dtype, key_sb, key_st, key_sh) ||
      !aligned_rows(values, dtype, value_sb, value_st, value_sh))
    return fail(PISA_ERR_UNSUPPORTED, "q, key and value rows must be 16-byte aligned");
  // the decode step routes over the caller's pyramid (a PyramidCache)
  if (!summary || !level_offsets || !level_sizes || num_levels < 1)
    return fail(PISA_ERR_INVALID, "the fused decode step needs the pyramid and its level tables");
  if (!aligned_rows(summary, dtype, summary_sb, H * D, D)) return fail(PISA_ERR_UNSUPPORTED, "summary rows must be 16-byte aligned");
  {
    // ceil(N / C) leaves, then ceil(n / b) per level; a table may end early
    // only at a single node (it stays that node above)
    int64_t n = blocks;
    for (int64_t l = 0; l < std::min<int64_t>(num_levels, kMaxLevels); ++l) {
      if (level_sizes[l] != n) return fail(PISA_ERR_INVALID, "pyramid level sizes do not match the keys, block_size and branching");
      if (level_offsets[l] < 0) return fail(PISA_ERR_INVALID, "pyramid level offsets must be nonnegative");
      n = (n + branching - 1) / branching;
    }
    if (num_levels < top + 1 && level_sizes[num_levels - 1] != 1)
      return fail(PISA_ERR_INVALID, "pyramid has fewer levels than the routing depth");
  }
  if (B * Tq * H >= (int64_t(1) << 31)) return fail(PISA_ERR_UNSUPPORTED, "too many (token, KV head) items");

  RouteArgs a{};
  a.summary = summary;
  a.s_sb = summary_sb;
  for (int l = 0; l <= top; ++l) {
    const int64_t src = std::min<int64_t>(l, num_levels - 1);
    a.levels.offset[l] = level_offsets[src];
    a.levels.size[l] = int32_t(level_sizes[src]);
  }
  a.q = q; a.q_sb = q_sb; a.q_st = q_st; a.q_sh = q_sh;
  a.keys = keys; a.k_sb = key_sb; a.k_st = key_st; a.k_sh = key_sh;
  a.positions = positions; a.pos_offset = position_offset;
  a.B = int(B); a.T = int(Tq); a.H = int(H); a.G = int(G); a.D = int(D); a.N = int(N);
  a.C = int(block_size); a.K = int(topk); a.br = int(branching); a.method = method;
  a.top = int(top); a.first_width = int(first_width);
  a.force_first = force_first ? 1 : 0; a.force_recent = int(force_recent);
  const double sc = 1.0 / std::sqrt(double(D));
  a.scale = float(sc);
  a.c2 = float(0.5 * sc * sc);
  a.out_ids = out_ids;
  a.coarse_only = 0;
  for (int l = 0; l < kMaxLevels; ++l) a.dense_off[l] = -1;
  a.row_levels = 0;
  a.t_begin = 0; a.t_count = int(Tq);
  a.attend = 1;
  a.values = values; a.v_sb = value_sb; a.v_st = value_st; a.v_sh = value_sh;
  a.Dv = int(Dv);
  a.attn_scale = scale;
  a.out = out;
  a.lse = lse;
  return route(a, dtype, static_cast<cudaStream_t>(stream));
}
