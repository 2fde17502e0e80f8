// extern "C" entry points of libpisa_b200: argument checks, workspace layout
// and dispatch.  Each function documents the reference operator it replaces
// in include/pisa_b200.h.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <string>

#include "internal.h"

namespace pisa {

static thread_local std::string g_last_error;

int fail(int code, const char* msg) {
  g_last_error = msg;
  return code;
}

int fail_cuda(cudaError_t err, const char* where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(err);
  return PISA_ERR_CUDA;
}

static bool is_pow2(int64_t x) { return x > 0 && (x & (x - 1)) == 0; }

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int make_tensor_map(CUtensorMap* map, const void* base, int dtype, int64_t B, int64_t T, int64_t H,
                    int64_t D, int64_t sb, int64_t st, int64_t sh, uint32_t box_h, uint32_t box_t) {
  auto encode = tensor_map_encoder();
  if (!encode) return fail(PISA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int64_t es = dtype == PISA_F32 ? 4 : 2;
  const cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(H), cuuint64_t(T), cuuint64_t(B)};
  const cuuint64_t strides[3] = {cuuint64_t(sh * es), cuuint64_t(st * es), cuuint64_t((B > 1 ? sb : T * st) * es)};
  const cuuint32_t box[4] = {64u, box_h, box_t, 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapDataType type = dtype == PISA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = encode(map, type, 4, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PISA_ERR_UNSUPPORTED, "tensor map encoding rejected the operand layout");
  return PISA_OK;
}

static int elem_size(int dtype) { return dtype == PISA_F32 ? 4 : 2; }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Rows of a [B, T, H, D] view are 16-byte aligned when the base is and every
// stride is a multiple of the 16-byte vector.
static bool rows_aligned(const void* p, int dtype, int64_t sb, int64_t st, int64_t sh) {
  const int64_t v = 16 / elem_size(dtype);
  return aligned16(p) && sb % v == 0 && st % v == 0 && sh % v == 0;
}

static int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Multiprocessor count of the current device (persistent grids).
static int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

struct Geometry {
  int64_t sizes[kMaxLevels];
  int64_t offsets[kMaxLevels];
  int64_t total;
};

// Node counts of levels 0..levels-1 for N keys: ceil(N/C), then ceil(n/br).
static Geometry level_geometry(int64_t N, int64_t C, int64_t br, int64_t levels) {
  Geometry g{};
  int64_t n = (N + C - 1) / C, off = 0;
  for (int64_t l = 0; l < levels && l < kMaxLevels; ++l) {
    g.sizes[l] = n;
    g.offsets[l] = off;
    off += n;
    n = (n + br - 1) / br;
  }
  g.total = off;
  return g;
}

}  // namespace pisa

using namespace pisa;

extern "C" {

int pisa_version(void) { return 100; }

const char* pisa_last_error(void) { return g_last_error.c_str(); }

int pisa_mean_pool(const void* keys, int dtype, int64_t B, int64_t N, int64_t H, int64_t D,
                   int64_t key_sb, int64_t key_st, int64_t key_sh, int64_t size, void* out,
                   pisa_stream_t stream) {
  if (dtype < PISA_F32 || dtype > PISA_F16) return fail(PISA_ERR_UNSUPPORTED, "dtype must be fp32, bf16 or fp16");
  if (size < 1) return fail(PISA_ERR_INVALID, "pool size must be positive");
  if (B <= 0 || N <= 0 || H <= 0 || D <= 0) return fail(PISA_ERR_INVALID, "pooling requires nonempty [B,N,H,D] input");
  if (D % (16 / elem_size(dtype)) != 0) return fail(PISA_ERR_UNSUPPORTED, "head_dim must fill whole 16-byte vectors");
  if (!rows_aligned(keys, dtype, key_sb, key_st, key_sh) || !aligned16(out))
    return fail(PISA_ERR_UNSUPPORTED, "rows must be 16-byte aligned");
  const int64_t blocks = (N + size - 1) / size;
  const int64_t off = 0;
  return build_pyramid(keys, dtype, B, N, H, D, key_sb, key_st, key_sh, size, 2, 1, out,
                       blocks * H * D, &off, 0, static_cast<cudaStream_t>(stream));
}

static int pyramid_checks(const void* keys, int dtype, int64_t B, int64_t N, int64_t H, int64_t D,
                          int64_t sb, int64_t st, int64_t sh, int64_t C, int64_t br, int64_t levels,
                          void* storage, int64_t ssb, const int64_t* offs) {
  if (dtype < PISA_F32 || dtype > PISA_F16) return fail(PISA_ERR_UNSUPPORTED, "dtype must be fp32, bf16 or fp16");
  if (B <= 0 || N <= 0 || H <= 0 || D <= 0) return fail(PISA_ERR_INVALID, "pyramid requires nonempty [B,N,H,D] keys");
  if (C < 1) return fail(PISA_ERR_INVALID, "block_size must be positive");
  if (br < 2) return fail(PISA_ERR_INVALID, "branching must be at least 2");
  if (levels < 1 || levels > kMaxLevels) return fail(PISA_ERR_INVALID, "level count out of range");
  if (!offs) return fail(PISA_ERR_INVALID, "level_offsets is required");
  if (D % (16 / elem_size(dtype)) != 0) return fail(PISA_ERR_UNSUPPORTED, "head_dim must fill whole 16-byte vectors");
  if (!rows_aligned(keys, dtype, sb, st, sh) || !rows_aligned(storage, dtype, ssb, H * D, D))
    return fail(PISA_ERR_UNSUPPORTED, "rows must be 16-byte aligned");
  return PISA_OK;
}

int pisa_build_pyramid(const void* keys, int dtype, int64_t B, int64_t N, int64_t H, int64_t D,
                       int64_t key_sb, int64_t key_st, int64_t key_sh, int64_t block_size,
                       int64_t branching, int64_t num_levels, void* storage, int64_t storage_sb,
                       const int64_t* level_offsets, pisa_stream_t stream) {
  int rc = pyramid_checks(keys, dtype, B, N, H, D, key_sb, key_st, key_sh, block_size, branching,
                          num_levels, storage, storage_sb, level_offsets);
  if (rc) return rc;
  return build_pyramid(keys, dtype, B, N, H, D, key_sb, key_st, key_sh, block_size, branching,
                       num_levels, storage, storage_sb, level_offsets, 0,
                       static_cast<cudaStream_t>(stream));
}

int pisa_pyramid_update(const void* keys, int dtype, int64_t B, int64_t N, int64_t H, int64_t D,
                        int64_t key_sb, int64_t key_st, int64_t key_sh, int64_t block_size,
                        int64_t branching, int64_t num_levels, void* storage, int64_t storage_sb,
                        const int64_t* level_offsets, int64_t first_token, pisa_stream_t stream) {
  int rc = pyramid_checks(keys, dtype, B, N, H, D, key_sb, key_st, key_sh, block_size, branching,
                          num_levels, storage, storage_sb, level_offsets);
  if (rc) return rc;
  if (first_token < 0 || first_token > N) return fail(PISA_ERR_INVALID, "first_token out of range");
  return build_pyramid(keys, dtype, B, N, H, D, key_sb, key_st, key_sh, block_size, branching,
                       num_levels, storage, storage_sb, level_offsets, first_token,
                       static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace pisa {

// Workspace layout of pisa_select_blocks.  The grouped tensor-core path needs
// the leaf candidates, their masks and scores, the bucket counters and the
// tile list; the fused path needs only the pyramid (when built here).
struct SelectPlan {
  bool grouped_tc = false;
  Geometry geo{};
  // dense tensor-core scoring of whole coarse levels (dense.cu), by token chunk
  int dense_off[kMaxLevels];
  uint32_t row_levels = 0;   // levels scored per row inside the warp router
  int64_t dense_row = 0, dense_chunk = 0, dense_off_ws = 0, status_off = 0;
  int64_t W0 = 0, NF = 0, NP = 0, nwin = 0, TW = 4096, RT = 0, rows = 0, num_buckets = 0, capacity = 0;
  int64_t pyramid_off = 0, cand_off = 0, flags_off = 0, scores_off = 0, counts_off = 0,
          cursors_off = 0, offsets_off = 0, misc_off = 0, owner_off = 0, req_off = 0, total = 0;
};

static bool grouped_tc_eligible(int64_t Hq, int64_t H, int64_t D, int dtype, int method,
                                int64_t C, int64_t br, int schedule) {
  const int64_t G = Hq / H;
  return schedule == PISA_SCHEDULE_GROUPED && (dtype == PISA_BF16 || dtype == PISA_F16) &&
         (method == PISA_METHOD_PISA || method == PISA_METHOD_PISA2) && is_pow2(G) && G <= 32 &&
         D % 8 == 0 && D <= 256 && br * C <= 256 &&
         (D <= 64 ? 1 : D <= 128 ? 2 : 4) * 128 * (3 * 128 + br * C) + 1024 + 8192 <= 227 * 1024;
}

static SelectPlan plan_select(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t N,
                              int dtype, int method, int64_t C, int64_t br, int64_t K, int64_t top,
                              int64_t fw, int schedule, int build_summary) {
  SelectPlan p;
  p.geo = level_geometry(N, C, br, top + 1);
  int64_t off = 0;
  p.status_off = off;  // device status word (timeouts of bounded waits) at offset 0
  off += 256;
  if (build_summary) {
    p.pyramid_off = off;
    off += align_up(B * p.geo.total * H * D * elem_size(dtype), 256);
  }
  // Coarse levels scored densely: only for prefill-sized batches of queries,
  // levels that can hold more than K candidates (else the all-fit shortcut
  // scores nothing; pisa1 has no shortcut), children counts up to 8192.
  const int64_t G = Hq / H;
  // (the dense kernel groups children in 1, 2 or 4 columns: pisa1 or b in {2, 4})
  const bool dense_ok = (dtype == PISA_BF16 || dtype == PISA_F16) && is_pow2(G) && G <= 32 &&
                        D % 8 == 0 && D <= 256 && Tq * G >= 1024 &&
                        (method == PISA_METHOD_PISA1 || br == 2 || br == 4);
  // A level can instead be scored by the warp router per row, over the row's
  // own candidates' children (at most 64 columns, G <= 16 heads, 16-bit
  // inputs): W*s child summaries per row, the descent's own work, where the
  // dense kernel scores every node of the level for every row -- work that
  // grows with the square of the sequence length.
  const bool row_ok = (dtype == PISA_BF16 || dtype == PISA_F16) && G <= 16 && D % 8 == 0 && D <= 256 &&
                      (method == PISA_METHOD_PISA1 || br == 2 || br == 4) && std::max(fw, K * br) <= 64;
  for (int l = 0; l < kMaxLevels; ++l) p.dense_off[l] = -1;
  p.row_levels = 0;
  for (int64_t l = top; l >= 0; --l) {
    const int64_t n = p.geo.sizes[l];
    int64_t children;
    if (method == PISA_METHOD_PISA1) {
      children = n;
    } else {
      if (l == 0 || n <= K) continue;
      children = p.geo.sizes[l - 1];
    }
    const int64_t cols = (l == top ? fw : K * br) * (method == PISA_METHOD_PISA1 ? 1 : br);
    const bool dense_level = dense_ok && children <= 8192;
    // (a dense level also reloads every row's queries, so at these widths the
    // row form is the cheaper one whatever the level's size)
    const bool row_level = row_ok && cols <= 64;
    if (row_level) {
      p.row_levels |= 1u << l;
    } else if (dense_level) {
      p.dense_off[l] = int(p.dense_row);
      p.dense_row += n;
    }
  }
  if (p.dense_row > 0) {
    const int64_t budget = int64_t(1) << 30;  // bytes of scores per token chunk
    const int64_t per_token = B * H * p.dense_row * 4;
    p.dense_chunk = std::min<int64_t>(Tq, std::max<int64_t>(128, budget / per_token / 128 * 128));
    p.dense_off_ws = off;
    off += align_up(B * p.dense_chunk * H * p.dense_row * 4, 256);
  }
  // The schedule selects an implementation, not a result: both give the same
  // selection.  The fused single-kernel router gives each (row, KV head) one
  // CTA of four warps, whose leaf scoring (b*K candidate blocks of raw keys)
  // is latency bound; from 32 rows on, a fused request runs the grouped tile
  // pipeline instead (measured at a 16K-token cache: 64 rows 123 against
  // 362 us, 128 rows 156 against 365 us).
  const int eff_schedule = (schedule == PISA_SCHEDULE_FUSED && B * Tq * H >= 32) ? PISA_SCHEDULE_GROUPED : schedule;
  p.grouped_tc = grouped_tc_eligible(Hq, H, D, dtype, method, C, br, eff_schedule);
  if (p.grouped_tc) {
    p.W0 = top == 0 ? fw : K * br;
    p.NF = p.W0 / br;
    p.NP = top == 0 ? fw / br : p.geo.sizes[1];
    p.nwin = (Tq + p.TW - 1) / p.TW;
    p.RT = 128 / (Hq / H);
    p.rows = B * Tq * H;
    p.num_buckets = B * p.nwin * H * p.NP;
    p.capacity = (p.rows * p.NF + p.RT - 1) / p.RT + p.num_buckets;
    // request and score-slot indices are decoded as 31-bit numbers
    if (p.rows * p.W0 >= (int64_t(1) << 31) || p.capacity * p.RT >= (int64_t(1) << 31)) p.grouped_tc = false;
  }
  if (p.grouped_tc) {
    const int64_t slots = p.rows * p.W0;
    p.cand_off = off; off += align_up(slots * 4, 256);
    p.flags_off = off; off += align_up(slots, 256);
    p.scores_off = off; off += align_up(slots * 4, 256);
    p.counts_off = off; off += align_up(p.num_buckets * 4, 256);
    p.cursors_off = off; off += align_up(p.num_buckets * 4, 256);
    p.offsets_off = off; off += align_up(p.num_buckets * 4, 256);
    p.misc_off = off; off += 256;
    p.owner_off = off; off += align_up(p.capacity * 4, 256);
    p.req_off = off; off += align_up(p.capacity * p.RT * 4, 256);
  }
  p.total = off;
  return p;
}

}  // namespace pisa

extern "C" {

int64_t pisa_select_workspace_bytes(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D,
                                    int64_t N, int dtype, int method, int64_t block_size,
                                    int64_t branching, int64_t topk, int64_t top,
                                    int64_t first_width, int schedule, int build_summary) {
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || D <= 0 || N <= 0 || block_size < 1 ||
      branching < 2 || top < 0 || top >= kMaxLevels || Hq % H)
    return 0;
  return plan_select(B, Tq, Hq, H, D, N, dtype, method, block_size, branching, topk, top,
                     first_width, schedule, build_summary).total;
}

int64_t pisa_select_level_plan(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t N, int dtype,
                               int method, int64_t block_size, int64_t branching, int64_t topk, int64_t top,
                               int64_t first_width, int schedule) {
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || D <= 0 || N <= 0 || block_size < 1 ||
      branching < 2 || top < 0 || top >= kMaxLevels || Hq % H)
    return -1;
  const SelectPlan p = plan_select(B, Tq, Hq, H, D, N, dtype, method, block_size, branching, topk, top,
                                   first_width, schedule, 0);
  int64_t dense = 0;
  for (int l = 0; l <= top; ++l)
    if (p.dense_off[l] >= 0) dense |= int64_t(1) << l;
  return dense | (int64_t(p.row_levels) << 32);
}

int pisa_select_blocks(const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh, const void* keys,
                       int64_t key_sb, int64_t key_st, int64_t key_sh, const void* summary,
                       int64_t summary_sb, const int64_t* level_offsets,
                       const int64_t* level_sizes, int64_t num_levels, const int64_t* positions,
                       int64_t position_offset, int dtype, int64_t B, int64_t Tq, int64_t Hq,
                       int64_t H, int64_t D, int64_t N, int method, int64_t block_size,
                       int64_t branching, int64_t topk, int force_first, int64_t force_recent,
                       int64_t top, int64_t first_width, int schedule, int64_t* out_ids,
                       void* workspace, int64_t workspace_bytes, pisa_stream_t stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype < PISA_F32 || dtype > PISA_F16) return fail(PISA_ERR_UNSUPPORTED, "GPU routing supports FP16, BF16 and FP32");
  if (method < PISA_METHOD_PISA1 || method > PISA_METHOD_PISA) return fail(PISA_ERR_INVALID, "method must be pisa1, pisa2 or pisa");
  if (schedule != PISA_SCHEDULE_GROUPED && schedule != PISA_SCHEDULE_FUSED) return fail(PISA_ERR_INVALID, "routing_schedule must be grouped or fused");
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || D <= 0 || N <= 0) return fail(PISA_ERR_INVALID, "nonempty tensors are required");
  if (Hq % H) return fail(PISA_ERR_INVALID, "a whole number of query heads per KV head is required");
  if (Hq / H > 32) return fail(PISA_ERR_UNSUPPORTED, "at most 32 query heads per KV head");
  if (D % 8 || D > 256) return fail(PISA_ERR_UNSUPPORTED, "head_dim must be a multiple of 8 and at most 256");
  if (!is_pow2(topk) || topk < 8 || topk > 64 || !is_pow2(block_size) || block_size < 16)
    return fail(PISA_ERR_UNSUPPORTED, "GPU routing requires power-of-two block_size >= 16 and topk in {8,16,32,64}");
  if (branching != 2 && branching != 4) return fail(PISA_ERR_UNSUPPORTED, "branching must be 2 or 4");
  if (force_recent < 1) return fail(PISA_ERR_INVALID, "causal pyramid routing requires force_recent >= 1");
  const int64_t blocks = (N + block_size - 1) / block_size;
  if (topk < std::min<int64_t>(blocks, force_recent + (force_first ? 1 : 0)))
    return fail(PISA_ERR_INVALID, "topk cannot hold all required blocks");
  if (top < 0 || top >= kMaxLevels) return fail(PISA_ERR_INVALID, "routing depth out of range");
  if (!is_pow2(first_width) || first_width < 16 || first_width > 256)
    return fail(PISA_ERR_UNSUPPORTED, "first network width must be a power of two in [16, 256]");
  if (topk * branching > 256) return fail(PISA_ERR_UNSUPPORTED, "topk * branching must be at most 256");
  if (!out_ids) return fail(PISA_ERR_INVALID, "out_ids is required");
  if (!rows_aligned(q, dtype, q_sb, q_st, q_sh) || !rows_aligned(keys, dtype, key_sb, key_st, key_sh))
    return fail(PISA_ERR_UNSUPPORTED, "q and key rows must be 16-byte aligned");

  if (summary != nullptr) {
    if (!level_offsets || !level_sizes || num_levels < 1) return fail(PISA_ERR_INVALID, "pyramid level tables are required");
    if (!rows_aligned(summary, dtype, summary_sb, H * D, D)) return fail(PISA_ERR_UNSUPPORTED, "summary rows must be 16-byte aligned");
    // The tables must describe the pyramid of these keys for this block size
    // and branching: ceil(N / C) leaves, then ceil(n / b) per level.  A table
    // may end early only at a single node (it stays that node above).
    {
      const Geometry want = level_geometry(N, block_size, branching, std::min<int64_t>(num_levels, kMaxLevels));
      for (int64_t l = 0; l < std::min<int64_t>(num_levels, kMaxLevels); ++l) {
        if (level_sizes[l] != want.sizes[l])
          return fail(PISA_ERR_INVALID, "pyramid level sizes do not match the keys, block_size and branching");
        if (level_offsets[l] < 0) return fail(PISA_ERR_INVALID, "pyramid level offsets must be nonnegative");
      }
      if (num_levels < top + 1 && level_sizes[num_levels - 1] != 1)
        return fail(PISA_ERR_INVALID, "pyramid has fewer levels than the routing depth");
    }
  }

  const SelectPlan plan = plan_select(B, Tq, Hq, H, D, N, dtype, method, block_size, branching,
                                      topk, top, first_width, schedule, summary == nullptr);
  if (plan.total > 0 && (!workspace || workspace_bytes < plan.total))
    return fail(PISA_ERR_INVALID, "workspace too small");
  char* ws = static_cast<char*>(workspace);
  {
    cudaError_t e = cudaMemsetAsync(ws + plan.status_off, 0, 256, s);
    if (e != cudaSuccess) return fail_cuda(e, "status clear");
  }

  RouteArgs a{};
  if (summary == nullptr) {
    const Geometry& g = plan.geo;
    int rc = build_pyramid(keys, dtype, B, N, H, D, key_sb, key_st, key_sh, block_size, branching,
                           top + 1, ws + plan.pyramid_off, g.total * H * D, g.offsets, 0, s);
    if (rc) return rc;
    a.summary = ws + plan.pyramid_off;
    a.s_sb = g.total * H * D;
    for (int l = 0; l <= top; ++l) { a.levels.offset[l] = g.offsets[l]; a.levels.size[l] = int32_t(g.sizes[l]); }
  } else {
    a.summary = summary;
    a.s_sb = summary_sb;
    // A one-node local pyramid remains that node at additional common levels
    // (top_k_pyramid_torch.py:145-147).
    for (int l = 0; l <= top; ++l) {
      const int64_t src = std::min<int64_t>(l, num_levels - 1);
      a.levels.offset[l] = level_offsets[src];
      a.levels.size[l] = int32_t(level_sizes[src]);
    }
  }
  a.q = q; a.q_sb = q_sb; a.q_st = q_st; a.q_sh = q_sh;
  a.keys = keys; a.k_sb = key_sb; a.k_st = key_st; a.k_sh = key_sh;
  a.positions = positions; a.pos_offset = position_offset;
  a.B = int(B); a.T = int(Tq); a.H = int(H); a.G = int(Hq / H); a.D = int(D); a.N = int(N);
  a.C = int(block_size); a.K = int(topk); a.br = int(branching); a.method = method;
  a.top = int(top); a.first_width = int(first_width);
  a.force_first = force_first ? 1 : 0; a.force_recent = int(force_recent);
  const double scale = 1.0 / std::sqrt(double(D));
  a.scale = float(scale);
  a.c2 = float(0.5 * scale * scale);
  a.out_ids = out_ids;
  a.coarse_only = plan.grouped_tc ? 1 : 0;
  if (plan.grouped_tc) {
    // grouped: coarse levels -> leaf candidates + masks (and, on the warp
    // router, the leaf bucket counts), then tensor-core leaf scoring
    a.W0 = int(plan.W0);
    a.candidates = reinterpret_cast<int32_t*>(ws + plan.cand_off);
    a.flags = reinterpret_cast<uint8_t*>(ws + plan.flags_off);
    a.fam_counts = reinterpret_cast<int32_t*>(ws + plan.counts_off);
    a.NP = int(plan.NP); a.nwin = int(plan.nwin); a.TW = int(plan.TW);
    cudaError_t e = cudaMemsetAsync(a.fam_counts, 0, sizeof(int32_t) * plan.num_buckets, s);
    if (e != cudaSuccess) return fail_cuda(e, "bucket counts clear");
  }
  bool counted = true;
  for (int l = 0; l < kMaxLevels; ++l) a.dense_off[l] = plan.dense_off[l];
  a.row_levels = plan.row_levels;
  int rc = PISA_OK;
  if (plan.dense_row == 0) {
    a.t_begin = 0; a.t_count = int(Tq);
    rc = route(a, dtype, s, &counted);
  } else {
    float* dense = reinterpret_cast<float*>(ws + plan.dense_off_ws);
    a.dense = dense;
    a.dense_stride = plan.dense_row;
    DenseArgs d{};
    d.q = q; d.q_sb = q_sb; d.q_st = q_st; d.q_sh = q_sh;
    d.summary = a.summary; d.s_sb = a.s_sb;
    d.positions = positions; d.pos_offset = position_offset;
    d.B = int(B); d.T = int(Tq); d.H = int(H); d.G = int(Hq / H); d.D = int(D);
    d.Dp = int(D <= 64 ? 64 : D <= 128 ? 128 : 256); d.method = method;
    d.bf16 = dtype == PISA_BF16 ? 1 : 0; d.scale = a.scale; d.c2 = a.c2;
    d.scores = dense; d.row_stride = plan.dense_row;
    d.status = reinterpret_cast<int*>(ws + plan.status_off);
    int64_t total_nodes = 0;
    for (int l = 0; l <= top; ++l) total_nodes = std::max<int64_t>(total_nodes, a.levels.offset[l] + a.levels.size[l]);
    rc = make_tensor_map(&d.tm_q, q, dtype, B, Tq, Hq, D, q_sb, q_st, q_sh, uint32_t(d.G), uint32_t(128 / d.G));
    if (rc == PISA_OK)
      rc = make_tensor_map(&d.tm_x, a.summary, dtype, B, total_nodes, H, D, a.s_sb, H * D, D, 1, 64);
    for (int64_t t0 = 0; t0 < Tq && rc == PISA_OK; t0 += plan.dense_chunk) {
      const int tc = int(std::min<int64_t>(plan.dense_chunk, Tq - t0));
      d.t_begin = int(t0); d.t_count = tc;
      for (int l = 0; l <= top && rc == PISA_OK; ++l) {
        if (plan.dense_off[l] < 0) continue;
        const bool self = method == PISA_METHOD_PISA1;
        const int child = self ? l : l - 1;
        d.child_off = a.levels.offset[child];
        d.n_child = a.levels.size[child];
        d.support = self ? 1 : int(branching);
        int64_t span = block_size;
        for (int i = 0; i < l; ++i) span *= branching;
        d.span = span;
        d.out_off = plan.dense_off[l];
        rc = dense_level(d, dtype, s);
      }
      if (rc) break;
      a.t_begin = int(t0); a.t_count = tc;
      bool c = false;
      rc = route(a, dtype, s, &c);
      counted = counted && c;
    }
  }
  if (rc || !plan.grouped_tc) return rc;
  GroupArgs g{};
  g.q = q; g.q_sb = q_sb; g.q_st = q_st; g.q_sh = q_sh;
  g.keys = keys; g.k_sb = key_sb; g.k_st = key_st; g.k_sh = key_sh;
  g.positions = positions; g.pos_offset = position_offset;
  g.B = int(B); g.T = int(Tq); g.H = int(H); g.G = int(Hq / H); g.D = int(D);
  g.Dp = int(D <= 64 ? 64 : D <= 128 ? 128 : 256); g.N = int(N); g.C = int(block_size); g.K = int(topk);
  g.br = int(branching); g.W0 = int(plan.W0); g.NF = int(plan.NF); g.NP = int(plan.NP);
  g.nwin = int(plan.nwin); g.TW = int(plan.TW); g.RT = int(plan.RT);
  g.method = method; g.bf16 = dtype == PISA_BF16 ? 1 : 0;
  g.scale = a.scale; g.c2 = a.c2;
  g.cand = a.candidates; g.flags = a.flags;
  g.scores = reinterpret_cast<float*>(ws + plan.scores_off);
  g.counts = reinterpret_cast<int32_t*>(ws + plan.counts_off);
  g.cursors = reinterpret_cast<int32_t*>(ws + plan.cursors_off);
  g.offsets = reinterpret_cast<int32_t*>(ws + plan.offsets_off);
  g.num_buckets = plan.num_buckets;
  g.total_tiles_w = reinterpret_cast<int32_t*>(ws + plan.misc_off);
  g.total_tiles = g.total_tiles_w;
  g.status = reinterpret_cast<int*>(ws + plan.status_off);
  g.tile_owner_w = reinterpret_cast<int32_t*>(ws + plan.owner_off);
  g.tile_owner = g.tile_owner_w;
  g.tile_req_w = reinterpret_cast<int32_t*>(ws + plan.req_off);
  g.tile_req = g.tile_req_w;
  g.tile_capacity = plan.capacity;
  g.tiles_per_cta = 8;
  g.counts_ready = counted ? 1 : 0;
  // two accumulators (double buffering) whenever they fit in the 512 TMEM columns
  const int64_t nk = branching * block_size;
  const int64_t want = nk <= 256 ? 2 * nk : nk;
  g.tmem_cols = want <= 32 ? 32 : want <= 64 ? 64 : want <= 128 ? 128 : want <= 256 ? 256 : 512;
  g.num_sms = num_sms();
  g.out_ids = out_ids;
  rc = make_tensor_map(&g.tm_q, q, dtype, B, Tq, Hq, D, q_sb, q_st, q_sh, uint32_t(g.G), 1);
  if (rc == PISA_OK)
    rc = make_tensor_map(&g.tm_k, keys, dtype, B, N, H, D, key_sb, key_st, key_sh, 1, uint32_t(nk));
  if (rc) return rc;
  return grouped_leaf(g, dtype, s);
}

}  // extern "C"

namespace pisa {

// Workspace layout of pisa_leaf_scores: status word, int32 ids, masks, then
// either the leaf means (pisa1 without caller means) or the buckets and tile
// list of the grouped tensor-core scorer (one family per candidate block).
struct LeafPlan {
  bool tc = false;
  int64_t rows = 0, blocks = 0, nwin = 0, TW = 4096, RT = 0, num_buckets = 0, capacity = 0;
  int64_t status_off = 0, cand_off = 0, flags_off = 0, means_off = -1, counts_off = 0, cursors_off = 0,
          offsets_off = 0, misc_off = 0, owner_off = 0, req_off = 0, total = 0;
};

static LeafPlan plan_leaf(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t N, int64_t W,
                          int dtype, int method, int64_t C, bool have_means) {
  LeafPlan p;
  p.rows = B * Tq * H;
  p.blocks = (N + C - 1) / C;
  int64_t off = 0;
  p.status_off = off; off += 256;
  p.cand_off = off; off += align_up(p.rows * W * 4, 256);
  p.flags_off = off; off += align_up(p.rows * W, 256);
  p.tc = grouped_tc_eligible(Hq, H, D, dtype, method, C, 1, PISA_SCHEDULE_GROUPED) && C <= 256;
  if (p.tc) {
    p.RT = 128 / (Hq / H);
    p.nwin = (Tq + p.TW - 1) / p.TW;
    p.num_buckets = B * p.nwin * H * p.blocks;
    p.capacity = (p.rows * W + p.RT - 1) / p.RT + p.num_buckets;
    if (p.rows * W >= (int64_t(1) << 31) || p.capacity * p.RT >= (int64_t(1) << 31) ||
        p.num_buckets >= (int64_t(1) << 31))
      p.tc = false;
  }
  if (p.tc) {
    p.counts_off = off; off += align_up(p.num_buckets * 4, 256);
    p.cursors_off = off; off += align_up(p.num_buckets * 4, 256);
    p.offsets_off = off; off += align_up(p.num_buckets * 4, 256);
    p.misc_off = off; off += 256;
    p.owner_off = off; off += align_up(p.capacity * 4, 256);
    p.req_off = off; off += align_up(p.capacity * p.RT * 4, 256);
  } else if (method == PISA_METHOD_PISA1 && !have_means) {
    p.means_off = off; off += align_up(B * p.blocks * H * D * elem_size(dtype), 256);
  }
  p.total = off;
  return p;
}

}  // namespace pisa

extern "C" {

int64_t pisa_leaf_scores_workspace_bytes(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t N,
                                         int64_t W, int dtype, int method, int64_t block_size,
                                         int have_means) {
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || D <= 0 || N <= 0 || W < 0 || block_size < 1 || Hq % H) return 0;
  return plan_leaf(B, Tq, Hq, H, D, N, W, dtype, method, block_size, have_means != 0).total;
}

int pisa_leaf_scores(const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh, const void* keys,
                     int64_t key_sb, int64_t key_st, int64_t key_sh, const void* leaf_means,
                     int64_t means_sb, const void* candidates, int cand_bytes, const int64_t* positions,
                     int dtype, int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t N,
                     int64_t W, int method, int64_t block_size, int64_t topk, int force_first,
                     int64_t force_recent, float* out_scores, void* workspace, int64_t workspace_bytes,
                     pisa_stream_t stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype < PISA_F32 || dtype > PISA_F16) return fail(PISA_ERR_UNSUPPORTED, "grouped leaf scoring supports FP16, BF16 and FP32");
  if (method < PISA_METHOD_PISA1 || method > PISA_METHOD_PISA) return fail(PISA_ERR_INVALID, "expected method pisa1/pisa2/pisa");
  if (block_size <= 0) return fail(PISA_ERR_INVALID, "block_size must be positive");
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || D <= 0 || N <= 0 || W < 0) return fail(PISA_ERR_INVALID, "nonempty tensors are required");
  if (Hq % H) return fail(PISA_ERR_INVALID, "a whole number of query heads per KV head is required");
  if (Hq / H > 32) return fail(PISA_ERR_UNSUPPORTED, "at most 32 query heads per KV head");
  if (D % 8 || D > 256) return fail(PISA_ERR_UNSUPPORTED, "head_dim must be a multiple of 8 and at most 256");
  if (cand_bytes != 4 && cand_bytes != 8) return fail(PISA_ERR_INVALID, "candidates must be int32 or int64");
  if (positions && method != PISA_METHOD_PISA1 && topk < 0) return fail(PISA_ERR_INVALID, "topk is required with positions");
  if (positions && force_recent < 0) return fail(PISA_ERR_INVALID, "force_recent must be nonnegative");
  if (!out_scores || (W > 0 && !candidates)) return fail(PISA_ERR_INVALID, "candidates and out_scores are required");
  if (!rows_aligned(q, dtype, q_sb, q_st, q_sh) || !rows_aligned(keys, dtype, key_sb, key_st, key_sh))
    return fail(PISA_ERR_UNSUPPORTED, "q and key rows must be 16-byte aligned");
  if (leaf_means && !rows_aligned(leaf_means, dtype, means_sb, H * D, D))
    return fail(PISA_ERR_UNSUPPORTED, "leaf mean rows must be 16-byte aligned");
  if (W == 0) return PISA_OK;
  const LeafPlan plan = plan_leaf(B, Tq, Hq, H, D, N, W, dtype, method, block_size, leaf_means != nullptr);
  if (!workspace || workspace_bytes < plan.total) return fail(PISA_ERR_INVALID, "workspace too small");
  char* ws = static_cast<char*>(workspace);
  cudaError_t e = cudaMemsetAsync(ws + plan.status_off, 0, 256, s);
  if (e != cudaSuccess) return fail_cuda(e, "status clear");

  LeafPrepArgs p{};
  p.cand = candidates; p.cand_bytes = cand_bytes; p.positions = positions;
  p.B = int(B); p.T = int(Tq); p.H = int(H); p.W = int(W); p.C = int(block_size);
  p.K = int(topk); p.method = method; p.force_first = force_first ? 1 : 0; p.force_recent = int(force_recent);
  p.blocks = plan.blocks;
  p.cand_out = reinterpret_cast<int32_t*>(ws + plan.cand_off);
  p.flags = reinterpret_cast<uint8_t*>(ws + plan.flags_off);
  p.scores = out_scores;
  int rc = leaf_prepare(p, s);
  if (rc) return rc;
  const double scale = 1.0 / std::sqrt(double(D));

  if (!plan.tc) {
    RouteArgs a{};
    a.q = q; a.q_sb = q_sb; a.q_st = q_st; a.q_sh = q_sh;
    a.keys = keys; a.k_sb = key_sb; a.k_st = key_st; a.k_sh = key_sh;
    a.B = int(B); a.T = int(Tq); a.H = int(H); a.G = int(Hq / H); a.D = int(D); a.N = int(N);
    a.C = int(block_size); a.method = method; a.scale = float(scale); a.c2 = float(0.5 * scale * scale);
    a.levels.size[0] = int32_t(plan.blocks);
    const void* means = leaf_means;
    int64_t msb = means_sb;
    if (method == PISA_METHOD_PISA1 && !means) {
      // leaf means of these keys (fp32 accumulation), as mean_pool(k, block_size)
      const int64_t zero = 0;
      rc = build_pyramid(keys, dtype, B, N, H, D, key_sb, key_st, key_sh, block_size, 2, 1,
                         ws + plan.means_off, plan.blocks * H * D, &zero, 0, s);
      if (rc) return rc;
      means = ws + plan.means_off;
      msb = plan.blocks * H * D;
    }
    return leaf_scores_simt(a, p.cand_out, p.flags, int(W), out_scores, means, msb, dtype, s);
  }

  GroupArgs g{};
  g.q = q; g.q_sb = q_sb; g.q_st = q_st; g.q_sh = q_sh;
  g.keys = keys; g.k_sb = key_sb; g.k_st = key_st; g.k_sh = key_sh;
  g.B = int(B); g.T = int(Tq); g.H = int(H); g.G = int(Hq / H); g.D = int(D);
  g.Dp = int(D <= 64 ? 64 : D <= 128 ? 128 : 256); g.N = int(N); g.C = int(block_size); g.K = int(topk);
  // one family per candidate block: W slots of one child each, bucketed by block id
  g.br = 1; g.W0 = int(W); g.NF = int(W); g.NP = int(plan.blocks);
  g.nwin = int(plan.nwin); g.TW = int(plan.TW); g.RT = int(plan.RT);
  g.method = method; g.bf16 = dtype == PISA_BF16 ? 1 : 0;
  g.scale = float(scale); g.c2 = float(0.5 * scale * scale);
  g.cand = p.cand_out; g.flags = p.flags; g.scores = out_scores;
  g.counts = reinterpret_cast<int32_t*>(ws + plan.counts_off);
  g.cursors = reinterpret_cast<int32_t*>(ws + plan.cursors_off);
  g.offsets = reinterpret_cast<int32_t*>(ws + plan.offsets_off);
  g.num_buckets = plan.num_buckets;
  g.total_tiles_w = reinterpret_cast<int32_t*>(ws + plan.misc_off);
  g.total_tiles = g.total_tiles_w;
  g.status = reinterpret_cast<int*>(ws + plan.status_off);
  g.tile_owner_w = reinterpret_cast<int32_t*>(ws + plan.owner_off);
  g.tile_owner = g.tile_owner_w;
  g.tile_req_w = reinterpret_cast<int32_t*>(ws + plan.req_off);
  g.tile_req = g.tile_req_w;
  g.tile_capacity = plan.capacity;
  g.tiles_per_cta = 8;
  g.counts_ready = 0;
  g.skip_final = 1;
  const int64_t nk = block_size;
  const int64_t want = 2 * nk;
  g.tmem_cols = want <= 32 ? 32 : want <= 64 ? 64 : want <= 128 ? 128 : want <= 256 ? 256 : 512;
  g.num_sms = num_sms();
  rc = make_tensor_map(&g.tm_q, q, dtype, B, Tq, Hq, D, q_sb, q_st, q_sh, uint32_t(g.G), 1);
  if (rc == PISA_OK) rc = make_tensor_map(&g.tm_k, keys, dtype, B, N, H, D, key_sb, key_st, key_sh, 1, uint32_t(nk));
  if (rc) return rc;
  return grouped_leaf(g, dtype, s);
}

}  // extern "C"

namespace pisa {

// Workspace layout of the bucketed tensor-core attention forward (one token
// chunk at a time; the partials of a chunk are bounded to kAttnPartialBudget).
// 16 GiB takes the 32K benchmark sequence in one chunk (about 10 GB of
// partials) and the 256K one in five: fewer bucketing passes and tile-kernel
// tails than 4 GiB chunks, on a GPU with 180 GB of HBM.
constexpr int64_t kAttnPartialBudget = int64_t(16) << 30;
struct AttnPlan {
  bool tc = false;
  int64_t TW = 4096, chunk = 0, NB = 0, RT = 0, num_buckets = 0, capacity = 0;
  int64_t sp_cols = 0, o_cols = 0, tmem_cols = 0, nacc = 1, nstages = 2;
  int64_t status_off = 0, counts_off = 0, cursors_off = 0, offsets_off = 0, misc_off = 0, owner_off = 0,
          req_off = 0, po_off = 0, pml_off = 0, total = 0;
};

static AttnPlan plan_attn(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t Dv,
                          int64_t N, int64_t S, int64_t C, int dtype) {
  AttnPlan p;
  const int64_t G = Hq / H;
  // TMEM: S/P buffers (C columns of S, then C/2 packed columns of P) and O
  // buffers (Dv columns), two of each when they fit in 512 columns
  p.sp_cols = (C + C / 2 + 31) / 32 * 32;
  p.o_cols = (Dv + 31) / 32 * 32;
  p.nacc = 2 * (p.sp_cols + p.o_cols) <= 512 ? 2 : 1;
  const int64_t cols = p.nacc * (p.sp_cols + p.o_cols);
  p.tmem_cols = cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
  const int64_t Dp = D <= 64 ? 64 : D <= 128 ? 128 : 256, Dvp = Dv <= 64 ? 64 : Dv <= 128 ? 128 : 256;
  // K/V buffers, alignment slack, readout staging (16 KB) and static shared memory
  const int64_t kv_smem = 2 * C * 2 * (Dp + Dvp) + 1024 + 16384 + 17408;
  p.nstages = 3 * 128 * 2 * Dp + kv_smem <= 227 * 1024 ? 3 : 2;
  const int64_t smem = p.nstages * 128 * 2 * Dp + kv_smem;
  p.tc = (dtype == PISA_BF16 || dtype == PISA_F16) && is_pow2(G) && G <= 32 && D % 16 == 0 &&
         Dv % 32 == 0 && D <= 256 && Dv <= 256 && is_pow2(C) && C >= 16 && C <= 256 &&
         cols <= 512 && smem <= 227 * 1024 && S > 0 && S <= 64 && B * Tq * H * S >= 4096 &&
         Tq * G >= 64;
  // (a bucket holds requests of one sequence, so its tiles of 128 rows fill
  // only when a sequence brings at least 64 query rows; below that, as in
  // batched decode, the gather kernel reads the selected blocks directly:
  // 202 us against 319 us per 64-sequence decode step at 128K)
  if (!p.tc) return p;
  const int64_t per_token = H * S * G * (Dv * elem_size(dtype) + 8) * 9 / 8;
  const int64_t fit = (kAttnPartialBudget / per_token) / p.TW * p.TW;
  p.chunk = std::min<int64_t>(Tq, std::max<int64_t>(p.TW, fit));
  p.NB = (N + C - 1) / C;
  p.RT = 128 / G;
  const int64_t nwin = (p.chunk + p.TW - 1) / p.TW;
  p.num_buckets = B * nwin * H * p.NB;
  const int64_t reqs = B * p.chunk * H * S;
  if (reqs >= (int64_t(1) << 31) || B * p.chunk * Hq >= (int64_t(1) << 31)) { p.tc = false; return p; }
  p.capacity = (reqs + p.RT - 1) / p.RT + p.num_buckets;
  // tile slots (tile * RT + slot) are decoded as 31-bit numbers
  if (p.capacity * p.RT >= (int64_t(1) << 31)) { p.tc = false; return p; }
  int64_t off = 0;
  p.status_off = off; off += 256;  // device status word (timeouts of bounded waits) at offset 0
  p.counts_off = off; off += align_up(p.num_buckets * 4, 256);
  p.cursors_off = off; off += align_up(p.num_buckets * 4, 256);
  p.offsets_off = off; off += align_up(p.num_buckets * 4, 256);
  p.misc_off = off; off += 256;
  p.owner_off = off; off += align_up(p.capacity * 4, 256);
  p.req_off = off; off += align_up(p.capacity * p.RT * 4, 256);
  // block partials, query-major: row (request, head) at request * G + head
  p.po_off = off; off += align_up(reqs * G * Dv * elem_size(dtype), 256);
  p.pml_off = off; off += align_up(reqs * G * 8, 256);
  p.total = off;
  return p;
}

}  // namespace pisa

extern "C" {

int64_t pisa_sparse_attn_fwd_workspace_bytes(int64_t B, int64_t Tq, int64_t Hq, int64_t H,
                                             int64_t D, int64_t Dv, int64_t N, int64_t S,
                                             int64_t block_size, int dtype) {
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || Hq % H || block_size < 1) return 0;
  return plan_attn(B, Tq, Hq, H, D, Dv, N, S, block_size, dtype).total;
}

int pisa_sparse_attn_fwd(const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh, const void* k,
                         int64_t k_sb, int64_t k_st, int64_t k_sh, const void* v, int64_t v_sb,
                         int64_t v_st, int64_t v_sh, const void* indices, int index_bytes,
                         const int64_t* positions, int64_t position_offset, int dtype, int64_t B,
                         int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t Dv, int64_t N,
                         int64_t S, int64_t block_size, float scale, int causal, void* out,
                         float* lse, void* workspace, int64_t workspace_bytes,
                         pisa_stream_t stream) {
  if (dtype < PISA_F32 || dtype > PISA_F16) return fail(PISA_ERR_UNSUPPORTED, "CUDA attention supports FP16, BF16 and FP32");
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || D <= 0 || Dv <= 0 || N <= 0) return fail(PISA_ERR_INVALID, "nonempty tensors are required");
  if (Hq % H) return fail(PISA_ERR_INVALID, "a whole number of query heads per KV head is required");
  if (S < 0) return fail(PISA_ERR_INVALID, "negative slot count");
  if (block_size < 1) return fail(PISA_ERR_INVALID, "invalid block_size");
  if (index_bytes != 4 && index_bytes != 8) return fail(PISA_ERR_INVALID, "indices must be int32 or int64");
  if (D % 8 || Dv % 8 || D > 256 || Dv > 256) return fail(PISA_ERR_UNSUPPORTED, "head_dim must be a multiple of 8 and at most 256");
  if (!rows_aligned(q, dtype, q_sb, q_st, q_sh) || !rows_aligned(k, dtype, k_sb, k_st, k_sh) ||
      !rows_aligned(v, dtype, v_sb, v_st, v_sh))
    return fail(PISA_ERR_UNSUPPORTED, "q, key and value rows must be 16-byte aligned");
  if (!out) return fail(PISA_ERR_INVALID, "out is required");
  const AttnPlan plan = plan_attn(B, Tq, Hq, H, D, Dv, N, S, block_size, dtype);
  if (plan.tc && workspace && workspace_bytes >= plan.total) {
    char* ws = static_cast<char*>(workspace);
    AttnTcArgs a{};
    a.q = q; a.q_sb = q_sb; a.q_st = q_st; a.q_sh = q_sh;
    a.k = k; a.k_sb = k_sb; a.k_st = k_st; a.k_sh = k_sh;
    a.v = v; a.v_sb = v_sb; a.v_st = v_st; a.v_sh = v_sh;
    a.indices = indices; a.index_bytes = index_bytes;
    a.positions = positions; a.pos_offset = position_offset;
    a.B = int(B); a.T = int(Tq); a.Hq = int(Hq); a.H = int(H); a.G = int(Hq / H);
    a.D = int(D); a.Dp = int(D <= 64 ? 64 : D <= 128 ? 128 : 256);
    a.Dv = int(Dv); a.Dvp = int(Dv <= 64 ? 64 : Dv <= 128 ? 128 : 256);
    a.N = int(N); a.S = int(S); a.C = int(block_size); a.NB = int(plan.NB); a.TW = int(plan.TW);
    a.RT = int(plan.RT); a.chunk = int(plan.chunk);
    a.scale = scale; a.causal = causal ? 1 : 0; a.bf16 = dtype == PISA_BF16 ? 1 : 0;
    a.counts = reinterpret_cast<int32_t*>(ws + plan.counts_off);
    a.cursors = reinterpret_cast<int32_t*>(ws + plan.cursors_off);
    a.offsets = reinterpret_cast<int32_t*>(ws + plan.offsets_off);
    a.total_tiles = reinterpret_cast<int32_t*>(ws + plan.misc_off);
    a.status = reinterpret_cast<int*>(ws + plan.status_off);
    {
      cudaError_t e = cudaMemsetAsync(ws + plan.status_off, 0, 256, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return fail_cuda(e, "status clear");
    }
    a.tile_owner = reinterpret_cast<int32_t*>(ws + plan.owner_off);
    a.tile_req = reinterpret_cast<int32_t*>(ws + plan.req_off);
    a.part_o = ws + plan.po_off;
    a.part_ml = reinterpret_cast<float*>(ws + plan.pml_off);
    a.tiles_per_cta = 8;
    a.tmem_cols = int(plan.tmem_cols); a.sp_cols = int(plan.sp_cols); a.o_cols = int(plan.o_cols);
    a.nacc = int(plan.nacc); a.nstages = int(plan.nstages); a.num_sms = num_sms();
    a.out = out; a.lse = lse;
    int rc = make_tensor_map(&a.tm_q, q, dtype, B, Tq, Hq, D, q_sb, q_st, q_sh, uint32_t(a.G), 1);
    if (rc == PISA_OK) rc = make_tensor_map(&a.tm_k, k, dtype, B, N, H, D, k_sb, k_st, k_sh, 1, uint32_t(block_size));
    if (rc == PISA_OK) rc = make_tensor_map(&a.tm_v, v, dtype, B, N, H, Dv, v_sb, v_st, v_sh, 1, uint32_t(block_size));
    if (rc) return rc;
    return attn_fwd_tc(a, dtype, static_cast<cudaStream_t>(stream));
  }
  AttnArgs a{};
  a.q = q; a.q_sb = q_sb; a.q_st = q_st; a.q_sh = q_sh;
  a.k = k; a.k_sb = k_sb; a.k_st = k_st; a.k_sh = k_sh;
  a.v = v; a.v_sb = v_sb; a.v_st = v_st; a.v_sh = v_sh;
  a.indices = indices; a.index_bytes = index_bytes;
  a.positions = positions; a.pos_offset = position_offset;
  a.B = int(B); a.T = int(Tq); a.Hq = int(Hq); a.H = int(H); a.G = int(Hq / H);
  a.D = int(D); a.Dv = int(Dv); a.N = int(N); a.S = int(S); a.C = int(block_size);
  a.scale = scale; a.causal = causal ? 1 : 0;
  a.out = out; a.lse = lse;
  return attn_fwd(a, dtype, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace pisa {

// Workspace of the tensor-core backward: status word, fp32 dK / dV / dQ
// accumulators, the row dot products D = dO . O, then the request buckets of
// one token chunk (chunks keep request indices below 2^31).
struct BwdPlan {
  bool tc = false;
  int64_t TW = 4096, chunk = 0, NB = 0, RT = 0, num_buckets = 0, capacity = 0;
  int64_t status_off = 0, dk_off = 0, dv_off = 0, dvec_off = 0, dq_off = 0, counts_off = 0, cursors_off = 0,
          offsets_off = 0, misc_off = 0, owner_off = 0, req_off = 0, total = 0;
};

static BwdPlan plan_attn_bwd(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t Dv, int64_t N,
                             int64_t S, int64_t C, int dtype) {
  BwdPlan p;
  const int64_t G = Hq / H;
  // (head_dim 64: two 64 KB operand stages, two K/V buffers and the P / dS
  // tiles fill 193 KB of shared memory; 128-wide heads would not fit)
  p.tc = (dtype == PISA_BF16 || dtype == PISA_F16) && is_pow2(G) && G <= 32 && C == 64 && D == 64 && Dv == 64 &&
         S > 0 && S <= 64 && B * Tq * Hq >= 128;
  if (!p.tc) return p;
  const int64_t per_token = B * H * S;
  p.chunk = std::min<int64_t>(Tq, std::max<int64_t>(p.TW, ((int64_t(1) << 31) - 1) / per_token / p.TW * p.TW));
  if (p.chunk * per_token >= (int64_t(1) << 31)) { p.tc = false; return p; }
  p.NB = (N + C - 1) / C;
  p.RT = 128 / G;
  const int64_t nwin = (p.chunk + p.TW - 1) / p.TW;
  p.num_buckets = B * nwin * H * p.NB;
  p.capacity = (p.chunk * per_token + p.RT - 1) / p.RT + p.num_buckets;
  if (p.capacity * p.RT >= (int64_t(1) << 31)) { p.tc = false; return p; }
  int64_t off = 0;
  p.status_off = off; off += 256;
  p.dk_off = off; off += align_up(B * N * H * D * 4, 256);
  p.dv_off = off; off += align_up(B * N * H * Dv * 4, 256);
  p.dvec_off = off; off += align_up(B * Tq * Hq * 4, 256);
  p.dq_off = off; off += align_up(B * Tq * Hq * D * 4, 256);
  p.counts_off = off; off += align_up(p.num_buckets * 4, 256);
  p.cursors_off = off; off += align_up(p.num_buckets * 4, 256);
  p.offsets_off = off; off += align_up(p.num_buckets * 4, 256);
  p.misc_off = off; off += 256;
  p.owner_off = off; off += align_up(p.capacity * 4, 256);
  p.req_off = off; off += align_up(p.capacity * p.RT * 4, 256);
  p.total = off;
  return p;
}

}  // namespace pisa

extern "C" {

int64_t pisa_sparse_attn_bwd_tc_workspace_bytes(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D,
                                                int64_t Dv, int64_t N, int64_t S, int64_t block_size, int dtype) {
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || Hq % H || N <= 0 || block_size < 1) return 0;
  const BwdPlan p = plan_attn_bwd(B, Tq, Hq, H, D, Dv, N, S, block_size, dtype);
  return p.tc ? p.total : 0;
}

int64_t pisa_sparse_attn_bwd_workspace_bytes(int64_t B, int64_t Tq, int64_t Hq, int64_t H,
                                             int64_t D, int64_t Dv, int64_t N) {
  (void)Tq; (void)Hq;
  return align_up(B * N * H * D * 4, 256) + align_up(B * N * H * Dv * 4, 256);
}

int pisa_sparse_attn_bwd(const void* q, const void* k, const void* v, const void* out,
                         const void* dout, const float* lse, const void* indices, int index_bytes,
                         const int64_t* positions, int64_t position_offset, int dtype, int64_t B,
                         int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t Dv, int64_t N,
                         int64_t S, int64_t block_size, float scale, int causal, void* dq,
                         void* dk, void* dv, void* workspace, int64_t workspace_bytes,
                         pisa_stream_t stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype < PISA_F32 || dtype > PISA_F16) return fail(PISA_ERR_UNSUPPORTED, "CUDA attention supports FP16, BF16 and FP32");
  if (B <= 0 || Tq <= 0 || Hq <= 0 || H <= 0 || D <= 0 || Dv <= 0 || N <= 0) return fail(PISA_ERR_INVALID, "nonempty tensors are required");
  if (Hq % H) return fail(PISA_ERR_INVALID, "a whole number of query heads per KV head is required");
  if (index_bytes != 4 && index_bytes != 8) return fail(PISA_ERR_INVALID, "indices must be int32 or int64");
  if (D % 8 || Dv % 8 || D > 256 || Dv > 256) return fail(PISA_ERR_UNSUPPORTED, "head_dim must be a multiple of 8 and at most 256");
  if (!lse || !dq || !dk || !dv) return fail(PISA_ERR_INVALID, "lse, dq, dk and dv are required");
  const BwdPlan bp = plan_attn_bwd(B, Tq, Hq, H, D, Dv, N, S, block_size, dtype);
  if (bp.tc && workspace && workspace_bytes >= bp.total && out) {
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(dout) || !aligned16(out))
      return fail(PISA_ERR_UNSUPPORTED, "rows must be 16-byte aligned");
    char* ws = static_cast<char*>(workspace);
    cudaError_t e = cudaMemsetAsync(ws + bp.status_off, 0, 256, s);
    if (e != cudaSuccess) return fail_cuda(e, "status clear");
    AttnTcArgs a{};
    a.q = q; a.q_st = Hq * D; a.q_sh = D; a.q_sb = Tq * Hq * D;
    a.k = k; a.k_st = H * D; a.k_sh = D; a.k_sb = N * H * D;
    a.v = v; a.v_st = H * Dv; a.v_sh = Dv; a.v_sb = N * H * Dv;
    a.indices = indices; a.index_bytes = index_bytes;
    a.positions = positions; a.pos_offset = position_offset;
    a.B = int(B); a.T = int(Tq); a.Hq = int(Hq); a.H = int(H); a.G = int(Hq / H);
    a.D = int(D); a.Dp = int(D); a.Dv = int(Dv); a.Dvp = int(Dv);
    a.N = int(N); a.S = int(S); a.C = int(block_size); a.NB = int(bp.NB); a.TW = int(bp.TW);
    a.RT = int(bp.RT); a.chunk = int(bp.chunk);
    a.scale = scale; a.causal = causal ? 1 : 0; a.bf16 = dtype == PISA_BF16 ? 1 : 0;
    a.counts = reinterpret_cast<int32_t*>(ws + bp.counts_off);
    a.cursors = reinterpret_cast<int32_t*>(ws + bp.cursors_off);
    a.offsets = reinterpret_cast<int32_t*>(ws + bp.offsets_off);
    a.total_tiles = reinterpret_cast<int32_t*>(ws + bp.misc_off);
    a.status = reinterpret_cast<int*>(ws + bp.status_off);
    a.tile_owner = reinterpret_cast<int32_t*>(ws + bp.owner_off);
    a.tile_req = reinterpret_cast<int32_t*>(ws + bp.req_off);
    a.num_sms = num_sms();
    a.out = const_cast<void*>(out); a.dout = dout; a.lse_in = lse;
    a.dvec = reinterpret_cast<float*>(ws + bp.dvec_off);
    a.dq_acc = reinterpret_cast<float*>(ws + bp.dq_off);
    a.dk_acc = reinterpret_cast<float*>(ws + bp.dk_off);
    a.dv_acc = reinterpret_cast<float*>(ws + bp.dv_off);
    int rc = make_tensor_map(&a.tm_k, k, dtype, B, N, H, D, a.k_sb, a.k_st, a.k_sh, 1, uint32_t(block_size));
    if (rc == PISA_OK) rc = make_tensor_map(&a.tm_v, v, dtype, B, N, H, Dv, a.v_sb, a.v_st, a.v_sh, 1, uint32_t(block_size));
    if (rc) return rc;
    return attn_bwd_tc(a, dtype, dq, dk, dv, s);
  }
  const int64_t need = pisa_sparse_attn_bwd_workspace_bytes(B, Tq, Hq, H, D, Dv, N);
  if (!workspace || workspace_bytes < need) return fail(PISA_ERR_INVALID, "workspace too small");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(dout)) return fail(PISA_ERR_UNSUPPORTED, "rows must be 16-byte aligned");
  AttnArgs a{};
  a.q = q; a.k = k; a.v = v; a.o = out; a.dout = dout; a.lse_in = lse;
  a.indices = indices; a.index_bytes = index_bytes;
  a.positions = positions; a.pos_offset = position_offset;
  a.B = int(B); a.T = int(Tq); a.Hq = int(Hq); a.H = int(H); a.G = int(Hq / H);
  a.D = int(D); a.Dv = int(Dv); a.N = int(N); a.S = int(S); a.C = int(block_size);
  a.scale = scale; a.causal = causal ? 1 : 0;
  a.dq = dq;
  a.dk_acc = static_cast<float*>(workspace);
  a.dv_acc = reinterpret_cast<float*>(static_cast<char*>(workspace) + align_up(B * N * H * D * 4, 256));
  cudaError_t e = cudaMemsetAsync(workspace, 0, need, s);
  if (e != cudaSuccess) return fail_cuda(e, "workspace clear");
  return attn_bwd(a, dtype, dk, dv, s);
}

}  // extern "C"
