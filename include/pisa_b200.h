/*
 * pisa_b200.h -- C ABI of the B200 (sm_100a) PISA hot path.
 *
 * PISA's hot path is hierarchical log-sum-exp block selection over a
 * mean-pooled key pyramid followed by attention over the selected key blocks.
 * Each entry point below replaces one operator of the reference Python
 * package `pisa` (Aphelios-Tang/NlogN_PISA; paths relative to that project).
 *
 * Conventions
 *  - Tensors are [batch, tokens, heads, dim] with a contiguous last dim and
 *    16-byte aligned rows; strides are in ELEMENTS.  Key/value tensors may be
 *    strided in batch and tokens (the reference's PyramidCache views).
 *  - All pointers are device pointers unless marked "host".
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call is
 *    asynchronous on that stream and never synchronises the host.
 *  - The return value is a status code (PISA_OK or a PISA_ERR_*); nothing
 *    throws across the ABI.  pisa_last_error() describes the last failure of
 *    the calling thread.
 *  - Workspaces are caller-allocated; the *_workspace_bytes functions give the
 *    size.  The library makes no device allocation calls; the only device
 *    memory it holds is the fixed scratch of pisa_sparse_attn_bwd_noalloc.
 */
#ifndef PISA_B200_H
#define PISA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define PISA_OK 0
#define PISA_ERR_INVALID 1     /* argument violates the operator contract (Python: ValueError) */
#define PISA_ERR_UNSUPPORTED 2 /* outside the GPU kernels' envelope (Python: ValueError) */
#define PISA_ERR_CUDA 3        /* CUDA launch or runtime error (Python: RuntimeError) */
#define PISA_ERR_TIMEOUT 4     /* a bounded device-side wait expired (Python: RuntimeError) */

/* ---- element types (the reference's GPU path accepts fp16, bf16 and fp32) ---- */
#define PISA_F32 0
#define PISA_BF16 1
#define PISA_F16 2

/* ---- scoring methods (pisa1 = first order, pisa2 = second order, pisa = LSE) ---- */
#define PISA_METHOD_PISA1 0
#define PISA_METHOD_PISA2 1
#define PISA_METHOD_PISA 2

/* ---- routing schedules (top_k_pyramid.py:16-24 `routing_schedule`) ---- */
#define PISA_SCHEDULE_GROUPED 0 /* coarse router -> grouped leaf scoring -> final top-K */
#define PISA_SCHEDULE_FUSED 1   /* one kernel: coarse levels, leaf scoring and top-K */

typedef void *pisa_stream_t; /* cudaStream_t */

#if defined(__GNUC__)
#define PISA_API __attribute__((visibility("default")))
#else
#define PISA_API
#endif

/* Library version (major*10000 + minor*100 + patch). */
PISA_API int pisa_version(void);

/* Text of the last error raised on the calling host thread ("" if none). */
PISA_API const char *pisa_last_error(void);

/*
 * Mean of the valid tokens of every `size`-token block; a partial tail block
 * divides by its real count.  Accumulates in fp32 and rounds to `dtype`.
 * Replaces mean_pool / torch_mean_pool / pool_kernel
 *   (pisa/pisa/ops/compress/mean_pooling/mean_pooling.py:8-42,
 *    mean_pooling_torch.py:7-14, mean_pooling_triton.py:8-51).
 * out: [B, ceil(N/size), H, D] contiguous.
 */
PISA_API int pisa_mean_pool(const void *keys, int dtype, int64_t B, int64_t N, int64_t H, int64_t D,
                   int64_t key_sb, int64_t key_st, int64_t key_sh, int64_t size, void *out,
                   pisa_stream_t stream);

/*
 * Key pyramid: level 0 = mean_pool(keys, block_size), level l+1 =
 * mean_pool(level l, branching), for levels 0..num_levels-1.  All levels go
 * to one storage [B, total, H, D] (node stride H*D, batch stride storage_sb)
 * at node offsets level_offsets[l] (host array) -- the PyramidCache layout
 * (xmixers/xmixers/utils/attention_cache.py:102-118).
 * Replaces build_pyramid (mean_pooling.py:45-52) and the level concatenation
 * of select_cuda (top_k_pyramid_triton.py:348-359).  branching 2 is the
 * reference; 4 is this library's extension.
 */
PISA_API int pisa_build_pyramid(const void *keys, int dtype, int64_t B, int64_t N, int64_t H, int64_t D,
                       int64_t key_sb, int64_t key_st, int64_t key_sh, int64_t block_size,
                       int64_t branching, int64_t num_levels, void *storage, int64_t storage_sb,
                       const int64_t *level_offsets, pisa_stream_t stream);

/*
 * Recompute the pyramid nodes that depend on key tokens [first_token, N):
 * the leaves they touch and those leaves' ancestors, as
 * PyramidCache.append (attention_cache.py:120-140) does after appending keys.
 * Levels 0..num_levels-1 must already hold the pyramid of keys[:, :first_token].
 */
PISA_API int pisa_pyramid_update(const void *keys, int dtype, int64_t B, int64_t N, int64_t H, int64_t D,
                        int64_t key_sb, int64_t key_st, int64_t key_sh, int64_t block_size,
                        int64_t branching, int64_t num_levels, void *storage, int64_t storage_sb,
                        const int64_t *level_offsets, int64_t first_token, pisa_stream_t stream);

/*
 * Block selection: ids [B, Tq, H, topk] int64 in network-rank order, -1
 * padded.  Replaces select_blocks/_select_unpacked -> select_cuda
 *   (pisa/pisa/ops/flash_sparse_attn/top_k_pyramid/top_k_pyramid.py:11-122,
 *    top_k_pyramid_triton.py:311-447) with the equations of the torch
 *    reference (top_k_pyramid_torch.py:6-177).
 * q: [B,Tq,Hq,D]; keys: [B,N,H,D]; Hq = G*H.
 * summary: pyramid storage as written by pisa_build_pyramid with levels
 *   0..top (level_offsets/level_sizes: host arrays of num_levels >= top+1
 *   entries), or NULL to build it inside `workspace`.
 * positions: device int64 [B,Tq] absolute query positions, or NULL for
 *   position = position_offset + token (validation.py:38-47).
 * top, first_width: routing geometry (top_k_pyramid_torch.py:124-133).
 * schedule: PISA_SCHEDULE_GROUPED or PISA_SCHEDULE_FUSED.
 * Constraints (as the reference's GPU path, top_k_pyramid_triton.py:327-335):
 *   block_size a power of two >= 16, topk in {8,16,32,64}, D % 8 == 0,
 *   D <= 256, branching in {2,4}, G <= 32.
 */
PISA_API int pisa_select_blocks(const void *q, int64_t q_sb, int64_t q_st, int64_t q_sh, const void *keys,
                       int64_t key_sb, int64_t key_st, int64_t key_sh, const void *summary,
                       int64_t summary_sb, const int64_t *level_offsets,
                       const int64_t *level_sizes, int64_t num_levels, const int64_t *positions,
                       int64_t position_offset, int dtype, int64_t B, int64_t Tq, int64_t Hq,
                       int64_t H, int64_t D, int64_t N, int method, int64_t block_size,
                       int64_t branching, int64_t topk, int force_first, int64_t force_recent,
                       int64_t top, int64_t first_width, int schedule, int64_t *out_ids,
                       void *workspace, int64_t workspace_bytes, pisa_stream_t stream);

/*
 * Workspace bytes for pisa_select_blocks with the same shapes and options
 * (build_summary != 0 when it will be called with summary == NULL).
 */
PISA_API int64_t pisa_select_workspace_bytes(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D,
                                             int64_t N, int dtype, int method, int64_t block_size,
                                             int64_t branching, int64_t topk, int64_t top,
                                             int64_t first_width, int schedule, int build_summary);

/*
 * How pisa_select_blocks will score the coarse levels for these shapes
 * (profiling aid; no counterpart in the reference): bit l of the low 32 bits
 * is set when level l is scored densely (every node for every row, on the
 * tensor cores), bit l of the high 32 bits when the router scores level l
 * per row over the row's own candidates.  Other levels need no scores (the
 * all-fit shortcut) or are scored by the per-item router.  -1 on bad shapes.
 */
PISA_API int64_t pisa_select_level_plan(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t N,
                                        int dtype, int method, int64_t block_size, int64_t branching,
                                        int64_t topk, int64_t top, int64_t first_width, int schedule);

/*
 * Leaf scores of arbitrary candidate lists.  Replaces grouped_leaf_scores
 * (pisa/pisa/ops/flash_sparse_attn/top_k_pyramid/leaf_triton.py:144-232)
 * with its masks (leaf_scoreable_mask, leaf_triton.py:23-60).
 * candidates: [B,Tq,H,W] int32 (cand_bytes 4) or int64 (8), contiguous.
 * out_scores: [B,Tq,H,W] fp32 in candidate order: the score summed over the
 *   G query heads (pisa: LSE over the block's keys; pisa2: scale*mean +
 *   0.5*scale^2*var of the logits; pisa1: q . leaf mean, scale 1), or -inf
 *   for an id outside [0, ceil(N/block_size)) and, when `positions` ([B,Tq]
 *   int64) is given, for ids past the query's position, forced ids (block 0
 *   with force_first, the force_recent most recent blocks) and every id of a
 *   row whose valid ids all fit in `topk` (pisa / pisa2).
 * leaf_means: [B, blocks, H, D] (node stride H*D, batch stride means_sb) for
 *   pisa1, or NULL to pool them from `keys` inside the workspace.
 * workspace: pisa_leaf_scores_workspace_bytes(...) bytes (have_means != 0
 *   when leaf_means will be passed).
 */
PISA_API int pisa_leaf_scores(const void *q, int64_t q_sb, int64_t q_st, int64_t q_sh, const void *keys,
                              int64_t key_sb, int64_t key_st, int64_t key_sh, const void *leaf_means,
                              int64_t means_sb, const void *candidates, int cand_bytes,
                              const int64_t *positions, int dtype, int64_t B, int64_t Tq, int64_t Hq,
                              int64_t H, int64_t D, int64_t N, int64_t W, int method, int64_t block_size,
                              int64_t topk, int force_first, int64_t force_recent, float *out_scores,
                              void *workspace, int64_t workspace_bytes, pisa_stream_t stream);

PISA_API int64_t pisa_leaf_scores_workspace_bytes(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D,
                                                  int64_t N, int64_t W, int dtype, int method,
                                                  int64_t block_size, int have_means);

/*
 * Flat BSA block selection, the reference's comparator for PISA routing.
 * Replaces bsa_fn / bsa_select (pisa/pisa/ops/flash_sparse_attn/bsa/bsa.py:9-52,
 * bsa_torch.py:63-106; GPU form bsa_triton.py:12-114), which select_blocks
 * reaches with method="bsa" (top_k_pyramid.py:60-63).  Per (query token, KV
 * head): each query head, scaled by D^-0.5 and rounded to `dtype`, scores
 * the leaf means of the complete blocks; blocks before the current one get
 * exp(logit - LSE of the complete blocks' logits), required blocks (block 0
 * with force_first, the force_recent most recent) get 1; the values are
 * summed over the G query heads and the best `topk` are kept by the
 * reference's streaming comparison network (tiles of pow2(max(block_size,
 * 2*topk)) blocks, bsa_torch.py:9-60), ids past the current block being -1.
 * out_ids: [B,Tq,H,topk] int64 in network-rank order.
 * leaf_means: [B, ceil(N/block_size), H, D] (node stride H*D, batch stride
 *   means_sb), or NULL to pool them from `keys` inside `workspace`
 *   (pisa_bsa_workspace_bytes(..., have_means=0) bytes).
 * positions: device int64 [B,Tq], or NULL for position_offset + token.  With
 *   `positions` the caller checks that topk holds every row's required blocks
 *   (the Python mirror does); without, the entry point checks it.
 * Constraints: G <= 16, D % 8 == 0 (fp32: D % 4) and D <= 256,
 *   max(block_size, 2*topk) <= 256.
 */
PISA_API int pisa_bsa_select(const void *q, int64_t q_sb, int64_t q_st, int64_t q_sh, const void *keys,
                             int64_t key_sb, int64_t key_st, int64_t key_sh, const void *leaf_means,
                             int64_t means_sb, const int64_t *positions, int64_t position_offset, int dtype,
                             int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t N,
                             int64_t block_size, int64_t topk, int force_first, int64_t force_recent,
                             int64_t *out_ids, void *workspace, int64_t workspace_bytes, pisa_stream_t stream);

/* Workspace bytes of pisa_bsa_select (0 when leaf means are passed; -1 on bad shapes). */
PISA_API int64_t pisa_bsa_workspace_bytes(int64_t B, int64_t N, int64_t H, int64_t D, int dtype,
                                          int64_t block_size, int have_means);

/*
 * Attention over selected key blocks with one softmax over their union
 * (causal inside blocks), forward.  Replaces sparse_attention's CUDA branch
 * (pisa/pisa/ops/flash_sparse_attn/sparse_attn/sparse_attn.py:10-61 ->
 * sparse_attn_fla.py:22-71 / decode_triton.py:82-115) with the semantics of
 * sparse_attn_torch.py:6-35.
 * indices: [B,Tq,H,S] int32 (index_bytes 4) or int64 (8), contiguous; ids < 0
 *   or past the keys are skipped; duplicates count once per occurrence.
 * out: [B,Tq,Hq,Dv] in dtype (contiguous); lse: [B,Tq,Hq] fp32 natural-log
 *   log-sum-exp of the scaled logits (-inf for rows without a visible key,
 *   whose output is 0).  lse may be NULL.
 * workspace: pisa_sparse_attn_fwd_workspace_bytes(...) bytes enable the
 *   block-bucketed tensor-core path for fp16/bf16 prefill; with NULL (or when
 *   that size is 0, as it is below 64 query rows per sequence, e.g. batched
 *   decode) the per-query gather kernels run.
 */
PISA_API int pisa_sparse_attn_fwd(const void *q, int64_t q_sb, int64_t q_st, int64_t q_sh, const void *k,
                         int64_t k_sb, int64_t k_st, int64_t k_sh, const void *v, int64_t v_sb,
                         int64_t v_st, int64_t v_sh, const void *indices, int index_bytes,
                         const int64_t *positions, int64_t position_offset, int dtype, int64_t B,
                         int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t Dv, int64_t N,
                         int64_t S, int64_t block_size, float scale, int causal, void *out,
                         float *lse, void *workspace, int64_t workspace_bytes,
                         pisa_stream_t stream);

/*
 * Fused single-token decode step: block selection and attention over the
 * selected blocks in one launch (one CTA per (sequence, token, KV head)).
 * Replaces the reference's decode pair select_blocks(routing_schedule=
 * "fused") -> top_k_pyramid_triton.py:125-276 (leaf scoring fused into the
 * router) followed by decode_attention (decode/decode_triton.py:8-115).
 * Selection arguments as pisa_select_blocks (the pyramid `summary` with its
 * level tables is required: the caller's PyramidCache); attention as
 * pisa_sparse_attn_fwd with causal masking at each query's position.
 * values: [B,N,H,Dv] (element strides); Dv in {64, 128, 256}; G <= 16 and
 *   G*Dv <= 2048.
 * out_ids [B,Tq,H,topk] int64 (network-rank order, -1 padded), out
 * [B,Tq,Hq,Dv] in dtype, lse [B,Tq,Hq] fp32 or NULL.  No workspace.
 */
PISA_API int pisa_decode_select_attend(const void *q, int64_t q_sb, int64_t q_st, int64_t q_sh, const void *keys,
                                       int64_t key_sb, int64_t key_st, int64_t key_sh, const void *values,
                                       int64_t value_sb, int64_t value_st, int64_t value_sh, const void *summary,
                                       int64_t summary_sb, const int64_t *level_offsets, const int64_t *level_sizes,
                                       int64_t num_levels, const int64_t *positions, int64_t position_offset,
                                       int dtype, int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D,
                                       int64_t Dv, int64_t N, int method, int64_t block_size, int64_t branching,
                                       int64_t topk, int force_first, int64_t force_recent, int64_t top,
                                       int64_t first_width, float scale, int64_t *out_ids, void *out, float *lse,
                                       pisa_stream_t stream);

/* Workspace bytes of pisa_sparse_attn_fwd for these shapes (0: none needed). */
PISA_API int64_t pisa_sparse_attn_fwd_workspace_bytes(int64_t B, int64_t Tq, int64_t Hq, int64_t H,
                                                      int64_t D, int64_t Dv, int64_t N, int64_t S,
                                                      int64_t block_size, int dtype);

/*
 * Backward of pisa_sparse_attn_fwd: dq [B,Tq,Hq,D], dk/dv [B,N,H,D|Dv] in
 * dtype, contiguous.  Gradient of the reference's autograd through
 * sparse_attn_torch.py:6-35.  q/k/v/out/dout/dq/dk/dv contiguous.
 * workspace: pisa_sparse_attn_bwd_tc_workspace_bytes(...) bytes (when that
 *   is nonzero: fp16/bf16, block size 64, D = Dv = 64) run the
 *   tensor-core backward over the forward's request buckets, with its status
 *   word at workspace offset 0; otherwise (or with a smaller workspace of at
 *   least pisa_sparse_attn_bwd_workspace_bytes(...) bytes) the per-query
 *   gather kernels run.  The reference's GPU backward is fla-core's
 *   ParallelNSAFunction (sparse_attn_fla.py:59-68).
 */
PISA_API int pisa_sparse_attn_bwd(const void *q, const void *k, const void *v, const void *out,
                         const void *dout, const float *lse, const void *indices, int index_bytes,
                         const int64_t *positions, int64_t position_offset, int dtype, int64_t B,
                         int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t Dv, int64_t N,
                         int64_t S, int64_t block_size, float scale, int causal, void *dq,
                         void *dk, void *dv, void *workspace, int64_t workspace_bytes,
                         pisa_stream_t stream);

PISA_API int64_t pisa_sparse_attn_bwd_workspace_bytes(int64_t B, int64_t Tq, int64_t Hq, int64_t H,
                                             int64_t D, int64_t Dv, int64_t N);

/* Workspace bytes of the tensor-core backward for these shapes (0: not eligible). */
PISA_API int64_t pisa_sparse_attn_bwd_tc_workspace_bytes(int64_t B, int64_t Tq, int64_t Hq, int64_t H, int64_t D,
                                                         int64_t Dv, int64_t N, int64_t S, int64_t block_size,
                                                         int dtype);

/*
 * pisa_sparse_attn_bwd without a caller workspace, for callers that cannot
 * allocate device memory (a host runtime bound to this C ABI that owns only
 * the tensors it passes, or a framework whose device memory is planned in
 * advance).  No counterpart in the reference.  The fp32 dK/dV accumulators
 * live in a fixed device array inside the library:
 * pisa_sparse_attn_bwd_noalloc_max_bytes() bytes (32 MiB) per GPU, held until
 * the process exits.  Shapes whose pisa_sparse_attn_bwd_workspace_bytes(...)
 * exceeds that return PISA_ERR_UNSUPPORTED.  The first call on a device looks
 * up the array's device address (set-up); under lazy module loading (the CUDA
 * default) that is also when the 32 MiB are reserved on the device, so make
 * that first call before fixing a memory plan and before any stream capture.
 * The current device must be the device of `stream` (PISA_ERR_INVALID
 * otherwise).  Every call uses the same array and clears it on `stream`
 * first, so calls that overlap on the GPU (other streams, other host
 * threads) race.  Arguments as pisa_sparse_attn_bwd.  Allocates nothing.
 */
PISA_API int pisa_sparse_attn_bwd_noalloc(const void *q, const void *k, const void *v, const void *out,
                                          const void *dout, const float *lse, const void *indices,
                                          int index_bytes, const int64_t *positions,
                                          int64_t position_offset, int dtype, int64_t B, int64_t Tq,
                                          int64_t Hq, int64_t H, int64_t D, int64_t Dv, int64_t N,
                                          int64_t S, int64_t block_size, float scale, int causal,
                                          void *dq, void *dk, void *dv, pisa_stream_t stream);

/* Size of the fixed scratch of pisa_sparse_attn_bwd_noalloc, in bytes. */
PISA_API int64_t pisa_sparse_attn_bwd_noalloc_max_bytes(void);

/*
 * Split-half rotary position encoding of the token mixer's q and k before
 * selection.  Replaces rotary_fn / rotary_torch
 * (pisa/pisa/ops/lrpe/rotary.py:9-17, rotary_torch.py:5-9) as called by
 * xmixers' RotaryEmbedding (xmixers/xmixers/modules/pes/lrpe.py:29-33).
 * x, out: [B,T,H,D] (element strides; out may equal x); frequency: D/2 fp32;
 * positions: int64 with batch stride positions_sb (0 broadcasts one row) and
 * unit token stride, or NULL for position_offset + token.
 */
PISA_API int pisa_rotary(const void *x, int64_t x_sb, int64_t x_st, int64_t x_sh, void *out, int64_t out_sb,
                         int64_t out_st, int64_t out_sh, const int64_t *positions, int64_t positions_sb,
                         int64_t position_offset, const float *frequency, int dtype, int64_t B, int64_t T,
                         int64_t H, int64_t D, pisa_stream_t stream);

/* ---- device status (no counterpart in the reference, whose Triton kernels never wait) ----
 * Every kernel that waits on another part of the GPU waits a bounded number
 * of tries.  A wait that expires records PISA_ERR_TIMEOUT in the 4-byte
 * status word at byte offset 0 of the call's workspace (pisa_select_blocks,
 * pisa_leaf_scores, and pisa_sparse_attn_fwd when it takes the tensor-core
 * path); the entry point clears that word on `stream` before its kernels run.
 *
 * pisa_workspace_status copies the word back and synchronises `stream`:
 * PISA_OK, or PISA_ERR_TIMEOUT (the call's outputs are not valid). */
PISA_API int pisa_workspace_status(const void *workspace, pisa_stream_t stream);

/* Exercises the timeout path without touching any operand: one warp waits up
 * to `max_tries` tries on an mbarrier that it arrives on first (arrive != 0)
 * or that nothing ever arrives on (arrive == 0), and records the outcome in
 * workspace[0..3] (256 bytes, cleared first) for pisa_workspace_status. */
PISA_API int pisa_wait_selftest(int arrive, int64_t max_tries, void *workspace, int64_t workspace_bytes,
                                pisa_stream_t stream);

/* Accuracy check of the leaf epilogue's two exponential forms (no
 * counterpart in the reference): poly[i] = the FMA-pipe polynomial 2^x[i],
 * mufu[i] = ex2.approx.ftz.f32 of x[i]; device arrays of n floats. */
PISA_API int pisa_ex2_selftest(const float *x, float *poly, float *mufu, int64_t n, pisa_stream_t stream);

/* ---- per-kernel device timing (profiling aid; the reference has no counterpart) ----
 * With timing on, the library records a pair of CUDA events on the launch
 * stream around every launch of the kernels below.  Reading returns the summed
 * device time and the launch count since the previous read of that kernel and
 * resets them; it waits for the recorded events.  Process-wide; calls from
 * several host threads are serialised by a lock. */
#define PISA_KERNEL_LEAF_TILES 0    /* tensor-core leaf scoring tiles */
#define PISA_KERNEL_ATTN_TILES 1    /* tensor-core attention tiles */
#define PISA_KERNEL_ATTN_COMBINE 2  /* merge of the attention block partials */
#define PISA_KERNEL_PYRAMID 3       /* key pyramid build (all its launches) */
#define PISA_KERNEL_DENSE_LEVEL 4   /* tensor-core scoring of whole coarse levels */
#define PISA_KERNEL_ROUTER 5        /* coarse-to-fine router (warp-per-row or per-item form) */
#define PISA_KERNEL_LEAF_FINAL 6    /* final top-K over the leaf candidates */
#define PISA_KERNEL_BSA 7           /* flat BSA selection (pisa_bsa_select) */
#define PISA_KERNEL_COUNT 8

/* Kernels this library has launched in this process so far. */
PISA_API int64_t pisa_launch_count(void);

/* enable = 1 starts recording, 0 stops it (recorded launches stay readable). */
PISA_API int pisa_kernel_timing(int enable);

/* Device milliseconds and launches of `kernel` since its last read. */
PISA_API int pisa_kernel_time(int kernel, double *total_ms, int64_t *launches);

#ifdef __cplusplus
}
#endif

#endif /* PISA_B200_H */
