// Internal declarations shared by the translation units of libpisa_b200.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "pisa_b200.h"

namespace pisa {

// Records `msg` as the calling thread's last error and returns `code`.
int fail(int code, const char* msg);
int fail_cuda(cudaError_t err, const char* where);

// 4-D TMA map over a [B, T, H, D] view (element strides sb, st, sh; 16-byte
// aligned rows) with 128-byte swizzle and a box of {64, box_h, box_t, 1}
// elements; out-of-range elements read as zero.
int make_tensor_map(CUtensorMap* map, const void* base, int dtype, int64_t B, int64_t T, int64_t H,
                    int64_t D, int64_t sb, int64_t st, int64_t sh, uint32_t box_h, uint32_t box_t);

// Scope guard that brackets one kernel launch with timing events when
// per-kernel timing is on (timing.cu); a no-op otherwise.
class TimedLaunch {
 public:
  TimedLaunch(int kernel, cudaStream_t stream);
  ~TimedLaunch();
  TimedLaunch(const TimedLaunch&) = delete;
  TimedLaunch& operator=(const TimedLaunch&) = delete;

 private:
  int kernel_, slot_;
  cudaStream_t stream_;
};

// Counts one launch of this library (pisa_launch_count) and reports a failed launch.
void count_launch();

#define PISA_CHECK_LAUNCH()                                        \
  do {                                                             \
    ::pisa::count_launch();                                        \
    cudaError_t _e = cudaGetLastError();                           \
    if (_e != cudaSuccess) return ::pisa::fail_cuda(_e, __func__); \
  } while (0)

struct LevelTable {
  int64_t offset[kMaxLevels];
  int32_t size[kMaxLevels];
};

int build_pyramid(const void* keys, int dtype, int64_t B, int64_t N, int64_t H, int64_t D,
                  int64_t sb, int64_t st, int64_t sh, int64_t C, int64_t br, int64_t levels,
                  void* storage, int64_t ssb, const int64_t* offs, int64_t first_token,
                  cudaStream_t stream);

struct RouteArgs {
  const void* q;
  int64_t q_sb, q_st, q_sh;
  const void* keys;
  int64_t k_sb, k_st, k_sh;
  const void* summary;
  int64_t s_sb;
  LevelTable levels;
  const int64_t* positions;
  int64_t pos_offset;
  int B, T, H, G, D, N;
  int C, K, br, method, top, first_width, force_first, force_recent;
  float scale, c2;
  int64_t* out_ids;     // [B,T,H,K] when the leaf level is scored here
  int32_t* candidates;  // [B,T,H,W0] when only the coarse levels run here
  uint8_t* flags;       // [B,T,H,W0] leaf masks: bit0 valid, bit1 forced, bit2 scoreable
  int W0;
  int coarse_only;
  int t_begin, t_count;  // token range routed by this launch
  const float* dense;   // precomputed level scores, rows local to the range
  int64_t dense_stride;
  int dense_off[kMaxLevels];  // per level offset in a dense row, -1 = compute here
  // bit l: level l is scored by the warp router itself, one warp per row,
  // with mma.sync over the row's own candidate children (router.cu)
  uint32_t row_levels;
  FastDiv fbr, fH, ftc;       // branching, KV heads, t_count (set by the launcher)
  // grouped leaf buckets: when set, the warp router counts each active
  // (row, family) request into fam_counts (bucket = (b, window, head, family))
  int32_t* fam_counts;
  int NP, nwin, TW;
  // fused decode (per-item router only): after the leaf top-K the same CTA
  // attends over the K selected blocks and writes out [B,T,Hq,Dv] and lse
  int attend;
  const void* values;
  int64_t v_sb, v_st, v_sh;
  int Dv;
  float attn_scale;
  void* out;
  float* lse;
};

// Routes the rows of a.t_begin .. a.t_begin + a.t_count; `counted` (may be
// null) reports whether the family buckets were counted on the way.

int route(const RouteArgs& a, int dtype, cudaStream_t stream, bool* counted = nullptr);

// Grouped leaf scoring: requests (row, family) bucketed by (batch, token
// window, KV head, level-1 survivor), scored on the tensor cores, then the
// final top-K.  Arrays are workspace slices laid out by the C entry point.
struct GroupArgs {
  CUtensorMap tm_q;   // q [B,T,Hq,D], box {64, G, 1, 1}
  CUtensorMap tm_k;   // keys [B,N,H,D], box {64, 1, b*C, 1}
  const void* q;
  int64_t q_sb, q_st, q_sh;
  const void* keys;
  int64_t k_sb, k_st, k_sh;
  const int64_t* positions;
  int64_t pos_offset;
  int B, T, H, G, D, Dp, N, C, K, br, W0, NF, NP, nwin, TW, RT;
  int method, bf16;
  float scale, c2;
  const int32_t* cand;
  const uint8_t* flags;
  float* scores;
  int32_t* counts;
  int32_t* cursors;
  int32_t* offsets;
  int64_t num_buckets;
  const int32_t* tile_owner;
  const int32_t* tile_req;
  const int32_t* total_tiles;
  int32_t* tile_owner_w;
  int32_t* tile_req_w;
  int32_t* total_tiles_w;
  int64_t tile_capacity;
  int tiles_per_cta;
  int tmem_cols;
  int num_sms;
  int counts_ready;   // bucket counts already produced by the router
  // divisors of the index decodes (set by the launcher from the fields above)
  FastDiv fNF, fH, fT, fNP, fTW, fRT, fbr, fnwin;
  int64_t* out_ids;
  int* status;
  int skip_final;     // 1: stop after the tile kernel (scores only, no top-K)
  int kbufs;          // key buffers of the tile kernel (set by grouped_leaf): 2 pairs with 2 query stages
};

int grouped_leaf(const GroupArgs& g, int dtype, cudaStream_t stream);

// Masks, int32 ids and -inf fills of the standalone leaf scorer (leafscore.cu).
struct LeafPrepArgs {
  const void* cand;            // [B, T, H, W] int32 or int64, contiguous
  int cand_bytes;
  const int64_t* positions;    // [B, T] or null (no causal / forced masks)
  int B, T, H, W, C, K, method, force_first, force_recent;
  int64_t blocks;
  int32_t* cand_out;           // [B, T, H, W]
  uint8_t* flags;              // bit0 valid, bit1 forced, bit2 scoreable
  float* scores;               // [B, T, H, W]: -inf written for unscored slots
};

int leaf_prepare(const LeafPrepArgs& p, cudaStream_t stream);

// SIMT scores of the scoreable slots (any dtype, all three methods); `means`
// ([B, blocks, H, D], node stride H*D, batch stride means_sb) for pisa1.
int leaf_scores_simt(const RouteArgs& a, const int32_t* cand, const uint8_t* flags, int W, float* scores,
                     const void* means, int64_t means_sb, int dtype, cudaStream_t stream);

// Dense scoring of every node of one coarse level (see dense.cu).
struct DenseArgs {
  CUtensorMap tm_q;          // q [B,T,Hq,D], box {64, G, 128/G tokens, 1}
  CUtensorMap tm_x;          // pyramid storage [B, total, H, D], box {64, 1, 256, 1}
  const void* q;
  int64_t q_sb, q_st, q_sh;
  const void* summary;       // pyramid storage [B, total, H, D]
  int64_t s_sb;
  int64_t child_off;         // node offset of the child level in the storage
  int n_child;               // children at the child level
  int support;               // children per node (b), or 1 for pisa1 (node itself)
  int64_t span;              // tokens covered by one node of the scored level
  const int64_t* positions;
  int64_t pos_offset;
  int B, T, H, G, D, Dp, method, bf16;
  int t_begin, t_count;      // token range scored by this launch
  float scale, c2;
  float* scores;             // [B, t_count, H, row_stride] (rows local to the range)
  int64_t row_stride, out_off;
  int* status;
};

int dense_level(const DenseArgs& a, int dtype, cudaStream_t stream);

struct AttnArgs {
  const void* q;
  int64_t q_sb, q_st, q_sh;
  const void* k;
  int64_t k_sb, k_st, k_sh;
  const void* v;
  int64_t v_sb, v_st, v_sh;
  const void* indices;
  int index_bytes;
  const int64_t* positions;
  int64_t pos_offset;
  int B, T, Hq, H, G, D, Dv, N, S, C;
  float scale;
  int causal;
  void* out;
  float* lse;
  // backward
  const void* o;
  const void* dout;
  const float* lse_in;
  void* dq;
  float* dk_acc;
  float* dv_acc;
};

int attn_fwd(const AttnArgs& a, int dtype, cudaStream_t stream);

// Bucketed tensor-core attention forward (prefill): see attn_tc.cu.
struct AttnTcArgs {
  CUtensorMap tm_q;   // q [B,T,Hq,D], box {64, G, 1, 1}
  CUtensorMap tm_k;   // k [B,N,H,D], box {64, 1, C, 1}
  CUtensorMap tm_v;   // v [B,N,H,Dv], box {64, 1, C, 1}
  const void* q;
  int64_t q_sb, q_st, q_sh;
  const void* k;
  int64_t k_sb, k_st, k_sh;
  const void* v;
  int64_t v_sb, v_st, v_sh;
  const void* indices;
  int index_bytes;
  const int64_t* positions;
  int64_t pos_offset;
  int B, T, Hq, H, G, D, Dp, Dv, Dvp, N, S, C, NB, TW, RT;
  int chunk, t0, tlen, nwin;
  float scale;
  int causal, bf16;
  int32_t* counts;
  int32_t* cursors;
  int32_t* offsets;
  int64_t num_buckets;
  int32_t* tile_owner;
  int32_t* tile_req;
  int32_t* total_tiles;
  int64_t capacity;
  int tiles_per_cta, tmem_cols, sp_cols, o_cols, nacc, nstages, num_sms;
  // divisors of the index decodes (set by the launcher from the fields above)
  FastDiv fS, fH, fHq, fNB, fTW, fRT, ftlen, fnwin;
  void* part_o;     // [request * G + head][Dv] block partials (query-major, chunk-local requests)
  float* part_ml;   // [request * G + head] (m, l)
  void* out;
  float* lse;
  int* status;
  // backward (attn_bwd_tc.cu): contiguous dout, the forward's lse, the row
  // dot products D = dout . out, and fp32 gradient accumulators
  const void* dout;
  const float* lse_in;
  float* dvec;        // [B, T, Hq]
  float* dq_acc;      // [B, T, Hq, D]
  float* dk_acc;      // [B, N, H, D]
  float* dv_acc;      // [B, N, H, Dv]
};

int attn_fwd_tc(const AttnTcArgs& a, int dtype, cudaStream_t stream);

// Buckets the requests of token chunk [t0, t0 + chunk) of `a` (count, scan,
// scatter into tile_owner / tile_req); sets the chunk fields of `a`.
int attn_bucket_chunk(AttnTcArgs& a, int t0, cudaStream_t stream);

// Tensor-core backward over the same buckets (attn_bwd_tc.cu); writes dq, dk, dv.
int attn_bwd_tc(const AttnTcArgs& a, int dtype, void* dq, void* dk, void* dv, cudaStream_t stream);
int attn_bwd(const AttnArgs& a, int dtype, void* dk, void* dv, cudaStream_t stream);

}  // namespace pisa
