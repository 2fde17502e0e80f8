// K4 (tensor-core form): attention over selected blocks, forward, for prefill.
//
// Semantics as sparse_attention_torch (pisa/pisa/ops/flash_sparse_attn/
// sparse_attn/sparse_attn_torch.py:6-35): one softmax over the union of the
// selected blocks' keys, causal inside blocks, scale * q.k logits.
//
// Selection gives every query its own K blocks, so queries that share a tile
// of keys are found by bucketing: requests (row, slot) with a visible block
// are grouped by (batch, token window, KV head, block id).  One tile = the
// block's C keys and values (staged once per run of tiles of the bucket)
// against up to 128/G requests (their G query-head rows gathered once):
//   MMA 1  S = Q K^T           (M=128 rows, N=C, K=head_dim) -> TMEM
//   softmax per row in registers (causal mask by the row's own position),
//          P = exp(S - m) rounded to the input type, stored back to TMEM
//   MMA 2  O = P V             (A = P from TMEM, B = V MN-major) -> TMEM
// and writes the block-local partial (m, l, O / l) of every row.  A combine
// pass merges the S partials of each query head into the output and its
// log-sum-exp.  Moving each query row to its blocks once (instead of every
// block to every query) cuts the L2->SM traffic by the bucket reuse factor;
// the token window keeps the gathered query rows L2-resident.  Token chunks
// bound the partial buffer.
#include <algorithm>
#include <type_traits>

#include "bucket.cuh"
#include "internal.h"
#include "tc.cuh"

namespace pisa {

namespace {

constexpr int kThreads = 128;

__device__ __forceinline__ int64_t index_at(const void* p, int bytes, int64_t i) {
  return bytes == 4 ? int64_t(static_cast<const int32_t*>(p)[i]) : static_cast<const int64_t*>(p)[i];
}

// Chunk-local request lr = ((b * tlen + tl) * H + h) * S + s.
struct Req {
  int b, tl, h, s;
};
__device__ __forceinline__ Req decode_req(int64_t lr, const AttnTcArgs& a) {
  Req r;
  r.s = int(lr % a.S);
  int64_t row = lr / a.S;
  r.h = int(row % a.H);
  row /= a.H;
  r.tl = int(row % a.tlen);
  r.b = int(row / a.tlen);
  return r;
}

__device__ __forceinline__ int64_t position_of(const AttnTcArgs& a, int b, int t) {
  return a.positions ? a.positions[int64_t(b) * a.T + t] : a.pos_offset + t;
}

// Visible block id of a request, or -1.
__device__ __forceinline__ int64_t visible_block(const AttnTcArgs& a, int b, int t, int h, int s) {
  const int64_t id = index_at(a.indices, a.index_bytes, ((int64_t(b) * a.T + t) * a.H + h) * a.S + s);
  if (id < 0 || id * a.C >= a.N) return -1;
  if (a.causal && id * a.C > position_of(a, b, t)) return -1;
  return id;
}

__device__ __forceinline__ int64_t bucket_of(const AttnTcArgs& a, const Req& r, int64_t id) {
  return ((int64_t(r.b) * a.nwin + r.tl / a.TW) * a.H + r.h) * a.NB + id;
}

__global__ void attn_count_kernel(const AttnTcArgs a) {
  const int64_t lr = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (lr >= int64_t(a.B) * a.tlen * a.H * a.S) return;
  const Req r = decode_req(lr, a);
  const int64_t id = visible_block(a, r.b, a.t0 + r.tl, r.h, r.s);
  if (id < 0) return;
  atomicAdd(a.counts + bucket_of(a, r, id), 1);
}

__global__ void attn_scatter_kernel(const AttnTcArgs a) {
  const int64_t lr = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (lr >= int64_t(a.B) * a.tlen * a.H * a.S) return;
  const Req r = decode_req(lr, a);
  const int64_t id = visible_block(a, r.b, a.t0 + r.tl, r.h, r.s);
  if (id < 0) return;
  const int64_t bucket = bucket_of(a, r, id);
  const int pos = atomicAdd(a.cursors + bucket, 1);
  const int64_t tile = a.offsets[bucket] + pos / a.RT;
  a.tile_req[tile * a.RT + pos % a.RT] = int32_t(lr);
  if (pos % a.RT == 0) a.tile_owner[tile] = int32_t(bucket);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) attn_tc_kernel(const AttnTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int qch = a.Dp / 64, vch = a.Dvp / 64;
  uint8_t* Qs = smem;                        // [qch][128 rows][128 B]
  uint8_t* Ks = Qs + qch * 128 * 128;        // [qch][C keys][128 B]
  uint8_t* Vs = Ks + qch * a.C * 128;        // [vch][C keys][128 B] (value dims contiguous)
  __shared__ uint64_t mbar;
  __shared__ uint32_t tmem_slot;
  __shared__ int32_t s_req[128];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = *a.total_tiles;
  const int first = blockIdx.x * a.tiles_per_cta;
  if (first >= total) return;
  const int last = min(first + a.tiles_per_cta, total);

  if (tid == 0) tc::mbar_init(&mbar, 1);
  if (warp == 0) tc::tmem_alloc(&tmem_slot, a.tmem_cols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_base = (uint32_t(warp) * 32) << 16;
  const uint32_t qs_addr = tc::smem_u32(Qs), ks_addr = tc::smem_u32(Ks), vs_addr = tc::smem_u32(Vs);
  const T* qbase = static_cast<const T*>(a.q);
  const T* kbase = static_cast<const T*>(a.k);
  const T* vbase = static_cast<const T*>(a.v);
  T* part_o = static_cast<T*>(a.part_o);
  const uint32_t idesc_s = tc::idesc_f16(128, a.C, a.bf16);
  const uint32_t idesc_o = tc::idesc_f16(128, a.Dv, a.bf16, 1);
  uint32_t phase = 0;
  int64_t cur_kv = -1;
  bool ok = true;

  for (int tile = first; tile < last; ++tile) {
    const int owner = a.tile_owner[tile];
    const int blk = owner % a.NB;
    const int h = (owner / a.NB) % a.H;
    const int b = owner / (a.NB * a.H * a.nwin);
    if (tid < a.RT) s_req[tid] = a.tile_req[int64_t(tile) * a.RT + tid];
    const int64_t kv_key = (int64_t(b) * a.H + h) * a.NB + blk;
    if (kv_key != cur_kv) {
      const int64_t tok0 = int64_t(blk) * a.C;
      const T* kb = kbase + b * a.k_sb + int64_t(h) * a.k_sh;
      const T* vb = vbase + b * a.v_sb + int64_t(h) * a.v_sh;
      const int kvec = a.Dp / 8, vvec = a.Dvp / 8;
      for (int idx = tid; idx < a.C * kvec; idx += kThreads) {
        const int r = idx / kvec, c = idx % kvec;
        const uint32_t dst = ks_addr + (c >> 3) * a.C * 128 + tc::swizzle128(r, c & 7);
        const int64_t tok = tok0 + r;
        if (tok < a.N && c < a.D / 8) cp_async16(dst, kb + tok * a.k_st + c * 8);
        else st_zero16(dst);
      }
      for (int idx = tid; idx < a.C * vvec; idx += kThreads) {
        const int r = idx / vvec, c = idx % vvec;
        const uint32_t dst = vs_addr + (c >> 3) * a.C * 128 + tc::swizzle128(r, c & 7);
        const int64_t tok = tok0 + r;
        if (tok < a.N && c < a.Dv / 8) cp_async16(dst, vb + tok * a.v_st + c * 8);
        else st_zero16(dst);
      }
      cur_kv = kv_key;
    }
    __syncthreads();  // s_req visible
    {
      const int qvec = a.Dp / 8;
      for (int idx = tid; idx < 128 * qvec; idx += kThreads) {
        const int row = idx / qvec, c = idx % qvec;
        const int r = row / a.G, g = row % a.G;
        const uint32_t dst = qs_addr + (c >> 3) * 128 * 128 + tc::swizzle128(row, c & 7);
        const int req = r < a.RT ? s_req[r] : -1;
        if (req >= 0 && c < a.D / 8) {
          const Req q = decode_req(req, a);
          cp_async16(dst, qbase + q.b * a.q_sb + int64_t(a.t0 + q.tl) * a.q_st +
                              int64_t(q.h * a.G + g) * a.q_sh + c * 8);
        } else {
          st_zero16(dst);
        }
      }
    }
    cp_async_wait_all();
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0) {
      for (int ks = 0; ks < a.Dp / 16; ++ks) {
        const int ch = ks >> 2, off = (ks & 3) * 32;
        tc::mma_f16(tmem, tc::desc_sw128(qs_addr + ch * 128 * 128 + off),
                    tc::desc_sw128(ks_addr + ch * a.C * 128 + off), idesc_s, ks > 0);
      }
      tc::mma_commit(&mbar);
    }
    if (!tc::mbar_wait(&mbar, phase)) ok = false;
    phase ^= 1;
    tc::fence_after_sync();

    // masked softmax of this thread's row; P back to TMEM in the input type
    const int row = tid;
    const int r = row / a.G, g = row % a.G;
    const int req = r < a.RT ? s_req[r] : -1;
    int nvalid = 0;
    if (req >= 0) {
      const Req q = decode_req(req, a);
      int64_t limit = a.N;
      if (a.causal) limit = min64(limit, position_of(a, q.b, a.t0 + q.tl) + 1);
      nvalid = int(max(int64_t(0), min64(int64_t(a.C), limit - int64_t(blk) * a.C)));
    }
    float mx = -INFINITY;
    for_columns(tmem + lane_base, a.C, [&](int c, float x) {
      if (c < nvalid) mx = fmaxf(mx, x * a.scale);
    });
    float l = 0.f;
    for (int c0 = 0; c0 < a.C; c0 += 32) {
      if (a.C - c0 >= 32) {
        float v[32];
        tc::tmem_ld32(tmem + lane_base + c0, v);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = (c0 + 2 * i < nvalid) ? expf(v[2 * i] * a.scale - mx) : 0.f;
          const float p1 = (c0 + 2 * i + 1 < nvalid) ? expf(v[2 * i + 1] * a.scale - mx) : 0.f;
          l += p0 + p1;
          w[i] = pack2<T>(p0, p1);
        }
        tc::tmem_st16(tmem + lane_base + a.p_col + c0 / 2, w);
      } else {
        float v[16];
        tc::tmem_ld16(tmem + lane_base + c0, v);
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float p0 = (c0 + 2 * i < nvalid) ? expf(v[2 * i] * a.scale - mx) : 0.f;
          const float p1 = (c0 + 2 * i + 1 < nvalid) ? expf(v[2 * i + 1] * a.scale - mx) : 0.f;
          l += p0 + p1;
          w[i] = pack2<T>(p0, p1);
        }
        tc::tmem_st8(tmem + lane_base + a.p_col + c0 / 2, w);
      }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0) {
      for (int ks = 0; ks < a.C / 16; ++ks) {
        const uint64_t vd = tc::desc_make(vs_addr + ks * 16 * 128, uint32_t(a.C) * 128, 1024, 2);
        tc::mma_f16_ts(tmem + a.o_col, tmem + a.p_col + ks * 8, vd, idesc_o, ks > 0);
      }
      tc::mma_commit(&mbar);
    }
    if (!tc::mbar_wait(&mbar, phase)) ok = false;
    phase ^= 1;
    tc::fence_after_sync();

    // block-local partial: (m, l) and O / l in the input type
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t pi = int64_t(req) * a.G + g;
    for (int c0 = 0; c0 < a.Dv; c0 += 32) {
      if (a.Dv - c0 >= 32) {
        float v[32];
        tc::tmem_ld32(tmem + lane_base + a.o_col + c0, v);
        if (req >= 0) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = pack2<T>(v[2 * i] * inv, v[2 * i + 1] * inv);
          uint4* dst = reinterpret_cast<uint4*>(part_o + pi * a.Dv + c0);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      } else {
        float v[16];
        tc::tmem_ld16(tmem + lane_base + a.o_col + c0, v);
        if (req >= 0) {
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = pack2<T>(v[2 * i] * inv, v[2 * i + 1] * inv);
          uint4* dst = reinterpret_cast<uint4*>(part_o + pi * a.Dv + c0);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
    }
    if (req >= 0) reinterpret_cast<float2*>(a.part_ml)[pi] = make_float2(mx, l);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }
  if (!ok && lane == 0) atomicExch(a.status, PISA_ERR_TIMEOUT);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_free(tmem, a.tmem_cols);
}

// Merge the S block partials of one query head (one warp per head row).
template <typename T, int DPL>
__global__ void __launch_bounds__(128) attn_combine_kernel(const AttnTcArgs a) {
  const int64_t idx = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (idx >= int64_t(a.B) * a.tlen * a.Hq) return;
  const int hq = int(idx % a.Hq);
  const int tl = int((idx / a.Hq) % a.tlen);
  const int b = int(idx / (int64_t(a.Hq) * a.tlen));
  const int h = hq / a.G, g = hq % a.G;
  const int t = a.t0 + tl;
  const int64_t row_local = (int64_t(b) * a.tlen + tl) * a.H + h;
  const T* part_o = static_cast<const T*>(a.part_o);
  float M = -INFINITY, L = 0.f, acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
  for (int s = 0; s < a.S; ++s) {
    if (visible_block(a, b, t, h, s) < 0) continue;
    const int64_t pi = (row_local * a.S + s) * a.G + g;
    const float2 ml = reinterpret_cast<const float2*>(a.part_ml)[pi];
    if (ml.y <= 0.f) continue;
    if (ml.x > M) {
      const float f = M == -INFINITY ? 0.f : expf(M - ml.x);
      L *= f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] *= f;
      M = ml.x;
    }
    const float w = expf(ml.x - M) * ml.y;
    L += w;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = lane * DPL + i;
      if (d < a.Dv) acc[i] = fmaf(w, to_f32<T>(part_o[pi * a.Dv + d]), acc[i]);
    }
  }
  T* out = static_cast<T*>(a.out) + ((int64_t(b) * a.T + t) * a.Hq + hq) * a.Dv;
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int d = lane * DPL + i;
    if (d < a.Dv) out[d] = from_f32<T>(acc[i] * inv);
  }
  if (lane == 0 && a.lse) a.lse[(int64_t(b) * a.T + t) * a.Hq + hq] = L > 0.f ? M + logf(L) : -INFINITY;
}

template <typename T>
int attn_tc_typed(AttnTcArgs a, cudaStream_t stream) {
  const int qch = a.Dp / 64, vch = a.Dvp / 64;
  size_t smem = size_t(128) * 128 * qch + size_t(a.C) * 128 * (qch + vch) + 1024;
  const size_t ctas_fit = 512 / size_t(a.tmem_cols);
  if (ctas_fit < 16) smem = std::max(smem, size_t(228 * 1024) / ctas_fit - 4096);
  cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return fail_cuda(e, "attention smem attribute");
  for (int t0 = 0; t0 < a.T; t0 += a.chunk) {
    a.t0 = t0;
    a.tlen = std::min(a.chunk, a.T - t0);
    a.nwin = (a.tlen + a.TW - 1) / a.TW;
    a.num_buckets = int64_t(a.B) * a.nwin * a.H * a.NB;
    const int64_t reqs = int64_t(a.B) * a.tlen * a.H * a.S;
    a.capacity = (reqs + a.RT - 1) / a.RT + a.num_buckets;
    e = cudaMemsetAsync(a.counts, 0, sizeof(int32_t) * a.num_buckets, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(a.cursors, 0, sizeof(int32_t) * a.num_buckets, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(a.tile_req, 0xFF, sizeof(int32_t) * a.capacity * a.RT, stream);
    if (e != cudaSuccess) return fail_cuda(e, "attention bucket clear");
    const unsigned grid = unsigned((reqs + 255) / 256);
    attn_count_kernel<<<grid, 256, 0, stream>>>(a);
    PISA_CHECK_LAUNCH();
    tile_scan_kernel<<<1, kScanThreads, 0, stream>>>(a.counts, a.offsets, a.total_tiles, a.num_buckets, a.RT);
    PISA_CHECK_LAUNCH();
    attn_scatter_kernel<<<grid, 256, 0, stream>>>(a);
    PISA_CHECK_LAUNCH();
    const int64_t ctas = (a.capacity + a.tiles_per_cta - 1) / a.tiles_per_cta;
    attn_tc_kernel<T><<<unsigned(ctas), kThreads, smem, stream>>>(a);
    PISA_CHECK_LAUNCH();
    const unsigned cgrid = unsigned((int64_t(a.B) * a.tlen * a.Hq + 3) / 4);
    if (a.Dv <= 32) attn_combine_kernel<T, 1><<<cgrid, 128, 0, stream>>>(a);
    else if (a.Dv <= 64) attn_combine_kernel<T, 2><<<cgrid, 128, 0, stream>>>(a);
    else if (a.Dv <= 128) attn_combine_kernel<T, 4><<<cgrid, 128, 0, stream>>>(a);
    else attn_combine_kernel<T, 8><<<cgrid, 128, 0, stream>>>(a);
    PISA_CHECK_LAUNCH();
  }
  return PISA_OK;
}

}  // namespace

int attn_fwd_tc(const AttnTcArgs& a, int dtype, cudaStream_t stream) {
  if (dtype == PISA_BF16) return attn_tc_typed<__nv_bfloat16>(a, stream);
  if (dtype == PISA_F16) return attn_tc_typed<__half>(a, stream);
  return fail(PISA_ERR_UNSUPPORTED, "tensor-core attention needs fp16 or bf16");
}

}  // namespace pisa
