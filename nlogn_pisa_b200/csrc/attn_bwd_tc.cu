// K4 backward on the tensor cores: gradients of the attention over selected
// blocks (the autograd of sparse_attn_torch.py:6-35; the reference's GPU
// backward is fla-core's ParallelNSAFunction, called at sparse_attn_fla.py:59-68).
//
// With s = scale * q.k over a row's visible keys, P = exp(s - lse) (lse from
// the forward), dP = dO . v, D = dO . O and dS = scale * P * (dP - D):
//   dQ = dS K,   dK = dS^T Q,   dV = P^T dO.
// The requests (row, slot) are bucketed exactly as in the forward (attn_tc.cu:
// bucket = (batch, token window, KV head, block)), so one tile is one key block
// against up to 128/G requests (128 query-head rows).  Per tile:
//   MMA  S  = Q K^T          (M=128 rows, N=C, K=D)      -> TMEM
//   MMA  dP = dO V^T         (M=128 rows, N=C, K=Dv)     -> TMEM
//   epilogue (thread = row): P and dS in bf16/fp16 into shared memory
//   MMA  dV^T += dO^T P      (M=128 dims, N=C, K=128 rows; A and B MN-major)
//   MMA  dK^T += Q^T dS      (M=128 dims, N=C, K=128 rows)
//   MMA  dQ  = dS K          (M=128 rows, N=D, K=C; B MN-major)
//   epilogue: dQ rows added into an fp32 accumulator; when the next tile
//   belongs to another block, the block's dK^T / dV^T columns are added
//   into fp32 accumulators once (one reduction per run of tiles instead of
//   one per row: the first and local blocks, selected by every query, see no
//   per-row atomics).
// The query and dO stages always hold 128 dims (two 64-wide chunks, the
// second zero when D = 64) so dK^T / dV^T are M=128 MMAs.  Block size 64.
#include <algorithm>
#include <type_traits>

#include "bucket.cuh"
#include "internal.h"
#include "tc.cuh"

namespace pisa {

namespace {

constexpr int kEpi = 4, kLoad = 8, kMma = kEpi + kLoad, kThreads = (kMma + 1) * 32;
constexpr int kStages = 2, kMeta = 8, kRowsPerLoader = 128 / kLoad;
constexpr int kBwdC = 64;

__device__ __forceinline__ int64_t index_at(const void* p, int bytes, int64_t i) {
  return bytes == 4 ? int64_t(static_cast<const int32_t*>(p)[i]) : static_cast<const int64_t*>(p)[i];
}

struct Req {
  int b, tl, h, s;
};
__device__ __forceinline__ Req decode_req(uint32_t lr, const AttnTcArgs& a) {
  Req r;
  const uint32_t row = a.fS.div(lr);
  r.s = int(lr - row * uint32_t(a.S));
  const uint32_t rest = a.fH.div(row);
  r.h = int(row - rest * uint32_t(a.H));
  const uint32_t b = a.ftlen.div(rest);
  r.tl = int(rest - b * uint32_t(a.tlen));
  r.b = int(b);
  return r;
}

__device__ __forceinline__ int64_t position_of(const AttnTcArgs& a, int b, int t) {
  return a.positions ? a.positions[int64_t(b) * a.T + t] : a.pos_offset + t;
}

// (batch, KV head, block) of a bucket, packed into one key
__device__ __forceinline__ void decode_owner(const AttnTcArgs& a, int owner, int& b, int& h, int& blk) {
  const uint32_t o1 = a.fNB.div(uint32_t(owner)), o2 = a.fH.div(o1);
  blk = owner - int(o1) * a.NB;
  h = int(o1) - int(o2) * a.H;
  b = int(a.fnwin.div(o2));
}
__device__ __forceinline__ int64_t block_key(const AttnTcArgs& a, int owner) {
  int b, h, blk;
  decode_owner(a, owner, b, h, blk);
  return (int64_t(b) * a.H + h) * a.NB + blk;
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

__device__ __forceinline__ void red_add4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" :: "l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) attn_bwd_tc_kernel(const __grid_constant__ AttnTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kTile = 128 * 128;                // one 64-wide chunk of 128 rows
  constexpr int kStageBytes = 4 * kTile;          // Q (2 chunks) + dO (2 chunks)
  const int qch = a.Dp / 64, vch = a.Dvp / 64;
  const int kv_bytes = (qch + vch) * kBwdC * 128;
  uint8_t* KV = smem + kStages * kStageBytes;
  uint8_t* Pt = KV + 2 * kv_bytes;                // P tile [128 rows][64 keys], swizzled
  uint8_t* dSt = Pt + kTile;                      // dS tile, same layout
  __shared__ uint64_t st_full[kStages], st_empty[kStages], s_full, p_full, o_full, o_empty;
  __shared__ uint64_t meta_full[kMeta];
  __shared__ uint32_t tmem_slot;
  __shared__ int s_kvb[kStages];
  __shared__ int s_req[kMeta][128], s_nv[kMeta][128];
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = *a.total_tiles;
  const int ngroups = (total + 7) / 8;
  const int my_groups = ngroups > int(blockIdx.x) ? (ngroups - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
  if (my_groups == 0) return;
  const int last_group = int(blockIdx.x) + (my_groups - 1) * int(gridDim.x);
  const int ntiles = (my_groups - 1) * 8 + min(8, total - last_group * 8);
  auto tile_of = [&](int it) { return (int(blockIdx.x) + (it / 8) * int(gridDim.x)) * 8 + it % 8; };

  // zero the operand stages once: padded dims (D = 64) and rows of empty
  // request slots must hold finite values (they meet zero P / dS rows)
  for (int i = tid * 16; i < kStages * kStageBytes; i += kThreads * 16) st_zero16(tc::smem_u32(smem + i));
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      tc::mbar_init(&st_full[i], kLoad * 32 + 1);
      tc::mbar_init(&st_empty[i], 1);
    }
    tc::mbar_init(&s_full, 1);
    tc::mbar_init(&p_full, kEpi);
    tc::mbar_init(&o_full, 1);
    tc::mbar_init(&o_empty, kEpi);
    for (int i = 0; i < kMeta; ++i) tc::mbar_init(&meta_full[i], kLoad);
    s_fail = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t tS = tmem, tdP = tmem + 64, tdQ = tmem + 128, tdV = tmem + 256, tdK = tmem + 320;
  const uint32_t st_addr = tc::smem_u32(smem), kv_addr = tc::smem_u32(KV);
  const uint32_t p_addr = tc::smem_u32(Pt), ds_addr = tc::smem_u32(dSt);
  const int lgG = 31 - __clz(a.G);

  if (warp >= kEpi && warp < kMma) {
    // ---------------- producers: Q and dO rows (cp.async), K/V blocks (TMA) ----------------
    const int pw = warp - kEpi;
    const int row = pw * kRowsPerLoader + (lane & (kRowsPerLoader - 1));
    const int j = row >> lgG, gq = row & (a.G - 1);
    const int lgQ = 31 - __clz(a.D / 8), lgV = 31 - __clz(a.Dv / 8);
    const T* qbase = static_cast<const T*>(a.q);
    const T* dbase = static_cast<const T*>(a.dout);
    int64_t cur_kv = -1;
    int kvb = 1;
    for (int it = 0; it < ntiles; ++it) {
      const int s = it % kStages;
      if (!tc::mbar_wait(&st_empty[s], ((it / kStages) & 1) ^ 1)) { s_fail = 1; break; }
      const int tile = tile_of(it);
      const int owner = a.tile_owner[tile];
      const int req = a.tile_req[int64_t(tile) * a.RT + j];
      int b, h, blk;
      decode_owner(a, owner, b, h, blk);
      const T* qsrc = nullptr;
      const T* dsrc = nullptr;
      int nv = 0;
      if (req >= 0) {
        const Req q = decode_req(uint32_t(req), a);
        const int t = a.t0 + q.tl;
        int64_t limit = a.N;
        if (a.causal) limit = min64(limit, position_of(a, q.b, t) + 1);
        nv = int(max(int64_t(0), min64(int64_t(kBwdC), limit - int64_t(blk) * kBwdC)));
        const int64_t r = (int64_t(q.b) * a.T + t) * a.Hq + q.h * a.G + gq;
        qsrc = qbase + r * a.D;
        dsrc = dbase + r * a.Dv;
      }
      const uint32_t qst = st_addr + s * kStageBytes, dst = qst + 2 * kTile;
      // Q rows: 16-byte segment `seg` of row r lands at chunk seg/8, position (seg%8)^(r%8)
      for (int u = 0; u < (kRowsPerLoader << lgQ) / 32; ++u) {
        const int f = u * 32 + lane;
        const int rl = f >> lgQ, seg = f & ((1 << lgQ) - 1);
        const T* rs = reinterpret_cast<const T*>(__shfl_sync(kFull, reinterpret_cast<uintptr_t>(qsrc), rl));
        if (rs != nullptr) {
          const int r = pw * kRowsPerLoader + rl;
          cp_async16(qst + (seg >> 3) * kTile + r * 128 + (((seg & 7) ^ (r & 7)) << 4), rs + seg * 8);
        }
      }
      for (int u = 0; u < (kRowsPerLoader << lgV) / 32; ++u) {
        const int f = u * 32 + lane;
        const int rl = f >> lgV, seg = f & ((1 << lgV) - 1);
        const T* rs = reinterpret_cast<const T*>(__shfl_sync(kFull, reinterpret_cast<uintptr_t>(dsrc), rl));
        if (rs != nullptr) {
          const int r = pw * kRowsPerLoader + rl;
          cp_async16(dst + (seg >> 3) * kTile + r * 128 + (((seg & 7) ^ (r & 7)) << 4), rs + seg * 8);
        }
      }
      tc::cp_async_arrive(&st_full[s]);
      const int slot = it & (kMeta - 1);
      if (gq == 0 && lane < kRowsPerLoader) {
        s_req[slot][j] = req;
        s_nv[slot][j] = nv;
      }
      uint32_t bytes = 0;
      if (pw == 0) {
        const int64_t kv_key = (int64_t(b) * a.H + h) * a.NB + blk;
        if (kv_key != cur_kv) {
          kvb ^= 1;
          // the buffer being replaced was last read by tile it-2 or earlier
          // (dQ MMA); its stage's empty barrier completed after that MMA
          if (it >= 2 && !tc::mbar_wait(&st_empty[s], ((it / kStages) & 1) ^ 1)) { s_fail = 1; break; }
          const uint32_t ks = kv_addr + kvb * kv_bytes, vs = ks + qch * kBwdC * 128;
          if (lane < qch)
            tc::tma_load_4d(ks + lane * kBwdC * 128, &a.tm_k, lane * 64, h, blk * kBwdC, b, &st_full[s]);
          else if (lane < qch + vch)
            tc::tma_load_4d(vs + (lane - qch) * kBwdC * 128, &a.tm_v, (lane - qch) * 64, h, blk * kBwdC, b,
                            &st_full[s]);
          bytes = uint32_t(qch + vch) * kBwdC * 128;
          cur_kv = kv_key;
        }
      }
      __syncwarp();
      if (lane == 0) {
        if (pw == 0) {
          s_kvb[s] = kvb;
          tc::mbar_arrive_expect_tx(&st_full[s], bytes);
        }
        tc::mbar_arrive(&meta_full[slot]);
      }
      __syncwarp();
    }
    cp_async_wait_all();
  } else if (warp == kMma) {
    // ---------------- MMA issue (one thread) ----------------
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_f16(128, kBwdC, a.bf16);
      // dV^T / dK^T: A = dO^T or Q^T (MN-major stage), B = P or dS (MN-major tile)
      const uint32_t id_kv = tc::idesc_f16(128, kBwdC, a.bf16, 1) | (1u << 15);
      const uint32_t id_q = tc::idesc_f16(128, a.D, a.bf16, 1);
      int64_t prev_key = -1;
      for (int it = 0; it < ntiles; ++it) {
        const int s = it % kStages;
        if (!tc::mbar_wait(&st_full[s], (it / kStages) & 1)) { s_fail = 1; break; }
        // S / dP of the previous tile were consumed (P, dS written)
        if (it > 0 && !tc::mbar_wait(&p_full, (it - 1) & 1)) { s_fail = 1; break; }
        tc::fence_async_smem();
        tc::fence_after_sync();
        const uint32_t qst = st_addr + s * kStageBytes, dst = qst + 2 * kTile;
        const uint32_t ks = kv_addr + s_kvb[s] * kv_bytes, vs = ks + qch * kBwdC * 128;
        for (int k = 0; k < a.Dp / 16; ++k) {
          const int ch = k >> 2, off = (k & 3) * 32;
          tc::mma_f16(tS, tc::desc_sw128(qst + ch * kTile + off), tc::desc_sw128(ks + ch * kBwdC * 128 + off),
                      id_s, k > 0);
        }
        for (int k = 0; k < a.Dvp / 16; ++k) {
          const int ch = k >> 2, off = (k & 3) * 32;
          tc::mma_f16(tdP, tc::desc_sw128(dst + ch * kTile + off), tc::desc_sw128(vs + ch * kBwdC * 128 + off),
                      id_s, k > 0);
        }
        tc::mma_commit(&s_full);
        if (!tc::mbar_wait(&p_full, it & 1)) { s_fail = 1; break; }
        if (it > 0 && !tc::mbar_wait(&o_empty, (it - 1) & 1)) { s_fail = 1; break; }
        tc::fence_async_smem();
        tc::fence_after_sync();
        const int64_t key = block_key(a, a.tile_owner[tile_of(it)]);
        const bool first = key != prev_key;
        prev_key = key;
        for (int k = 0; k < 128 / 16; ++k) {
          // K = 16 rows of the tile per instruction; 64-dim chunks 16 KB apart
          const uint64_t pd = tc::desc_make(p_addr + k * 16 * 128, kTile, 1024, 2);
          const uint64_t sd = tc::desc_make(ds_addr + k * 16 * 128, kTile, 1024, 2);
          tc::mma_f16(tdV, tc::desc_make(dst + k * 16 * 128, kTile, 1024, 2), pd, id_kv, !(first && k == 0));
          tc::mma_f16(tdK, tc::desc_make(qst + k * 16 * 128, kTile, 1024, 2), sd, id_kv, !(first && k == 0));
        }
        for (int k = 0; k < kBwdC / 16; ++k)
          tc::mma_f16(tdQ, tc::desc_sw128(ds_addr + k * 32), tc::desc_make(ks + k * 16 * 128, kBwdC * 128, 1024, 2),
                      id_q, k > 0);
        tc::mma_commit(&o_full);
        tc::mma_commit(&st_empty[s]);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 0-3, thread = TMEM lane = tile row) ----------------
    const int row = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t(warp) * 32) << 16;
    const int r = row >> lgG, g = row & (a.G - 1);
    const float l2e = 1.4426950408889634f;
    const float sl = a.scale * l2e;
    const uint32_t prow = p_addr + row * 128, dsrow = ds_addr + row * 128;
    for (int it = 0; it < ntiles; ++it) {
      bool got = tc::mbar_wait(&s_full, it & 1);
      if (!tc::mbar_wait(&meta_full[it & (kMeta - 1)], (it / kMeta) & 1)) got = false;
      if (!got) s_fail = 1;
      tc::fence_after_sync();
      const int req = r < a.RT ? s_req[it & (kMeta - 1)][r] : -1;
      const int nv = r < a.RT ? s_nv[it & (kMeta - 1)][r] : 0;
      float lse2 = INFINITY, dd = 0.f;
      int64_t orow = -1;
      if (req >= 0) {
        const Req q = decode_req(uint32_t(req), a);
        orow = (int64_t(q.b) * a.T + a.t0 + q.tl) * a.Hq + q.h * a.G + g;
        const float lse = a.lse_in[orow];
        lse2 = lse == -INFINITY ? INFINITY : lse * l2e;   // no visible key: P = 0
        dd = a.dvec[orow];
      }
      // P and dS, 32 columns at a time, packed into the swizzled tiles
      for (int c0 = 0; c0 < kBwdC; c0 += 32) {
        float sv[32], dp[32];
        tc::tmem_ld32(tS + lane_base + c0, sv);
        tc::tmem_ld32(tdP + lane_base + c0, dp);
        uint32_t pw[16], dw[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float p0 = 0.f, p1 = 0.f;
          if (c0 + i < nv) p0 = tc::ex2f(fmaf(sv[i], sl, -lse2));
          if (c0 + i + 1 < nv) p1 = tc::ex2f(fmaf(sv[i + 1], sl, -lse2));
          pw[i / 2] = pack2<T>(p0, p1);
          dw[i / 2] = pack2<T>(a.scale * p0 * (dp[i] - dd), a.scale * p1 * (dp[i + 1] - dd));
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int chunk = (c0 / 8) + c;   // 16-byte chunk of the 128-byte row
          const uint32_t off = uint32_t((chunk ^ (row & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" :: "r"(prow + off), "r"(pw[4 * c]), "r"(pw[4 * c + 1]),
                       "r"(pw[4 * c + 2]), "r"(pw[4 * c + 3]) : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" :: "r"(dsrow + off), "r"(dw[4 * c]), "r"(dw[4 * c + 1]),
                       "r"(dw[4 * c + 2]), "r"(dw[4 * c + 3]) : "memory");
        }
      }
      tc::fence_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&p_full);
      if (!tc::mbar_wait(&o_full, it & 1)) { s_fail = 1; got = false; }
      tc::fence_after_sync();
      // dQ row into its fp32 accumulator
      for (int c0 = 0; c0 < a.D; c0 += 32) {
        float v[32];
        tc::tmem_ld32(tdQ + lane_base + c0, v);
        if (orow >= 0) {
          float* dq = a.dq_acc + orow * a.D + c0;
#pragma unroll
          for (int i = 0; i < 32; i += 4) red_add4(dq + i, v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
      }
      // end of a block run: its dK^T / dV^T columns (lane = dim) into the accumulators
      const int owner = a.tile_owner[tile_of(it)];
      const bool flush = it + 1 == ntiles || block_key(a, a.tile_owner[tile_of(it + 1)]) != block_key(a, owner);
      if (flush) {
        int b, h, blk;
        decode_owner(a, owner, b, h, blk);
        const int d = row;   // TMEM lane of the transposed accumulators
        for (int c0 = 0; c0 < kBwdC; c0 += 32) {
          float kv[32], vv[32];
          tc::tmem_ld32(tdK + lane_base + c0, kv);
          tc::tmem_ld32(tdV + lane_base + c0, vv);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int64_t tok = int64_t(blk) * kBwdC + c0 + i;
            if (tok < a.N) {
              const int64_t base = (int64_t(b) * a.N + tok) * a.H + h;
              if (d < a.D) atomicAdd(a.dk_acc + base * a.D + d, kv[i]);
              if (d < a.Dv) atomicAdd(a.dv_acc + base * a.Dv + d, vv[i]);
            }
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&o_empty);
      if (!got) break;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (tid == 0 && s_fail) atomicExch(a.status, PISA_ERR_TIMEOUT);
  if (warp == 0) tc::tmem_free(tmem, 512);
}

// D = dO . O per (batch, token, query head), one warp per row.
template <typename T>
__global__ void row_dot_kernel(const T* __restrict__ dout, const T* __restrict__ out, float* __restrict__ dvec,
                               int64_t rows, int Dv) {
  const int64_t r = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float acc = 0.f;
  for (int d = lane; d < Dv; d += 32) acc += to_f32<T>(dout[r * Dv + d]) * to_f32<T>(out[r * Dv + d]);
  acc = warp_sum(acc);
  if (lane == 0) dvec[r] = acc;
}

template <typename T>
__global__ void cast_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i < n) dst[i] = from_f32<T>(src[i]);
}

template <typename T>
int bwd_typed(AttnTcArgs a, void* dq, void* dk, void* dv, cudaStream_t stream) {
  const int qch = a.Dp / 64, vch = a.Dvp / 64;
  const size_t smem = size_t(kStages) * 4 * 128 * 128 + size_t(2) * (qch + vch) * kBwdC * 128 + 2 * 128 * 128 + 1024;
  cudaError_t e = cudaFuncSetAttribute(attn_bwd_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return fail_cuda(e, "attention backward smem attribute");
  const int64_t rows = int64_t(a.B) * a.T * a.Hq;
  const int64_t nk = int64_t(a.B) * a.N * a.H;
  e = cudaMemsetAsync(a.dq_acc, 0, sizeof(float) * rows * a.D, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(a.dk_acc, 0, sizeof(float) * nk * a.D, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(a.dv_acc, 0, sizeof(float) * nk * a.Dv, stream);
  if (e != cudaSuccess) return fail_cuda(e, "attention backward clear");
  row_dot_kernel<T><<<unsigned((rows + 3) / 4), 128, 0, stream>>>(static_cast<const T*>(a.dout),
                                                                   static_cast<const T*>(a.out), a.dvec, rows, a.Dv);
  PISA_CHECK_LAUNCH();
  a.fS = FastDiv::make(uint32_t(a.S));
  a.fH = FastDiv::make(uint32_t(a.H));
  a.fHq = FastDiv::make(uint32_t(a.Hq));
  a.fNB = FastDiv::make(uint32_t(a.NB));
  a.fTW = FastDiv::make(uint32_t(a.TW));
  a.fRT = FastDiv::make(uint32_t(a.RT));
  for (int t0 = 0; t0 < a.T; t0 += a.chunk) {
    int rc = attn_bucket_chunk(a, t0, stream);
    if (rc != PISA_OK) return rc;
    attn_bwd_tc_kernel<T><<<unsigned(a.num_sms), kThreads, smem, stream>>>(a);
    PISA_CHECK_LAUNCH();
  }
  cast_kernel<T><<<unsigned((rows * a.D + 255) / 256), 256, 0, stream>>>(a.dq_acc, static_cast<T*>(dq), rows * a.D);
  PISA_CHECK_LAUNCH();
  cast_kernel<T><<<unsigned((nk * a.D + 255) / 256), 256, 0, stream>>>(a.dk_acc, static_cast<T*>(dk), nk * a.D);
  PISA_CHECK_LAUNCH();
  cast_kernel<T><<<unsigned((nk * a.Dv + 255) / 256), 256, 0, stream>>>(a.dv_acc, static_cast<T*>(dv), nk * a.Dv);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

}  // namespace

int attn_bwd_tc(const AttnTcArgs& a, int dtype, void* dq, void* dk, void* dv, cudaStream_t stream) {
  if (dtype == PISA_BF16) return bwd_typed<__nv_bfloat16>(a, dq, dk, dv, stream);
  if (dtype == PISA_F16) return bwd_typed<__half>(a, dq, dk, dv, stream);
  return fail(PISA_ERR_UNSUPPORTED, "tensor-core attention backward needs fp16 or bf16");
}

}  // namespace pisa
