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
// and writes the block-local partial (m, l, sum_k e^(s_k - m) v_k) of every
// row.  A combine pass merges the S partials of each query head into the
// output and its log-sum-exp.  Moving each query row to its blocks once (instead of every
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

__device__ __forceinline__ int64_t index_at(const void* p, int bytes, int64_t i) {
  return bytes == 4 ? int64_t(static_cast<const int32_t*>(p)[i]) : static_cast<const int64_t*>(p)[i];
}

// Chunk-local request lr = ((b * tlen + tl) * H + h) * S + s.
struct Req {
  int b, tl, h, s;
};
__device__ __forceinline__ Req decode_req(int64_t lr64, const AttnTcArgs& a) {
  // chunk-local request indices are below 2^31 (checked on the host)
  const uint32_t lr = uint32_t(lr64);
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

// Visible block id of a request, or -1.
__device__ __forceinline__ int64_t visible_block(const AttnTcArgs& a, int b, int t, int h, int s) {
  const int64_t id = index_at(a.indices, a.index_bytes, ((int64_t(b) * a.T + t) * a.H + h) * a.S + s);
  if (id < 0 || id * a.C >= a.N) return -1;
  if (a.causal && id * a.C > position_of(a, b, t)) return -1;
  return id;
}

__device__ __forceinline__ int64_t bucket_of(const AttnTcArgs& a, const Req& r, int64_t id) {
  return ((int64_t(r.b) * a.nwin + int(a.fTW.div(uint32_t(r.tl)))) * a.H + r.h) * a.NB + id;
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
  const int q = int(a.fRT.div(uint32_t(pos))), slot = pos - q * a.RT;
  const int64_t tile = a.offsets[bucket] + q;
  a.tile_req[tile * a.RT + slot] = int32_t(lr);
  if (slot == 0) a.tile_owner[tile] = int32_t(bucket);
}

// streaming store / load (partials are written once and read once) and the
// shared-memory staging accesses of the partial readout
__device__ __forceinline__ void st_cs16(void* p, uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3) {
  asm volatile("st.global.cs.v4.b32 [%0], {%1,%2,%3,%4};" :: "l"(p), "r"(x0), "r"(x1), "r"(x2), "r"(x3)
               : "memory");
}
__device__ __forceinline__ void st_shared16(uint32_t addr, uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" :: "r"(addr), "r"(x0), "r"(x1), "r"(x2), "r"(x3)
               : "memory");
}
__device__ __forceinline__ void ld_shared16(uint32_t addr, uint32_t& x0, uint32_t& x1, uint32_t& x2, uint32_t& x3) {
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(x0), "=r"(x1), "=r"(x2), "=r"(x3) : "r"(addr)
               : "memory");
}
// CTA-scope release store / acquire load of a shared-memory counter
__device__ __forceinline__ void st_release_cta(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" :: "r"(tc::smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_cta(int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(tc::smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void ld_cs32(const void* p, uint32_t (&w)[8]) {
  asm volatile("ld.global.cs.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]),
                 "=r"(w[7]) : "l"(p));
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

// Warp roles (one persistent CTA per SM):
//   warps 0-3        softmax: S into P for every tile (registers, P back to
//                    TMEM) and the row's (m, l); thread = TMEM lane = row
//   warps 4-7        readout: O of every tile into its block partial
//   next kLoadWarps  producers: query rows into a 3-stage ring (cp.async),
//                    block K/V (TMA, first producer warp)
//   last warp        MMA issue: S = Q K^T and O = P V, whichever is ready
// mbarriers per stage/buffer: q_full/q_empty (query stages), s_full, p_full,
// o_full, o_empty (TMEM buffers of S/P and O).  All waits are bounded.
constexpr int kEpiWarps = 8, kLoadWarps = 8, kMmaWarp = kEpiWarps + kLoadWarps, kStages = 3, kGroup = 8;
constexpr int kRowsPerLoader = 128 / kLoadWarps;  // tile rows per producer warp
constexpr int kMeta = 16;                          // metadata ring slots
constexpr int kPipeThreads = (kMmaWarp + 1) * 32;

template <typename T>
__global__ void __launch_bounds__(kPipeThreads, 1) attn_tc_kernel(const __grid_constant__ AttnTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int qch = a.Dp / 64, vch = a.Dvp / 64;
  const int q_stage_bytes = qch * 128 * 128;
  // two K/V buffers, each [qch][C keys][128 B] of keys then [vch][C keys][128 B]
  // of values (value dims contiguous); a block change switches buffers
  const int kv_bytes = (qch + vch) * a.C * 128;
  uint8_t* KV = smem + a.nstages * q_stage_bytes;
  __shared__ uint64_t q_full[kStages], q_empty[kStages], s_full[2], p_full[2], o_full[2], o_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int s_kvb[kStages];
  // per-tile metadata ring for the epilogue (16 slots): the producer of tile
  // i waits for S(i-3), S(i-3) for O(i-5) and O(i-5) for the readout of
  // tile i-7, so the slot of tile i (i % 16) is no longer read when refilled
  __shared__ uint64_t meta_full[kMeta];
  __shared__ int s_req[kMeta][128], s_nv[kMeta][128];
  __shared__ int s_fail;
  // tiles whose P.V has completed, published by the readout (which waits for
  // every one in order): the producer, which needs only some of them, reads
  // this count instead of waiting on o_full, whose phase parity no longer
  // names the phase it wants once the barrier is two phases behind
  __shared__ int s_o_done;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = *a.total_tiles;
  // Tiles go out in groups of kGroup consecutive tiles (one bucket run keeps
  // its staged keys), group k to CTA k mod gridDim: at any moment all SMs work
  // on neighbouring buckets, so the gathered query rows stay in L2.
  const int ngroups = (total + kGroup - 1) / kGroup;
  const int my_groups = ngroups > int(blockIdx.x) ? (ngroups - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
  if (my_groups == 0) return;
  const int last_group = int(blockIdx.x) + (my_groups - 1) * int(gridDim.x);
  const int ntiles = (my_groups - 1) * kGroup + min(kGroup, total - last_group * kGroup);
  auto tile_of = [&](int it) { return (int(blockIdx.x) + (it / kGroup) * int(gridDim.x)) * kGroup + it % kGroup; };
  const int first = tile_of(0);
  const int nacc = a.nacc;                    // S/P and O buffers: 2 (double) or 1
  const int nst = a.nstages;                  // query stages: 3 or 2
  // stage of tile i and the parity of its round (constant divisors only)
  auto stage_of = [&](int i) { return nst == 3 ? i % 3 : (i & 1); };
  auto round_par = [&](int i) { return (nst == 3 ? i / 3 : (i >> 1)) & 1; };

  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      // one cp.async arrival per producer thread + the K/V arrival of the first producer warp
      tc::mbar_init(&q_full[i], kLoadWarps * 32 + 1);
      tc::mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&s_full[i], 1);
      tc::mbar_init(&p_full[i], 4);     // one arrival per epilogue warp of the group
      tc::mbar_init(&o_full[i], 1);
      tc::mbar_init(&o_empty[i], 4);
    }
    for (int i = 0; i < kMeta; ++i) tc::mbar_init(&meta_full[i], kLoadWarps);
    s_fail = 0;
    s_o_done = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, a.tmem_cols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t qs_addr = tc::smem_u32(smem), kv_addr = tc::smem_u32(KV);
  const int lgG = 31 - __clz(a.G);
  // round of tile `it` on its TMEM buffer
  auto acc_of = [&](int it) { return nacc == 2 ? (it & 1) : 0; };
  auto round_of = [&](int it) { return nacc == 2 ? (it >> 1) : it; };

  if (warp >= kEpiWarps && warp < kMmaWarp) {
    // ---------------- producer warps ----------------
    // Query rows move with 16-byte asynchronous copies (cp.async) straight
    // into their swizzled K-major positions; every producer thread's copies
    // arrive on the stage barrier when they land (cp.async.mbarrier.arrive),
    // so the warps go on to the next stage without waiting for the data.
    // Producer warp pw owns kRowsPerLoader tile rows, lane l decodes the
    // request of its l-th row, and one warp instruction moves 512 contiguous
    // bytes.  (A TMA box per request holds only G rows x 128 bytes, and the
    // TMA unit's per-copy cost then bounds the tile rate.)  Producer warp 0
    // also loads K/V of a new block through TMA (C rows per 64-dim chunk,
    // zero past the end of the keys) into the other K/V buffer; those bytes
    // count toward the same tile's barrier.
    const int pw = warp - kEpiWarps;
    const int row = pw * kRowsPerLoader + (lane & (kRowsPerLoader - 1));  // tile row of this lane
    const int j = row >> lgG, gq = row & (a.G - 1);   // its request and head
    const int lgS = 31 - __clz(a.Dp / 8);             // 16-byte segments per row (log2)
    const int nseg = 1 << lgS, dsegs = a.D / 8;
    const T* qbase = static_cast<const T*>(a.q);
    int64_t cur_kv = -1;
    int kvb = 1, used0 = 0, used1 = 0;
    // request of this lane's row in tile `it`: K/V block coordinates, source
    // row and valid keys; decoded one tile ahead, while the copies of the
    // previous tile drain
    int blk = 0, h = 0, b = 0, nv = 0;
    const T* src = nullptr;
    auto decode = [&](int owner, int req) {
      const uint32_t o1 = a.fNB.div(uint32_t(owner)), o2 = a.fH.div(o1);
      blk = owner - int(o1) * a.NB;
      h = int(o1) - int(o2) * a.H;
      b = int(a.fnwin.div(o2));
      src = nullptr;
      nv = 0;
      if (req >= 0) {
        const Req q = decode_req(req, a);
        const int t = a.t0 + q.tl;
        int64_t limit = a.N;
        if (a.causal) limit = min64(limit, position_of(a, q.b, t) + 1);
        nv = int(max(int64_t(0), min64(int64_t(a.C), limit - int64_t(blk) * a.C)));
        src = qbase + int64_t(q.b) * a.q_sb + int64_t(t) * a.q_st + int64_t(q.h * a.G + gq) * a.q_sh;
      }
      return req;
    };
    int req = decode(a.tile_owner[first], a.tile_req[int64_t(first) * a.RT + j]);
    // the next tile's owner and request index are loaded one iteration early
    int owner_n = 0, req_n = -1;
    if (ntiles > 1) {
      owner_n = a.tile_owner[tile_of(1)];
      req_n = a.tile_req[int64_t(tile_of(1)) * a.RT + j];
    }
    for (int it = 0; it < ntiles; ++it) {
      const int s = stage_of(it), rpar = round_par(it);
      if (!tc::mbar_wait(&q_empty[s], rpar ^ 1)) { s_fail = 1; break; }
      // rows of requests without a visible block are left as they are: their
      // results are never read.  Dimensions past D are zero-filled.
      const uint32_t stage = qs_addr + s * q_stage_bytes;
      for (int u = 0; u < (kRowsPerLoader << lgS) / 32; ++u) {
        const int f = u * 32 + lane;
        const int rl = f >> lgS, seg = f & (nseg - 1);
        const T* rs = reinterpret_cast<const T*>(__shfl_sync(kFull, reinterpret_cast<uintptr_t>(src), rl));
        if (rs != nullptr) {
          const int r = pw * kRowsPerLoader + rl, kc = seg >> 3, c = seg & 7;
          const uint32_t dst = stage + kc * 128 * 128 + r * 128 + ((c ^ (r & 7)) << 4);
          if (seg < dsegs) cp_async16(dst, rs + seg * 8);
          else cp_async16_zfill(dst, qbase);
        }
      }
      tc::cp_async_arrive(&q_full[s]);
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
          // The buffer being replaced was last read by tile it-2 or earlier:
          // wait for that P.V (with one TMEM buffer, the in-order issue makes
          // P.V of tile it-1 the one to wait for; it never needs tile it).
          if (kvb ? used1 : used0) {
            const int wt = nacc == 2 ? it - 2 : it - 1;
            bool freed = wt < 0;
            for (uint32_t i = 0; !freed && i < (1u << 24); ++i) {
              freed = ld_acquire_cta(&s_o_done) > wt;
              if (!freed && i >= 64) __nanosleep(32);
            }
            if (!freed) { s_fail = 1; break; }
          }
          if (kvb) used1 = 1; else used0 = 1;
          const uint32_t ks_addr = kv_addr + kvb * kv_bytes, vs_addr = ks_addr + qch * a.C * 128;
          if (lane < qch)
            tc::tma_load_4d(ks_addr + lane * a.C * 128, &a.tm_k, lane * 64, h, blk * a.C, b, &q_full[s]);
          else if (lane < qch + vch)
            tc::tma_load_4d(vs_addr + (lane - qch) * a.C * 128, &a.tm_v, (lane - qch) * 64, h, blk * a.C, b, &q_full[s]);
          bytes = uint32_t(qch + vch) * a.C * 128;
          cur_kv = kv_key;
        }
      }
      __syncwarp();
      if (lane == 0) {
        if (pw == 0) {
          s_kvb[s] = kvb;
          tc::mbar_arrive_expect_tx(&q_full[s], bytes);
        }
        tc::mbar_arrive(&meta_full[slot]);
      }
      __syncwarp();
      if (it + 1 < ntiles) {
        req = decode(owner_n, req_n);
        if (it + 2 < ntiles) {
          owner_n = a.tile_owner[tile_of(it + 2)];
          req_n = a.tile_req[int64_t(tile_of(it + 2)) * a.RT + j];
        }
      }
    }
    cp_async_wait_all();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issue ----------------
    if (lane == 0) {
      const uint32_t idesc_s = tc::idesc_f16(128, a.C, a.bf16);
      const uint32_t idesc_o = tc::idesc_f16(128, a.Dv, a.bf16, 1);
      int kv_even = 0, kv_odd = 0;  // K/V buffer of the last even / odd tile
      // S = Q K^T of tile `it` into its S/P buffer (its query stage has landed)
      auto issue_s = [&](int it) {
        const int s = stage_of(it), ab = acc_of(it);
        tc::fence_async_smem();
        tc::fence_after_sync();
        const int kvb = s_kvb[s];
        if (it & 1) kv_odd = kvb; else kv_even = kvb;
        const uint32_t ks_addr = kv_addr + kvb * kv_bytes;
        const uint32_t qa = qs_addr + s * q_stage_bytes;
        const uint32_t sacc = tmem + ab * a.sp_cols;
        for (int ks = 0; ks < a.Dp / 16; ++ks) {
          const int ch = ks >> 2, off = (ks & 3) * 32;
          tc::mma_f16(sacc, tc::desc_sw128(qa + ch * 128 * 128 + off),
                      tc::desc_sw128(ks_addr + ch * a.C * 128 + off), idesc_s, ks > 0);
        }
        tc::mma_commit(&s_full[ab]);
        tc::mma_commit(&q_empty[s]);
      };
      // O = P V of tile `pt` (its P is in TMEM and its O buffer was read out)
      auto issue_o = [&](int pt) {
        const int ab = acc_of(pt);
        tc::fence_after_sync();
        const uint32_t sp = tmem + ab * a.sp_cols;
        const uint32_t ob = tmem + nacc * a.sp_cols + ab * a.o_cols;
        const uint32_t vs_addr = kv_addr + ((pt & 1) ? kv_odd : kv_even) * kv_bytes + qch * a.C * 128;
        for (int ks = 0; ks < a.C / 16; ++ks) {
          const uint64_t vd = tc::desc_make(vs_addr + ks * 16 * 128, uint32_t(a.C) * 128, 1024, 2);
          tc::mma_f16_ts(ob, sp + a.C + ks * 8, vd, idesc_o, ks > 0);
        }
        tc::mma_commit(&o_full[ab]);
      };
      // Issue whichever of O(no) and S(ns) is ready, O first: P.V of a tile
      // never waits for the next tile's query rows.  Order rules (tensor-core
      // operations run in issue order): S(ns) overwrites the S/P buffer of
      // tile ns - nacc, so that tile's P.V must have been issued; O(no)
      // needs S(no) issued, P(no) in TMEM and its O buffer read out.
      int ns = 0, no = 0;
      uint32_t idle = 0;
      while (no < ntiles) {
        bool issued = false;
        if (no < ns) {
          const int ab = acc_of(no), ph = round_of(no) & 1;
          if (tc::mbar_test(&p_full[ab], ph) && tc::mbar_test(&o_empty[ab], ph ^ 1)) {
            issue_o(no++);
            issued = true;
          }
        }
        if (!issued && ns < ntiles && no >= ns - nacc + 1) {
          if (tc::mbar_test(&q_full[stage_of(ns)], round_par(ns))) {
            issue_s(ns++);
            issued = true;
          }
        }
        if (issued) {
          idle = 0;
        } else if (++idle > (1u << 24)) {
          s_fail = 1;
          break;
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: softmax warps 0-3, readout warps 4-7 ----------------
    // Both roles walk every tile: warps 0-3 turn S into P (and write the
    // row's (m, l)), warps 4-7 read O out; so the softmax of tile i+1 runs
    // while tile i's P.V and readout are in flight.
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t(quarter) * 32) << 16;
    const int r = row >> lgG;
    T* part_o = static_cast<T*>(a.part_o);
    const float l2e = 1.4426950408889634f;
    const float sl = a.scale * l2e;
    if (warp < 4) {
      for (int it = 0; it < ntiles; ++it) {
        const int ab = acc_of(it), rnd = round_of(it), tile = tile_of(it);
        const bool got = tc::mbar_wait(&s_full[ab], rnd & 1);
        if (!got) s_fail = 1;
        tc::fence_after_sync();
        if (!tc::mbar_wait(&meta_full[it & (kMeta - 1)], (it >> 4) & 1)) s_fail = 1;
        const int req = r < a.RT ? s_req[it & (kMeta - 1)][r] : -1;
        const int nvalid = r < a.RT ? s_nv[it & (kMeta - 1)][r] : 0;
        const uint32_t base = tmem + lane_base + ab * a.sp_cols;                 // S, then P at +C
        float mx = -INFINITY;
        float l = 0.f;
        if (a.C == 64) {
          // one TMEM load; masked keys -> -inf -> exp 0; packed arithmetic
          float v[64];
          tc::tmem_ld64(base, v);
          if (nvalid < 64) {
#pragma unroll
            for (int i = 0; i < 64; ++i) if (i >= nvalid) v[i] = -INFINITY;
          }
          mx = tc::max64(v);
          const float mb = nvalid > 0 ? mx * sl : 0.f;
          const float2 kk = make_float2(sl, sl), cc = make_float2(-mb, -mb);
          float2 acc2 = make_float2(0.f, 0.f);
          uint32_t w[32];
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const float2 x = tc::fma2(make_float2(v[i], v[i + 1]), kk, cc);
            const float2 pr = make_float2(tc::ex2f(x.x), tc::ex2f(x.y));
            acc2 = tc::add2(acc2, pr);
            w[i / 2] = pack2<T>(pr.x, pr.y);
          }
          l = acc2.x + acc2.y;
          uint32_t w0[16], w1[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) { w0[i] = w[i]; w1[i] = w[16 + i]; }
          tc::tmem_st16(base + a.C, w0);
          tc::tmem_st16(base + a.C + 16, w1);
        } else {
          for_columns(base, a.C, [&](int c, float x) {
            if (c < nvalid) mx = fmaxf(mx, x);
          });
          const float mb = mx * sl;
          for (int c0 = 0; c0 < a.C; c0 += 32) {
            if (a.C - c0 >= 32) {
              float v[32];
              tc::tmem_ld32(base + c0, v);
              uint32_t w[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float p0 = (c0 + 2 * i < nvalid) ? exp2f(fmaf(v[2 * i], sl, -mb)) : 0.f;
                const float p1 = (c0 + 2 * i + 1 < nvalid) ? exp2f(fmaf(v[2 * i + 1], sl, -mb)) : 0.f;
                l += p0 + p1;
                w[i] = pack2<T>(p0, p1);
              }
              tc::tmem_st16(base + a.C + c0 / 2, w);
            } else {
              float v[16];
              tc::tmem_ld16(base + c0, v);
              uint32_t w[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float p0 = (c0 + 2 * i < nvalid) ? exp2f(fmaf(v[2 * i], sl, -mb)) : 0.f;
                const float p1 = (c0 + 2 * i + 1 < nvalid) ? exp2f(fmaf(v[2 * i + 1], sl, -mb)) : 0.f;
                l += p0 + p1;
                w[i] = pack2<T>(p0, p1);
              }
              tc::tmem_st8(base + a.C + c0 / 2, w);
            }
          }
        }
        // the row's block max (scaled) and sum of exponentials
        if (req >= 0)
          __stcs(reinterpret_cast<float2*>(a.part_ml) + int64_t(req) * a.G + (row & (a.G - 1)),
                 make_float2(mx * a.scale, l));
        // one arrival per warp once all its lanes' TMEM stores are done
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&p_full[ab]);
        if (!got) break;
      }
    } else {
      // block-local partial O = sum_k exp(s_k - m) v_k (not divided by l) of
      // the row's request and head, query-major: row request * G + head.
      // Thread = row in TMEM, but a warp store of one value slice per row
      // would touch 32 lines; so each 64-value slice of the warp's 32 rows is
      // staged in shared memory (16-byte chunks XOR-swizzled by row) and
      // written back as 8 warp stores of 4 rows x 128 contiguous bytes.
      const uint32_t stg = tc::smem_u32(smem + nst * q_stage_bytes + 2 * kv_bytes) + quarter * 4096;
      const int srow = lane >> 3, schunk = lane & 7;  // copy-out: row (of 4) and 16-byte chunk
      for (int it = 0; it < ntiles; ++it) {
        const int ab = acc_of(it), rnd = round_of(it);
        const bool got = tc::mbar_wait(&o_full[ab], rnd & 1);
        if (!got) s_fail = 1;
        tc::fence_after_sync();
        if (warp == 4 && lane == 0) st_release_cta(&s_o_done, it + 1);
        if (!tc::mbar_wait(&meta_full[it & (kMeta - 1)], (it >> 4) & 1)) s_fail = 1;
        const int req = r < a.RT ? s_req[it & (kMeta - 1)][r] : -1;
        const uint32_t obase = tmem + lane_base + nacc * a.sp_cols + ab * a.o_cols;
        // this lane's partial row, or null (request without a visible block)
        T* prow = req >= 0 ? part_o + (int64_t(req) * a.G + (row & (a.G - 1))) * a.Dv : nullptr;
        for (int c0 = 0; c0 < a.Dv; c0 += 64) {
          const int ncol = min(64, a.Dv - c0);     // 32 or 64 (Dv % 32 == 0)
          // stage: row = lane, 16-byte chunk c at (c ^ (lane & 7)); 32 values at a time
          for (int half = 0; half < ncol / 32; ++half) {
            float v[32];
            tc::tmem_ld32(obase + c0 + 32 * half, v);
            if (c0 + 32 * half + 32 >= a.Dv) {
              // every TMEM load of this tile has completed: release the O buffer
              tc::fence_before_sync();
              __syncwarp();
              if (lane == 0) tc::mbar_arrive(&o_empty[ab]);
            }
#pragma unroll
            for (int c = 0; c < 4; ++c)
              st_shared16(stg + lane * 128 + (((4 * half + c) ^ (lane & 7)) << 4), pack2<T>(v[8 * c], v[8 * c + 1]),
                          pack2<T>(v[8 * c + 2], v[8 * c + 3]), pack2<T>(v[8 * c + 4], v[8 * c + 5]),
                          pack2<T>(v[8 * c + 6], v[8 * c + 7]));
          }
          __syncwarp();
          // copy out: warp store k covers rows 4k..4k+3, lane -> (row, chunk)
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int rr = 4 * k + srow;
            const T* dst = reinterpret_cast<const T*>(__shfl_sync(kFull, reinterpret_cast<uintptr_t>(prow), rr));
            if (dst != nullptr && schunk * 8 < ncol) {
              uint32_t x0, x1, x2, x3;
              ld_shared16(stg + rr * 128 + ((schunk ^ (rr & 7)) << 4), x0, x1, x2, x3);
              st_cs16(const_cast<T*>(dst) + c0 + schunk * 8, x0, x1, x2, x3);
            }
          }
          __syncwarp();
        }
        if (!got) break;
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (tid == 0 && s_fail) atomicExch(a.status, PISA_ERR_TIMEOUT);
  if (warp == 0) tc::tmem_free(tmem, a.tmem_cols);
}

// Merge the S block partials of each query head into its output row and LSE.
// One warp per (batch, token, KV head, group of hpw heads): the partials of a
// (token, KV head) are contiguous (request-major, heads inner), so one warp
// instruction reads 32 x 32 bytes = 32 / NCG whole rows.  Lane = (replica,
// head, column group of 16 values); replicas take every R-th slot and are
// summed at the end.  Pass 1 turns each head's S (m, l) pairs into weights
// exp(m_s - M) (kept in shared memory) and the normaliser L.
template <typename T, int NCG>
__global__ void __launch_bounds__(128) attn_combine_kernel(const AttnTcArgs a) {
  __shared__ float s_w[4][64][16];           // [warp][slot][head of the warp]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hpw = min(a.G, 32 / NCG);        // heads per warp (power of two)
  const int wpr = a.G / hpw;                 // warps per (token, KV head)
  const uint32_t idx = blockIdx.x * 4u + uint32_t(warp);
  if (idx >= uint32_t(a.B) * uint32_t(a.tlen) * uint32_t(a.H) * uint32_t(wpr)) return;
  const uint32_t row = idx / uint32_t(wpr);  // (b, tl, h), wpr a power of two
  const int gsub = int(idx - row * uint32_t(wpr));
  const uint32_t r1 = a.fH.div(row), r2 = a.ftlen.div(r1);
  const int h = int(row - r1 * uint32_t(a.H));
  const int tl = int(r1 - r2 * uint32_t(a.tlen));
  const int b = int(r2);
  const int t = a.t0 + tl;
  const int64_t lr0 = int64_t(row) * a.S;    // chunk-local request of slot 0
  const int g0 = gsub * hpw;
  const T* part_o = static_cast<const T*>(a.part_o);
  const float2* part_ml = reinterpret_cast<const float2*>(a.part_ml);

  // slots this lane checks in pass 1: s = lane, lane + 32
  bool vis[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int sl = lane + 32 * k;
    vis[k] = sl < a.S && visible_block(a, b, t, h, sl) >= 0;
  }
  float my_M = -INFINITY, my_L = 0.f;
  const int g_lane = (lane / NCG) & (hpw - 1);
  for (int gl = 0; gl < hpw; ++gl) {
    float m_s[2] = {-INFINITY, -INFINITY}, l_s[2] = {0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (vis[k]) {
        const float2 ml = __ldcs(part_ml + (lr0 + lane + 32 * k) * a.G + g0 + gl);
        if (ml.y > 0.f) { m_s[k] = ml.x; l_s[k] = ml.y; }
      }
    }
    const float M = warp_max(fmaxf(m_s[0], m_s[1]));
    float lw = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float w = (M == -INFINITY || m_s[k] == -INFINITY) ? 0.f : expf(m_s[k] - M);
      lw += l_s[k] * w;
      const int sl = lane + 32 * k;
      if (sl < a.S) s_w[warp][sl][gl] = w;
    }
    const float L = warp_sum(lw);
    if (gl == g_lane) { my_M = M; my_L = L; }
  }
  __syncwarp();

  const int cg = lane % NCG;
  const int R = 32 / (NCG * hpw);            // replicas
  const int rep = lane / (NCG * hpw);
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  const T* base = part_o + (lr0 * a.G + g0 + g_lane) * a.Dv + cg * 16;
  const int64_t slot_stride = int64_t(a.G) * a.Dv;
  constexpr int kLoads = 4;
  for (int s0 = rep; s0 < a.S; s0 += kLoads * R) {
    float w[kLoads];
    uint32_t raw[kLoads][8];
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
      const int sl = s0 + u * R;
      w[u] = sl < a.S ? s_w[warp][sl][g_lane] : 0.f;
      if (w[u] > 0.f) {
        ld_cs32(base + sl * slot_stride, raw[u]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) raw[u][i] = 0u;
      }
    }
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
      const T* e = reinterpret_cast<const T*>(raw[u]);
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = fmaf(w[u], to_f32<T>(e[i]), acc[i]);
    }
  }
  for (int o = NCG * hpw; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] += __shfl_xor_sync(kFull, acc[i], o);
  if (rep == 0) {
    const int hq = h * a.G + g0 + g_lane;
    T* out = static_cast<T*>(a.out) + ((int64_t(b) * a.T + t) * a.Hq + hq) * a.Dv;
    const float inv = my_L > 0.f ? 1.f / my_L : 0.f;
    uint32_t wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) wv[i] = pack2<T>(acc[2 * i] * inv, acc[2 * i + 1] * inv);
    uint4* dst = reinterpret_cast<uint4*>(out + cg * 16);
    dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
    if (cg == 0 && a.lse) a.lse[(int64_t(b) * a.T + t) * a.Hq + hq] = my_L > 0.f ? my_M + logf(my_L) : -INFINITY;
  }
}

template <typename T>
int attn_tc_typed(AttnTcArgs a, cudaStream_t stream) {
  const int qch = a.Dp / 64, vch = a.Dvp / 64;
  // query stages, two K/V buffers, the readout's staging (4 warps x 32 rows x 128 B)
  const size_t smem = size_t(a.nstages) * 128 * 128 * qch + size_t(2) * a.C * 128 * (qch + vch) + 16384 + 1024;
  cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return fail_cuda(e, "attention smem attribute");
  a.fS = FastDiv::make(uint32_t(a.S));
  a.fH = FastDiv::make(uint32_t(a.H));
  a.fHq = FastDiv::make(uint32_t(a.Hq));
  a.fNB = FastDiv::make(uint32_t(a.NB));
  a.fTW = FastDiv::make(uint32_t(a.TW));
  a.fRT = FastDiv::make(uint32_t(a.RT));
  for (int t0 = 0; t0 < a.T; t0 += a.chunk) {
    const int rc = attn_bucket_chunk(a, t0, stream);
    if (rc != PISA_OK) return rc;
    {
      TimedLaunch timed(PISA_KERNEL_ATTN_TILES, stream);
      attn_tc_kernel<T><<<unsigned(a.num_sms), kPipeThreads, smem, stream>>>(a);
      PISA_CHECK_LAUNCH();
    }
    const int ncg = a.Dv / 16;
    const int hpw = std::min(a.G, 32 / ncg);
    const unsigned cgrid = unsigned((int64_t(a.B) * a.tlen * a.H * (a.G / hpw) + 3) / 4);
    {
      TimedLaunch timed(PISA_KERNEL_ATTN_COMBINE, stream);
      switch (ncg) {
        case 2: attn_combine_kernel<T, 2><<<cgrid, 128, 0, stream>>>(a); break;
        case 4: attn_combine_kernel<T, 4><<<cgrid, 128, 0, stream>>>(a); break;
        case 8: attn_combine_kernel<T, 8><<<cgrid, 128, 0, stream>>>(a); break;
        default: attn_combine_kernel<T, 16><<<cgrid, 128, 0, stream>>>(a); break;
      }
      PISA_CHECK_LAUNCH();
    }
  }
  return PISA_OK;
}

}  // namespace

int attn_bucket_chunk(AttnTcArgs& a, int t0, cudaStream_t stream) {
  a.t0 = t0;
  a.tlen = std::min(a.chunk, a.T - t0);
  a.nwin = (a.tlen + a.TW - 1) / a.TW;
  a.ftlen = FastDiv::make(uint32_t(a.tlen));
  a.fnwin = FastDiv::make(uint32_t(a.nwin));
  a.num_buckets = int64_t(a.B) * a.nwin * a.H * a.NB;
  const int64_t reqs = int64_t(a.B) * a.tlen * a.H * a.S;
  a.capacity = (reqs + a.RT - 1) / a.RT + a.num_buckets;
  cudaError_t e = cudaMemsetAsync(a.counts, 0, sizeof(int32_t) * a.num_buckets, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(a.cursors, 0, sizeof(int32_t) * a.num_buckets, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(a.tile_req, 0xFF, sizeof(int32_t) * a.capacity * a.RT, stream);
  if (e != cudaSuccess) return fail_cuda(e, "attention bucket clear");
  const unsigned grid = unsigned((reqs + 255) / 256);
  attn_count_kernel<<<grid, 256, 0, stream>>>(a);
  PISA_CHECK_LAUNCH();
  e = launch_tile_scan(a.counts, a.offsets, a.total_tiles, a.num_buckets, a.RT, stream);
  if (e != cudaSuccess) return fail_cuda(e, "attention tile scan");
  attn_scatter_kernel<<<grid, 256, 0, stream>>>(a);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

int attn_fwd_tc(const AttnTcArgs& a, int dtype, cudaStream_t stream) {
  if (dtype == PISA_BF16) return attn_tc_typed<__nv_bfloat16>(a, stream);
  if (dtype == PISA_F16) return attn_tc_typed<__half>(a, stream);
  return fail(PISA_ERR_UNSUPPORTED, "tensor-core attention needs fp16 or bf16");
}

}  // namespace pisa
