// K3: grouped leaf scoring on the tensor cores, and the final top-K.
//
// The coarse router leaves, for every (batch, token, KV head) row, W0 = b*K
// leaf candidates: the b children of each of its K level-1 survivors
// ("families", in network order).  Scoring a candidate needs the query's G
// head rows and the candidate block's C keys (top_k_pyramid_torch.py:48-80;
// grouped_leaf_kernel, leaf_triton.py:63-141, does the same with four queries
// per key-block load).
//
// Here requests are (row, family) pairs bucketed by (batch, token window, KV
// head, survivor id): one tile = up to 128/G requests of one bucket, so one
// tcgen05 MMA multiplies the tile's 128 query-head rows (gathered once, 1 KiB
// per request at G=4, D=128) by the family's b*C contiguous keys (staged once
// per run of tiles of the bucket).  The token window keeps the queries of the
// tiles in flight resident in L2.  Accumulators land in TMEM; the epilogue
// (one thread per TMEM lane = query-head row) reduces each child's C columns
// to an LSE (pisa) or mean/variance (pisa2) score, sums the G heads with warp
// shuffles, and scatters the b scores to the request's candidate slots.
//
// Bucketing is count -> scan -> scatter on the device with no host sync:
// the tile list has a fixed capacity and the kernels read the real count.
#include <algorithm>

#include "bucket.cuh"
#include "internal.h"
#include "tc.cuh"

namespace pisa {

namespace {

// (batch, token, KV head) of a row index b*T*H + t*H + h (rows < 2^31)
__device__ __forceinline__ void decode_row(const GroupArgs& g, uint32_t row, int& b, int& t, int& h) {
  const uint32_t r1 = g.fH.div(row), r2 = g.fT.div(r1);
  h = int(row - r1 * uint32_t(g.H));
  t = int(r1 - r2 * uint32_t(g.T));
  b = int(r2);
}

// Requests: one per (row, family) with at least one scoreable child.
__global__ void family_count_kernel(const GroupArgs g, int32_t* __restrict__ counts) {
  const int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  const int64_t total = int64_t(g.B) * g.T * g.H * g.NF;
  if (idx >= total) return;
  const uint32_t row = g.fNF.div(uint32_t(idx));
  const int k = int(uint32_t(idx) - row * uint32_t(g.NF));
  const uint8_t* f = g.flags + int64_t(row) * g.W0 + k * g.br;
  bool active = false;
  for (int j = 0; j < g.br; ++j) active |= (f[j] & 4) != 0;
  if (!active) return;
  int b, t, h;
  decode_row(g, row, b, t, h);
  const int p = int(g.fbr.div(uint32_t(g.cand[int64_t(row) * g.W0 + k * g.br])));
  const int64_t bucket = ((int64_t(b) * g.nwin + int(g.fTW.div(uint32_t(t)))) * g.H + h) * g.NP + p;
  atomicAdd(counts + bucket, 1);
}

__global__ void family_scatter_kernel(const GroupArgs g, const int32_t* __restrict__ offsets,
                                      int32_t* __restrict__ cursors, int32_t* __restrict__ tile_owner,
                                      int32_t* __restrict__ tile_req) {
  const int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  const int64_t total = int64_t(g.B) * g.T * g.H * g.NF;
  if (idx >= total) return;
  const uint32_t row = g.fNF.div(uint32_t(idx));
  const int k = int(uint32_t(idx) - row * uint32_t(g.NF));
  const uint8_t* f = g.flags + int64_t(row) * g.W0 + k * g.br;
  bool active = false;
  for (int j = 0; j < g.br; ++j) active |= (f[j] & 4) != 0;
  if (!active) return;
  int b, t, h;
  decode_row(g, row, b, t, h);
  const int p = int(g.fbr.div(uint32_t(g.cand[int64_t(row) * g.W0 + k * g.br])));
  const int64_t bucket = ((int64_t(b) * g.nwin + int(g.fTW.div(uint32_t(t)))) * g.H + h) * g.NP + p;
  const int pos = atomicAdd(cursors + bucket, 1);
  const int q = int(g.fRT.div(uint32_t(pos))), r = pos - q * g.RT;
  const int64_t tile = offsets[bucket] + q;
  tile_req[tile * g.RT + r] = int32_t(idx);
  if (r == 0) tile_owner[tile] = int32_t(bucket);
}

// Warp roles of the pipelined tile kernel (one persistent CTA per SM):
//   warps 0-7   epilogue: warp w reads TMEM lanes 32*(w%4).. (one query-head
//               row per thread) and handles half of the b children
//               (warps 0-3 the first ceil(b/2), warps 4-7 the rest)
//   next kLoadWarps warps  producers: gather the tile's query rows into a
//               3-stage ring (cp.async), restage the family keys (TMA) when the
//               bucket changes
//   last warp   MMA issue (one thread): tile i accumulates into TMEM buffer i%2
// mbarriers: full_q/empty_q guard the query stages, full_acc/empty_acc the
// accumulators; the parity of round r is r & 1 (empty waits start at 1, so the
// first round passes).  Every wait is bounded and records a timeout status.
// Epilogue warps come in groups of four (one per TMEM lane quarter); group g
// scores children [g*b/groups, (g+1)*b/groups) of every tile.
// (Two groups, each thread scoring two children with interleaved chains,
// measured faster than four groups of one child each: 3.06 against 3.36 ms
// per 32K step.)
#ifndef PISA_LEAF_EPI_GROUPS
#define PISA_LEAF_EPI_GROUPS 2
#endif
constexpr int kEpiGroups = PISA_LEAF_EPI_GROUPS;
constexpr int kEpiWarps = 4 * kEpiGroups, kLoadWarps = 4, kMmaWarp = kEpiWarps + kLoadWarps, kStages = 3, kGroup = 8;
constexpr int kRowsPerLoader = 128 / kLoadWarps;  // tile rows per producer warp
constexpr int kPipeThreads = (kMmaWarp + 1) * 32;
// Of every four pairs of LSE exponentials in the two-children epilogue, this
// many are evaluated by tc::ex2_poly2 on the FMA pipe, the rest by ex2.approx.
// Measured per 32K step: 0 -> 3.04 ms, 1 -> 3.30, 2 -> 3.52, 3 -> 3.95; the
// epilogue is bound by its dependency latency, not by the MUFU unit's rate.
#ifndef PISA_LEAF_POLY_PAIRS
#define PISA_LEAF_POLY_PAIRS 0
#endif
constexpr int kPolyPairs = PISA_LEAF_POLY_PAIRS;

template <typename T, int KB>
__global__ void __launch_bounds__(kPipeThreads, 1) leaf_tc_kernel(const __grid_constant__ GroupArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int Dp = g.Dp;                       // padded head_dim: 64, 128 or 256
  const int chunks = Dp / 64;                // 128-byte K chunks per row
  const int NK = g.br * g.C;                 // keys per family = MMA N
  const int q_stage_bytes = chunks * 128 * 128;
  // query stages: 3, or 2 with two key buffers (decode-like runs of one tile
  // per family, whose next keys then load while the current tile is scored)
  constexpr int nst = KB == 2 ? 2 : kStages;
  auto stage_of = [](int i) { return i % nst; };
  auto round_of = [](int i) { return i / nst; };
  uint8_t* Ks = smem + nst * q_stage_bytes;        // kbufs x [chunks][NK][128 B]
  const uint32_t kbuf_bytes = uint32_t(chunks) * NK * 128;
  __shared__ uint64_t full_q[kStages], empty_q[kStages], full_acc[2], empty_acc[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int s_fail;
  // per-tile metadata ring for the epilogue (8 slots): the producer runs at
  // most kStages tiles ahead of the MMAs and they at most two ahead of the
  // epilogue, so slot it%8 is free again when tile it is produced
  __shared__ uint64_t meta_full[8];
  __shared__ int s_dst[8][128], s_fam[8], s_kb[8];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = *g.total_tiles;
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

  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      // one cp.async arrival per producer thread + the key arrival of the first producer warp
      tc::mbar_init(&full_q[i], kLoadWarps * 32 + 1);
      tc::mbar_init(&empty_q[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&full_acc[i], 1);
      tc::mbar_init(&empty_acc[i], kEpiWarps);
    }
    for (int i = 0; i < 8; ++i) tc::mbar_init(&meta_full[i], kLoadWarps);
    s_fail = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, g.tmem_cols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const int nacc = g.tmem_cols >= 2 * NK ? 2 : 1;
  const uint32_t qs_addr = tc::smem_u32(smem), ks_addr = tc::smem_u32(Ks);
  const int lgG = 31 - __clz(g.G);

  if (warp >= kEpiWarps && warp < kMmaWarp) {
    // ---------------- producer warps ----------------
    // Query rows move with 16-byte asynchronous copies (cp.async) into their
    // swizzled K-major positions; each producer thread's copies arrive on the
    // stage barrier when they land.  Producer warp pw owns kRowsPerLoader
    // tile rows and lane l decodes the request of its l-th row.  Producer
    // warp 0 also restages a new family's b*C keys through TMA (one box per
    // 64-dim chunk, zero past the sequence end); those bytes count on the
    // same barrier.
    const int pw = warp - kEpiWarps;
    const int row = pw * kRowsPerLoader + (lane & (kRowsPerLoader - 1));
    const int j = row >> lgG, gq = row & (g.G - 1);
    const int lgS = 31 - __clz(Dp / 8);
    const int nseg = 1 << lgS, dsegs = g.D / 8;
    const T* qbase = static_cast<const T*>(g.q);
    int cur_key = -1, kb = 0;
    int last_use0 = -1, last_use1 = -1;   // last tile that reads each key buffer
    // request of this lane's row in tile `it` (family coordinates, source
    // row, score slot), decoded one tile ahead while the previous tile's
    // copies drain
    int p = 0, h = 0, b = 0, dst = -1;
    const T* src = nullptr;
    auto decode = [&](int owner, int req) {
      const uint32_t o1 = g.fNP.div(uint32_t(owner)), o2 = g.fH.div(o1);
      p = owner - int(o1) * g.NP;
      h = int(o1) - int(o2) * g.H;
      b = int(g.fnwin.div(o2));
      src = nullptr;
      dst = -1;
      if (req >= 0) {
        const int rowid = int(g.fNF.div(uint32_t(req)));
        int bb, t, hh;
        decode_row(g, uint32_t(rowid), bb, t, hh);
        dst = rowid * g.W0 + (req - rowid * g.NF) * g.br;
        src = qbase + int64_t(bb) * g.q_sb + int64_t(t) * g.q_st + int64_t(hh * g.G + gq) * g.q_sh;
      }
    };
    decode(g.tile_owner[first], g.tile_req[int64_t(first) * g.RT + j]);
    // the next tile's owner and request index are loaded one iteration early
    int owner_n = 0, req_n = -1;
    if (ntiles > 1) {
      owner_n = g.tile_owner[tile_of(1)];
      req_n = g.tile_req[int64_t(tile_of(1)) * g.RT + j];
    }
    for (int it = 0; it < ntiles; ++it) {
      const int s = stage_of(it), rnd = round_of(it);
      if (!tc::mbar_wait(&empty_q[s], (rnd & 1) ^ 1)) { s_fail = 1; break; }
      // rows of empty request slots are left as they are (their scores are
      // never written); dimensions past D are zero-filled
      const uint32_t stage = qs_addr + s * q_stage_bytes;
      for (int u = 0; u < (kRowsPerLoader << lgS) / 32; ++u) {
        const int f = u * 32 + lane;
        const int rl = f >> lgS, seg = f & (nseg - 1);
        const T* rs = reinterpret_cast<const T*>(__shfl_sync(kFull, reinterpret_cast<uintptr_t>(src), rl));
        if (rs != nullptr) {
          const int r = pw * kRowsPerLoader + rl, kc = seg >> 3, c = seg & 7;
          const uint32_t dsta = stage + kc * 128 * 128 + r * 128 + ((c ^ (r & 7)) << 4);
          if (seg < dsegs) cp_async16(dsta, rs + seg * 8);
          else cp_async16_zfill(dsta, qbase);
        }
      }
      tc::cp_async_arrive(&full_q[s]);
      const int slot = it & 7;
      if (gq == 0 && lane < kRowsPerLoader) s_dst[slot][j] = dst;
      uint32_t bytes = 0;
      if (pw == 0) {
        const int kkey = (b * g.H + h) * g.NP + p;
        if (kkey != cur_key) {
          // the last tile that read the buffer being refilled must have
          // finished its MMAs; tiles up to it - nst are (the stage wait
          // above), and a later one is at most one phase ahead on its stage
          const int nb = KB == 2 ? kb ^ 1 : 0;
          const int lu = nb ? last_use1 : last_use0;
          if (lu >= 0 && lu > it - nst &&
              !tc::mbar_wait(&empty_q[stage_of(lu)], round_of(lu) & 1)) { s_fail = 1; break; }
          if (lane < chunks)
            tc::tma_load_4d(ks_addr + nb * kbuf_bytes + lane * NK * 128, &g.tm_k, lane * 64, h, p * NK, b,
                            &full_q[s]);
          bytes = kbuf_bytes;
          cur_key = kkey;
          kb = nb;
        }
        if (kb) last_use1 = it; else last_use0 = it;
      }
      __syncwarp();
      if (lane == 0) {
        if (pw == 0) {
          s_fam[slot] = p;
          s_kb[slot] = kb;
          tc::mbar_arrive_expect_tx(&full_q[s], bytes);
        }
        tc::mbar_arrive(&meta_full[slot]);
      }
      __syncwarp();
      if (it + 1 < ntiles) {
        decode(owner_n, req_n);
        if (it + 2 < ntiles) {
          owner_n = g.tile_owner[tile_of(it + 2)];
          req_n = g.tile_req[int64_t(tile_of(it + 2)) * g.RT + j];
        }
      }
    }
    cp_async_wait_all();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issue ----------------
    if (lane == 0) {
      for (int it = 0; it < ntiles; ++it) {
        const int s = stage_of(it), a = nacc == 2 ? (it & 1) : 0;
        const int ra = nacc == 2 ? (it >> 1) : it;
        if (!tc::mbar_wait(&full_q[s], round_of(it) & 1)) { s_fail = 1; break; }
        if (!tc::mbar_wait(&empty_acc[a], (ra & 1) ^ 1)) { s_fail = 1; break; }
        tc::fence_async_smem();
        tc::fence_after_sync();
        const uint32_t acc = tmem + a * NK;
        const uint32_t qa = qs_addr + s * q_stage_bytes;
        const uint32_t kbase = KB == 2 ? ks_addr + uint32_t(s_kb[it & 7]) * kbuf_bytes : ks_addr;
        for (int n0 = 0; n0 < NK; n0 += 256) {
          const int n = min(256, NK - n0);
          const uint32_t idesc = tc::idesc_f16(128, n, g.bf16);
          for (int ks = 0; ks < Dp / 16; ++ks) {
            const int ch = ks >> 2, off = (ks & 3) * 32;
            tc::mma_f16(acc + n0, tc::desc_sw128(qa + ch * 128 * 128 + off),
                        tc::desc_sw128(kbase + ch * NK * 128 + n0 * 128 + off), idesc, ks > 0);
          }
        }
        tc::mma_commit(&full_acc[a]);
        tc::mma_commit(&empty_q[s]);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3, group = warp >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t(quarter) * 32) << 16;
    const int r = row >> lgG;
    const int j_begin = group * g.br / kEpiGroups, j_end = (group + 1) * g.br / kEpiGroups;
    const float l2e = 1.4426950408889634f;
    const float sl = g.scale * l2e;          // exp(scale*x - m) = 2^(x*sl - m*l2e)
    for (int it = 0; it < ntiles; ++it) {
      const int tile = tile_of(it);
      const int a = nacc == 2 ? (it & 1) : 0;
      const int ra = nacc == 2 ? (it >> 1) : it;
      const bool got = tc::mbar_wait(&full_acc[a], ra & 1);
      if (!got) s_fail = 1;
      tc::fence_after_sync();
      if (!tc::mbar_wait(&meta_full[it & 7], (it >> 3) & 1)) s_fail = 1;
      const int p = s_fam[it & 7];
      const int dst = r < g.RT ? s_dst[it & 7][r] : -1;
      (void)tile;
      const uint32_t acc = tmem + lane_base + a * NK;
      // a warp whose 32 rows hold no request (the tail of a bucket's last
      // tile; decode tiles carry only G rows) has no scores to compute
      const bool live = __any_sync(kFull, dst >= 0);
      int j_first = live ? j_begin : j_end;
      if (live && kEpiGroups < 4 && g.C == 64 && g.method == PISA_METHOD_PISA && j_end - j_begin >= 2 &&
          (int64_t(p) * g.br + j_begin + 2) * 64 <= g.N) {
        // two full 64-key children at once: both TMEM loads in flight, then the
        // two max / exponential chains interleaved
        uint32_t r0[64], r1[64];
        tc::tmem_ld64_nowait(acc + j_begin * 64, r0);
        tc::tmem_ld64_nowait(acc + (j_begin + 1) * 64, r1);
        tc::tmem_wait_ld2(r0, r1);
        // row maxima with four independent three-input chains per child
        float ma[4], mb[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) { ma[c] = __uint_as_float(r0[c]); mb[c] = __uint_as_float(r1[c]); }
#pragma unroll
        for (int i = 4; i < 64; i += 8) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            ma[c] = tc::max3f(ma[c], __uint_as_float(r0[i + 2 * c]), __uint_as_float(r0[i + 2 * c + 1]));
            mb[c] = tc::max3f(mb[c], __uint_as_float(r1[i + 2 * c]), __uint_as_float(r1[i + 2 * c + 1]));
          }
        }
        const float m0 = fmaxf(tc::max3f(ma[0], ma[1], ma[2]), ma[3]);
        const float m1 = fmaxf(tc::max3f(mb[0], mb[1], mb[2]), mb[3]);
        const float2 kk = make_float2(sl, sl), c0 = make_float2(-m0 * sl, -m0 * sl), c1 = make_float2(-m1 * sl, -m1 * sl);
        float2 s0 = make_float2(0.f, 0.f), s1 = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          const float2 x0 = tc::fma2(make_float2(__uint_as_float(r0[i]), __uint_as_float(r0[i + 1])), kk, c0);
          const float2 x1 = tc::fma2(make_float2(__uint_as_float(r1[i]), __uint_as_float(r1[i + 1])), kk, c1);
          if (((i >> 1) & 3) < kPolyPairs) {
            // this pair on the FMA pipe (the MUFU unit bounds the epilogue)
            s0 = tc::add2(s0, tc::ex2_poly2(x0));
            s1 = tc::add2(s1, tc::ex2_poly2(x1));
          } else {
            s0 = tc::add2(s0, make_float2(tc::ex2f(x0.x), tc::ex2f(x0.y)));
            s1 = tc::add2(s1, make_float2(tc::ex2f(x1.x), tc::ex2f(x1.y)));
          }
        }
        float sc0 = m0 * g.scale + logf(s0.x + s0.y), sc1 = m1 * g.scale + logf(s1.x + s1.y);
        for (int o = 1; o < g.G; o <<= 1) {
          sc0 += __shfl_xor_sync(kFull, sc0, o);
          sc1 += __shfl_xor_sync(kFull, sc1, o);
        }
        if (dst >= 0 && (row & (g.G - 1)) == 0) {
          g.scores[int64_t(dst) + j_begin] = sc0;
          g.scores[int64_t(dst) + j_begin + 1] = sc1;
        }
        j_first = j_begin + 2;
      }
      for (int j = j_first; j < j_end; ++j) {
        const int64_t key0 = (int64_t(p) * g.br + j) * g.C;
        const int valid_keys = int(min64(g.C, max(int64_t(0), g.N - key0)));
        float score;
        if (kEpiGroups == 4 && g.C == 64 && valid_keys == 64) {
          // full 64-key block in two 32-column halves (32 live values: the
          // 16 epilogue warps leave at most 80 registers a thread); the LSE
          // merges the halves' maxima, the moments simply add
          float v[32];
          tc::tmem_ld32(acc + j * 64, v);
          if (g.method == PISA_METHOD_PISA) {
            const float m1 = tc::max32(v);
            const float s1 = tc::sum_ex2_32(v, sl, m1 * sl);
            tc::tmem_ld32(acc + j * 64 + 32, v);
            const float mx = fmaxf(m1, tc::max32(v));
            const float sum = fmaf(s1, tc::ex2f((m1 - mx) * sl), tc::sum_ex2_32(v, sl, mx * sl));
            score = mx * g.scale + logf(sum);
          } else {
            float2 a1 = make_float2(0.f, 0.f), a2 = make_float2(0.f, 0.f);
            for (int hh = 0; hh < 2; ++hh) {
              if (hh) tc::tmem_ld32(acc + j * 64 + 32, v);
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const float2 pv = make_float2(v[i], v[i + 1]);
                a1 = tc::add2(a1, pv);
                a2 = tc::fma2(pv, pv, a2);
              }
            }
            const float mean = (a1.x + a1.y) / 64.f;
            const float var = fmaxf((a2.x + a2.y) / 64.f - mean * mean, 0.f);
            score = g.scale * mean + g.c2 * var;
          }
        } else if (kEpiGroups < 4 && g.C == 64 && valid_keys == 64) {
          // full 64-key block: one TMEM load, packed arithmetic, no masks
          float v[64];
          tc::tmem_ld64(acc + j * 64, v);
          if (g.method == PISA_METHOD_PISA) {
            const float mx = tc::max64(v);
            score = mx * g.scale + logf(tc::sum_ex2_64(v, sl, mx * sl));
          } else {
            float2 a1 = make_float2(0.f, 0.f), a2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 64; i += 2) {
              const float2 pv = make_float2(v[i], v[i + 1]);
              a1 = tc::add2(a1, pv);
              a2 = tc::fma2(pv, pv, a2);
            }
            const float mean = (a1.x + a1.y) / 64.f;
            const float var = fmaxf((a2.x + a2.y) / 64.f - mean * mean, 0.f);
            score = g.scale * mean + g.c2 * var;
          }
        } else if (g.method == PISA_METHOD_PISA) {
          float mx = -INFINITY;
          for_columns(acc + j * g.C, g.C, [&](int cc, float x) {
            if (cc < valid_keys) mx = fmaxf(mx, x);
          });
          const float mb = mx * sl;
          float sum = 0.f;
          for_columns(acc + j * g.C, g.C, [&](int cc, float x) {
            if (cc < valid_keys) sum += exp2f(fmaf(x, sl, -mb));
          });
          score = mx * g.scale + logf(sum);
        } else {
          float s1 = 0.f, s2 = 0.f;
          for_columns(acc + j * g.C, g.C, [&](int cc, float x) {
            if (cc < valid_keys) { s1 += x; s2 = fmaf(x, x, s2); }
          });
          const float n = float(valid_keys > 0 ? valid_keys : 1);
          const float mean = s1 / n, var = fmaxf(s2 / n - mean * mean, 0.f);
          score = g.scale * mean + g.c2 * var;
        }
        if (valid_keys == 0) score = 0.f;
        for (int o = 1; o < g.G; o <<= 1) score += __shfl_xor_sync(kFull, score, o);
        if (dst >= 0 && (row & (g.G - 1)) == 0) g.scores[int64_t(dst) + j] = score;
      }
      // one arrival per warp once all its lanes' TMEM loads are done
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty_acc[a]);
      if (!got) break;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (tid == 0 && s_fail) atomicExch(g.status, PISA_ERR_TIMEOUT);
  if (warp == 0) tc::tmem_free(tmem, g.tmem_cols);
}

// Final top-K over the W0 leaf candidates of each row (final_kernel,
// top_k_pyramid_triton.py:279-308): fill, bitonic network, causal mask.
template <int WP>
__global__ void __launch_bounds__(128) leaf_final_kernel(const GroupArgs g) {
  const int64_t row = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t rows = int64_t(g.B) * g.T * g.H;
  if (row >= rows) return;
  int b, t, h;
  decode_row(g, uint32_t(row), b, t, h);
  const int64_t pos = g.positions ? g.positions[int64_t(b) * g.T + t] : g.pos_offset + t;
  constexpr int E = Network<WP>::E;
  float s[E];
  int id[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    if (i < g.W0) {
      const int f = g.flags[row * g.W0 + i];
      float v = (f & 4) ? g.scores[row * g.W0 + i] : 0.f;
      if (!(f & 1)) v = kNegFill;
      if (f & 2) v = kPosFill;
      s[e] = v;
      id[e] = g.cand[row * g.W0 + i];
    } else {
      s[e] = kNegFill;
      id[e] = -1;
    }
  }
  Network<WP>::sort(s, id, lane);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    if (i < g.K) {
      const int v = id[e];
      g.out_ids[row * g.K + i] = (v < 0 || int64_t(v) * g.C > pos) ? -1 : v;
    }
  }
}

}  // namespace

int grouped_leaf(const GroupArgs& args, int dtype, cudaStream_t stream) {
  GroupArgs g = args;
  g.fNF = FastDiv::make(uint32_t(g.NF));
  g.fH = FastDiv::make(uint32_t(g.H));
  g.fT = FastDiv::make(uint32_t(g.T));
  g.fNP = FastDiv::make(uint32_t(g.NP));
  g.fTW = FastDiv::make(uint32_t(g.TW));
  g.fRT = FastDiv::make(uint32_t(g.RT));
  g.fbr = FastDiv::make(uint32_t(g.br));
  g.fnwin = FastDiv::make(uint32_t(g.nwin));
  const int64_t families = int64_t(g.B) * g.T * g.H * g.NF;
  const int64_t rows = int64_t(g.B) * g.T * g.H;
  cudaError_t e;
  if (!g.counts_ready) {
    e = cudaMemsetAsync(g.counts, 0, sizeof(int32_t) * g.num_buckets, stream);
    if (e != cudaSuccess) return fail_cuda(e, "bucket counts clear");
  }
  e = cudaMemsetAsync(g.cursors, 0, sizeof(int32_t) * g.num_buckets, stream);
  if (e != cudaSuccess) return fail_cuda(e, "bucket cursors clear");
  e = cudaMemsetAsync(g.tile_req_w, 0xFF, sizeof(int32_t) * g.tile_capacity * g.RT, stream);
  if (e != cudaSuccess) return fail_cuda(e, "tile list clear");
  const unsigned grid = unsigned((families + 255) / 256);
  if (!g.counts_ready) {
    family_count_kernel<<<grid, 256, 0, stream>>>(g, g.counts);
    PISA_CHECK_LAUNCH();
  }
  e = launch_tile_scan(g.counts, g.offsets, g.total_tiles_w, g.num_buckets, g.RT, stream);
  if (e != cudaSuccess) return fail_cuda(e, "leaf tile scan");
  family_scatter_kernel<<<grid, 256, 0, stream>>>(g, g.offsets, g.cursors, g.tile_owner_w, g.tile_req_w);
  PISA_CHECK_LAUNCH();

  const int chunks = g.Dp / 64;
  // Two key buffers (and two query stages) when a query run is too short to
  // give a family more than about one tile (decode and short chunks): the
  // next family's keys then load while the current tile is scored.  Prefill
  // keeps one key buffer behind three query stages.
  const size_t smem2 = size_t(chunks) * 128 * (2 * 128 + 2 * g.br * g.C) + 1024;
  g.kbufs = (g.T < 64 && smem2 <= size_t(200) * 1024) ? 2 : 1;
  const size_t smem = g.kbufs == 2 ? smem2 : size_t(chunks) * 128 * (kStages * 128 + g.br * g.C) + 1024;
  auto kernel = dtype == PISA_BF16 ? (g.kbufs == 2 ? leaf_tc_kernel<__nv_bfloat16, 2> : leaf_tc_kernel<__nv_bfloat16, 1>)
                                   : (g.kbufs == 2 ? leaf_tc_kernel<__half, 2> : leaf_tc_kernel<__half, 1>);
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return fail_cuda(e, "leaf smem attribute");
  {
    TimedLaunch timed(PISA_KERNEL_LEAF_TILES, stream);
    kernel<<<unsigned(g.num_sms), kPipeThreads, smem, stream>>>(g);
    PISA_CHECK_LAUNCH();
  }

  if (g.skip_final) return PISA_OK;
  const unsigned fgrid = unsigned((rows + 3) / 4);
  TimedLaunch timed(PISA_KERNEL_LEAF_FINAL, stream);
  switch (g.W0) {
    case 16: leaf_final_kernel<16><<<fgrid, 128, 0, stream>>>(g); break;
    case 32: leaf_final_kernel<32><<<fgrid, 128, 0, stream>>>(g); break;
    case 64: leaf_final_kernel<64><<<fgrid, 128, 0, stream>>>(g); break;
    case 128: leaf_final_kernel<128><<<fgrid, 128, 0, stream>>>(g); break;
    default: leaf_final_kernel<256><<<fgrid, 128, 0, stream>>>(g); break;
  }
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

}  // namespace pisa
