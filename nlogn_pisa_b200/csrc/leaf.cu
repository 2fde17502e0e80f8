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

constexpr int kLeafThreads = 128;

__device__ __forceinline__ void decode_row(int64_t row, int T, int H, int& b, int& t, int& h) {
  h = int(row % H);
  t = int((row / H) % T);
  b = int(row / (int64_t(H) * T));
}

// Requests: one per (row, family) with at least one scoreable child.
__global__ void family_count_kernel(const GroupArgs g, int32_t* __restrict__ counts) {
  const int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  const int64_t total = int64_t(g.B) * g.T * g.H * g.NF;
  if (idx >= total) return;
  const int64_t row = idx / g.NF;
  const int k = int(idx % g.NF);
  const uint8_t* f = g.flags + row * g.W0 + k * g.br;
  bool active = false;
  for (int j = 0; j < g.br; ++j) active |= (f[j] & 4) != 0;
  if (!active) return;
  int b, t, h;
  decode_row(row, g.T, g.H, b, t, h);
  const int p = g.cand[row * g.W0 + k * g.br] / g.br;
  const int64_t bucket = ((int64_t(b) * g.nwin + t / g.TW) * g.H + h) * g.NP + p;
  atomicAdd(counts + bucket, 1);
}

__global__ void family_scatter_kernel(const GroupArgs g, const int32_t* __restrict__ offsets,
                                      int32_t* __restrict__ cursors, int32_t* __restrict__ tile_owner,
                                      int32_t* __restrict__ tile_req) {
  const int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  const int64_t total = int64_t(g.B) * g.T * g.H * g.NF;
  if (idx >= total) return;
  const int64_t row = idx / g.NF;
  const int k = int(idx % g.NF);
  const uint8_t* f = g.flags + row * g.W0 + k * g.br;
  bool active = false;
  for (int j = 0; j < g.br; ++j) active |= (f[j] & 4) != 0;
  if (!active) return;
  int b, t, h;
  decode_row(row, g.T, g.H, b, t, h);
  const int p = g.cand[row * g.W0 + k * g.br] / g.br;
  const int64_t bucket = ((int64_t(b) * g.nwin + t / g.TW) * g.H + h) * g.NP + p;
  const int pos = atomicAdd(cursors + bucket, 1);
  const int64_t tile = offsets[bucket] + pos / g.RT;
  tile_req[tile * g.RT + pos % g.RT] = int32_t(idx);
  if (pos % g.RT == 0) tile_owner[tile] = int32_t(bucket);
}

// One CTA walks `tiles_per_cta` consecutive tiles, restaging the family keys
// only when the bucket changes.  Four warps: all load, thread 0 issues the
// MMAs, all four read back one TMEM lane (= one query-head row) each.
template <typename T>
__global__ void __launch_bounds__(kLeafThreads) leaf_tc_kernel(const GroupArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int Dp = g.Dp;                     // head_dim rounded up to 64
  const int chunks = Dp / 64;              // 128-byte K chunks
  const int NK = g.br * g.C;               // keys per family = MMA N (total)
  uint8_t* Qs = smem;                      // [chunks][128 rows][128 B]
  uint8_t* Ks = smem + chunks * 128 * 128; // [chunks][NK rows][128 B]
  __shared__ uint64_t mbar;
  __shared__ uint32_t tmem_slot;
  __shared__ int32_t s_req[128];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = *g.total_tiles;
  const int first = blockIdx.x * g.tiles_per_cta;
  if (first >= total) return;
  const int last = min(first + g.tiles_per_cta, total);

  if (tid == 0) tc::mbar_init(&mbar, 1);
  if (warp == 0) tc::tmem_alloc(&tmem_slot, g.tmem_cols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_base = (uint32_t(warp) * 32) << 16;
  const uint32_t qs_addr = tc::smem_u32(Qs), ks_addr = tc::smem_u32(Ks);
  const T* qbase = static_cast<const T*>(g.q);
  const T* kbase = static_cast<const T*>(g.keys);
  const int vec_per_row = Dp / 8;          // 16-byte vectors per row (8 elements of 2 bytes)
  const int dvec = g.D / 8;
  uint32_t phase = 0;
  int cur_owner = -1;
  bool ok = true;

  for (int tile = first; tile < last; ++tile) {
    const int owner = g.tile_owner[tile];
    const int p = owner % g.NP;
    const int h = (owner / g.NP) % g.H;
    const int b = owner / (g.NP * g.H * g.nwin);
    if (tid < g.RT) s_req[tid] = g.tile_req[int64_t(tile) * g.RT + tid];
    if (owner != cur_owner) {
      // stage the family's NK contiguous keys (zero past the sequence end / head_dim)
      const int64_t tok0 = int64_t(p) * NK;
      const T* kb = kbase + b * g.k_sb + int64_t(h) * g.k_sh;
      for (int idx = tid; idx < NK * vec_per_row; idx += kLeafThreads) {
        const int r = idx / vec_per_row, c = idx % vec_per_row;
        const uint32_t dst = ks_addr + (c >> 3) * NK * 128 + tc::swizzle128(r, c & 7);
        const int64_t tok = tok0 + r;
        if (tok < g.N && c < dvec) cp_async16(dst, kb + tok * g.k_st + c * 8);
        else st_zero16(dst);
      }
      cur_owner = owner;
    }
    __syncthreads();  // s_req visible
    for (int idx = tid; idx < 128 * vec_per_row; idx += kLeafThreads) {
      const int row = idx / vec_per_row, c = idx % vec_per_row;
      const int r = row / g.G, gh = row % g.G;
      const uint32_t dst = qs_addr + (c >> 3) * 128 * 128 + tc::swizzle128(row, c & 7);
      const int req = r < g.RT ? s_req[r] : -1;
      if (req >= 0 && c < dvec) {
        int bb, t, hh;
        decode_row(req / g.NF, g.T, g.H, bb, t, hh);
        cp_async16(dst, qbase + bb * g.q_sb + t * g.q_st + int64_t(hh * g.G + gh) * g.q_sh + c * 8);
      } else {
        st_zero16(dst);
      }
    }
    cp_async_wait_all();
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0) {
      for (int n0 = 0; n0 < NK; n0 += 256) {
        const int n = min(256, NK - n0);
        const uint32_t idesc = tc::idesc_f16(128, n, g.bf16);
        for (int ks = 0; ks < Dp / 16; ++ks) {
          const int ch = ks >> 2, off = (ks & 3) * 32;
          const uint64_t ad = tc::desc_sw128(qs_addr + ch * 128 * 128 + off);
          const uint64_t bd = tc::desc_sw128(ks_addr + ch * NK * 128 + n0 * 128 + off);
          tc::mma_f16(tmem + n0, ad, bd, idesc, ks > 0);
        }
      }
      tc::mma_commit(&mbar);
    }
    if (!tc::mbar_wait(&mbar, phase)) ok = false;
    phase ^= 1;
    tc::fence_after_sync();

    // epilogue: thread <-> TMEM lane <-> query-head row
    const int row = tid;
    const int r = row / g.G;
    const int req = (r < g.RT) ? s_req[r] : -1;
    for (int j = 0; j < g.br; ++j) {
      const int64_t key0 = (int64_t(p) * g.br + j) * g.C;
      const int col0 = j * g.C;
      const int valid_keys = int(min64(g.C, max(int64_t(0), g.N - key0)));
      float score;
      if (g.method == PISA_METHOD_PISA) {
        float mx = -INFINITY;
        for_columns(tmem + lane_base + col0, g.C, [&](int c, float x) {
          if (c < valid_keys) mx = fmaxf(mx, x * g.scale);
        });
        float sum = 0.f;
        for_columns(tmem + lane_base + col0, g.C, [&](int c, float x) {
          if (c < valid_keys) sum += expf(x * g.scale - mx);
        });
        score = mx + logf(sum);
      } else {
        float s1 = 0.f, s2 = 0.f;
        for_columns(tmem + lane_base + col0, g.C, [&](int c, float x) {
          if (c < valid_keys) { s1 += x; s2 += x * x; }
        });
        const float n = float(valid_keys > 0 ? valid_keys : 1);
        const float mean = s1 / n, var = fmaxf(s2 / n - mean * mean, 0.f);
        score = g.scale * mean + g.c2 * var;
      }
      if (key0 >= g.N) score = 0.f;  // child past the end: never scoreable
      for (int o = 1; o < g.G; o <<= 1) score += __shfl_xor_sync(kFull, score, o);
      if (req >= 0 && (row % g.G) == 0) {
        const int64_t rowid = req / g.NF;
        const int k = req % g.NF;
        g.scores[rowid * g.W0 + k * g.br + j] = score;
      }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }
  if (!ok && lane == 0) atomicExch(g.status, PISA_ERR_TIMEOUT);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
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
  decode_row(row, g.T, g.H, b, t, h);
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

int grouped_leaf(const GroupArgs& g, int dtype, cudaStream_t stream) {
  const int64_t families = int64_t(g.B) * g.T * g.H * g.NF;
  const int64_t rows = int64_t(g.B) * g.T * g.H;
  cudaError_t e;
  e = cudaMemsetAsync(g.counts, 0, sizeof(int32_t) * g.num_buckets, stream);
  if (e != cudaSuccess) return fail_cuda(e, "bucket counts clear");
  e = cudaMemsetAsync(g.cursors, 0, sizeof(int32_t) * g.num_buckets, stream);
  if (e != cudaSuccess) return fail_cuda(e, "bucket cursors clear");
  e = cudaMemsetAsync(g.tile_req_w, 0xFF, sizeof(int32_t) * g.tile_capacity * g.RT, stream);
  if (e != cudaSuccess) return fail_cuda(e, "tile list clear");
  const unsigned grid = unsigned((families + 255) / 256);
  family_count_kernel<<<grid, 256, 0, stream>>>(g, g.counts);
  PISA_CHECK_LAUNCH();
  tile_scan_kernel<<<1, kScanThreads, 0, stream>>>(g.counts, g.offsets, g.total_tiles_w, g.num_buckets, g.RT);
  PISA_CHECK_LAUNCH();
  family_scatter_kernel<<<grid, 256, 0, stream>>>(g, g.offsets, g.cursors, g.tile_owner_w, g.tile_req_w);
  PISA_CHECK_LAUNCH();

  const int chunks = g.Dp / 64;
  size_t smem = size_t(chunks) * 128 * (128 + g.br * g.C) + 1024;
  // Keep (resident CTAs per SM) x (TMEM columns per CTA) <= 512 so that no
  // CTA waits in tcgen05.alloc: shared memory bounds the residency.
  const size_t per_sm = 228 * 1024, ctas_fit = 512 / size_t(g.tmem_cols);
  if (ctas_fit < 16) smem = std::max(smem, per_sm / ctas_fit - 4096);
  auto kernel = dtype == PISA_BF16 ? leaf_tc_kernel<__nv_bfloat16> : leaf_tc_kernel<__half>;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return fail_cuda(e, "leaf smem attribute");
  const int64_t ctas = (g.tile_capacity + g.tiles_per_cta - 1) / g.tiles_per_cta;
  kernel<<<unsigned(ctas), kLeafThreads, smem, stream>>>(g);
  PISA_CHECK_LAUNCH();

  const unsigned fgrid = unsigned((rows + 3) / 4);
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
