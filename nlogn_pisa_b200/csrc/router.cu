// K2: coarse-to-fine router (and, in the fused schedule, leaf scoring + top-K).
//
// One CTA of four warps (up to sixteen in the fused decode kernel) routes one
// (batch, query token, KV head) item through
// levels top..0, as pyramid_select (pisa/pisa/ops/flash_sparse_attn/
// top_k_pyramid/top_k_pyramid_torch.py:137-177):
//   masks      valid = id>=0 & id*(C*b^l) <= pos; forced = first block or an
//              ancestor of leaf pos//C - r (r < force_recent); scoreable =
//              valid & !forced & (#valid > K) (pisa1: no identity shortcut)
//              (:6-14, :114-120; triton score_masks :105-122)
//   scores     LSE / second-order over the b child summaries (levels >= 1),
//              over the C raw keys (level 0), or q . node mean (pisa1),
//              fp32, summed over the G query heads of the KV head (:48-80)
//   fill       unscoreable 0, invalid -1e9, forced +1e9 (:169-171)
//   top-K      the descending bitonic network with its tie order (:84-110)
//   expand     children b*id + {0..b-1} (:173-175)
// Scoring threads own one candidate each at coarse levels and one warp per
// candidate block at the leaf level (lanes own keys; warp shuffles combine the
// per-lane running max / sum of exponentials).  Warp 0 runs the network in
// registers (element i in lane i%32, slot i/32).
#include <algorithm>
#include <type_traits>

#include "internal.h"
#include "score.cuh"
#include "tc.cuh"

namespace pisa {

namespace {

constexpr int kThreads = 128;
// the fused decode kernel with few items: sixteen warps per (sequence,
// token, KV head), so that more candidate and selected key blocks are read
// at once
constexpr int kAttendThreads = 512;
constexpr int kMaxWidth = 256;

// 16-bit inputs score coarse levels with mma.sync (bf16 / fp16 operands)
template <typename T>
constexpr bool kMmaCoarse = std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value;

template <int WP>
__device__ __forceinline__ void network_step(float* sc, int* ids, int width, int K, int br,
                                             int level, int64_t pos, int C, int lane,
                                             int64_t* out, int* next_ids) {
  constexpr int E = Network<WP>::E;
  float s[E];
  int id[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    const bool in = i < width;
    s[e] = in ? sc[i] : kNegFill;
    id[e] = in ? ids[i] : -1;
  }
  __syncwarp();
  Network<WP>::sort(s, id, lane);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    if (i < K) {
      const int v = id[e];
      if (level > 0) {
        for (int j = 0; j < br; ++j) next_ids[i * br + j] = v < 0 ? -1 : v * br + j;
      } else {
        // final ids (also kept in shared memory for a fused attention)
        const int fin = (v < 0 || int64_t(v) * C > pos) ? -1 : v;
        if (out) out[i] = fin;
        next_ids[i] = fin;
      }
    }
  }
}

// Fused decode: attention of the row's G query heads over its K selected
// blocks (ids in shared memory, -1 = none) with the semantics of
// sparse_attn_torch.py:6-35 (one softmax over the union of the blocks'
// visible keys, causal at the row's position).  Warp w takes slots w, w+4,
// ...; per chunk of 32 keys: logits with lane = key (q from shared memory),
// online softmax per head, then P.V with lane = VPL value columns (the warp
// reads each value row whole).  The warps merge through shared memory.
template <typename T, int GMAX, int VPL, int NT>
__device__ void decode_attend(const RouteArgs& a, const int* sel, const float* qs, int b, int t, int h,
                              int64_t pos, float* scratch) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int W = NT / 32;
  const int G = a.G, Dv = a.Dv;
  float* pw = scratch;                     // [W][G][32] probabilities of the current chunk
  float* mw = pw + W * G * 32;             // [W][G]
  float* lw = mw + W * G;                  // [W][G]
  float* ow = lw + W * G;                  // [W][G][Dv]
  const T* kbase = static_cast<const T*>(a.keys) + int64_t(b) * a.k_sb + int64_t(h) * a.k_sh;
  const T* vbase = static_cast<const T*>(a.values) + int64_t(b) * a.v_sb + int64_t(h) * a.v_sh + lane * VPL;
  float m[GMAX], l[GMAX], o[GMAX][VPL];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) o[g][j] = 0.f;
  }
  for (int s = warp; s < a.K; s += W) {
    const int id = sel[s];
    if (id < 0) continue;
    const int64_t k0 = int64_t(id) * a.C;
    const int64_t k1 = min64(min64(k0 + a.C, int64_t(a.N)), pos + 1);
    for (int64_t base = k0; base < k1; base += 32) {
      const int nk = int(min64(32, k1 - base));
      float z[GMAX];
      if (lane < nk) {
        row_dots<T, GMAX>(kbase + (base + lane) * a.k_st, qs, G, a.D, z);
      }
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        if (g >= G) continue;
        const float zv = lane < nk ? z[g] * a.attn_scale : -INFINITY;
        const float mnew = fmaxf(m[g], warp_max(zv));
        const float alpha = m[g] == -INFINITY ? 0.f : expf(m[g] - mnew);
        const float pv = zv == -INFINITY ? 0.f : expf(zv - mnew);
        l[g] = l[g] * alpha + warp_sum(pv);
        m[g] = mnew;
#pragma unroll
        for (int j = 0; j < VPL; ++j) o[g][j] *= alpha;
        pw[(warp * G + g) * 32 + lane] = pv;
      }
      __syncwarp();
      // P.V: four value rows in flight, each read whole by the warp
      for (int k0 = 0; k0 < nk; k0 += 4) {
        float x[4][VPL];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (k0 + u < nk) {
            const T* vr = vbase + (base + k0 + u) * a.v_st;
#pragma unroll
            for (int j = 0; j < VPL; ++j) x[u][j] = to_f32<T>(vr[j]);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (k0 + u >= nk) break;
#pragma unroll
          for (int g = 0; g < GMAX; ++g) {
            if (g >= G) continue;
            const float pv = pw[(warp * G + g) * 32 + k0 + u];
#pragma unroll
            for (int j = 0; j < VPL; ++j) o[g][j] = fmaf(pv, x[u][j], o[g][j]);
          }
        }
      }
      __syncwarp();
    }
  }
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    if (g >= G) continue;
    if (lane == 0) { mw[warp * G + g] = m[g]; lw[warp * G + g] = l[g]; }
#pragma unroll
    for (int j = 0; j < VPL; ++j) ow[(warp * G + g) * Dv + lane * VPL + j] = o[g][j];
  }
  __syncthreads();
  T* op = static_cast<T*>(a.out) + ((int64_t(b) * a.T + t) * (int64_t(a.H) * G) + int64_t(h) * G) * Dv;
  for (int i = tid; i < G * Dv; i += NT) {
    const int g = i / Dv, d = i - g * Dv;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, mw[w * G + g]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const float mm = mw[w * G + g];
        if (mm == -INFINITY) continue;
        const float f = expf(mm - M);
        L += lw[w * G + g] * f;
        O += ow[(w * G + g) * Dv + d] * f;
      }
    }
    op[i] = from_f32<T>(L > 0.f ? O / L : 0.f);
    if (d == 0 && a.lse)
      a.lse[(int64_t(b) * a.T + t) * (int64_t(a.H) * G) + int64_t(h) * G + g] = L > 0.f ? M + logf(L) : -INFINITY;
  }
}

// Per-row mma.sync scoring of a coarse level (defined with the warp router below).
template <typename T, int KP>
__device__ void row_level_scores(const RouteArgs& a, const uint4 (&q0)[KP], const uint4 (&q1)[KP],
                                 int sid0, int sid1, int width, int level, int b, int h, int lane,
                                 float* sc_out);
template <typename T, int KP>
__device__ __forceinline__ void load_q_frags(const RouteArgs& a, int b, int t, int h, int lane,
                                             uint4 (&q0)[KP], uint4 (&q1)[KP]);

// Coarse-level scores of the per-item router on the tensor cores: warp w
// scores candidates 32w .. 32w+31 of the level (then 128 more per round)
// with the row scorer's m16n8k16 MMAs over their child summaries; entries of
// unscoreable candidates are left alone.
template <typename T, int KP, int NT>
__device__ void item_coarse_mma(const RouteArgs& a, const int* ids, const unsigned char* fl, bool identity,
                                int width, int level, int b, int t, int h, int warp, int lane, float* sc) {
  uint4 q0[KP], q1[KP];
  load_q_frags<T, KP>(a, b, t, h, lane, q0, q1);
  for (int base = warp * 32; base < width; base += NT) {
    const int i = base + lane;
    const int f = i < width ? fl[i] : 0;
    const bool scoreable = (f & 1) && !(f & 2) && !identity;
    const int sid = scoreable ? ids[i] : -1;
    if (__ballot_sync(kFull, sid >= 0) == 0) continue;   // warp-uniform
    row_level_scores<T, KP>(a, q0, q1, sid, -1, min(32, width - base), level, b, h, lane, sc + base);
  }
}

// Without the fused attention and with G <= 4 the kernel is held to four CTAs
// per SM (128 registers): the 512 items of a 64-sequence decode step then run
// in one wave (104 -> 66 us for their coarse levels).
template <typename T, int GMAX, bool ATTEND, int NT>
__global__ void __launch_bounds__(NT, ATTEND ? kAttendThreads / NT : (GMAX <= 4 ? 4 : 1)) route_kernel(const RouteArgs a) {
  extern __shared__ __align__(16) float smem[];
  float* qs = smem;                                    // [G][D]
  int* ids = reinterpret_cast<int*>(qs + a.G * a.D);   // [kMaxWidth]
  float* sc = reinterpret_cast<float*>(ids + kMaxWidth);
  unsigned char* fl = reinterpret_cast<unsigned char*>(sc + kMaxWidth);
  __shared__ int s_valid;

  const int local = blockIdx.x;                 // (b, token in range, h)
  const int h = local % a.H;
  const int tl = (local / a.H) % a.t_count;
  const int b = local / (a.H * a.t_count);
  const int t = a.t_begin + tl;
  const int64_t item = (int64_t(b) * a.T + t) * a.H + h;
  const float* dense_row = a.dense ? a.dense + int64_t(local) * a.dense_stride : nullptr;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t pos = a.positions ? a.positions[int64_t(b) * a.T + t] : a.pos_offset + t;

  const T* qp = static_cast<const T*>(a.q) + b * a.q_sb + t * a.q_st + int64_t(h) * a.G * a.q_sh;
  for (int e = tid; e < a.G * a.D; e += NT) {
    const int g = e / a.D, d = e % a.D;
    qs[e] = to_f32<T>(qp[g * a.q_sh + d]);
  }
  int width = a.first_width;
  for (int w = tid; w < width; w += NT) ids[w] = w;
  const T* summary = static_cast<const T*>(a.summary) + b * a.s_sb + int64_t(h) * a.D;
  const T* key_base = static_cast<const T*>(a.keys) + b * a.k_sb + int64_t(h) * a.k_sh;
  const int64_t node_stride = int64_t(a.H) * a.D;
  __syncthreads();

  int64_t span = a.C;  // C * br^level
  int64_t div = 1;     // br^level
  for (int l = 0; l < a.top; ++l) { span *= a.br; div *= a.br; }
  const int64_t leaf = pos / a.C;

  for (int level = a.top; level >= 0; --level) {
    const int len = a.levels.size[level];
    for (int w = tid; w < width; w += NT) {
      int id = ids[w];
      if (id >= len) id = -1;
      ids[w] = id;
      const bool valid = id >= 0 && int64_t(id) * span <= pos;
      bool forced = false;
      if (valid) {
        if (a.force_first && id == 0) forced = true;
        for (int r = 0; r < a.force_recent; ++r) {
          const int64_t target = leaf - r;
          if (target >= 0 && id == target / div) forced = true;
        }
      }
      fl[w] = (valid ? 1 : 0) | (forced ? 2 : 0);
    }
    __syncthreads();
    if (warp == 0) {
      int cnt = 0;
      for (int w = lane; w < width; w += 32) cnt += fl[w] & 1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(kFull, cnt, o);
      if (lane == 0) s_valid = cnt;
    }
    __syncthreads();
    const bool identity = a.method != PISA_METHOD_PISA1 && s_valid <= a.K;

    if (level == 0 && a.coarse_only) {
      // Leaf candidates with their masks: bit0 valid, bit1 forced, bit2 scoreable.
      int32_t* dst = a.candidates + int64_t(item) * a.W0;
      uint8_t* fdst = a.flags + int64_t(item) * a.W0;
      for (int w = tid; w < width; w += NT) {
        const int f = fl[w];
        const bool scoreable = (f & 1) && !(f & 2) && !identity;
        dst[w] = ids[w];
        fdst[w] = uint8_t(f | (scoreable ? 4 : 0));
      }
      return;
    }

    // fill values and thread-per-candidate scoring (coarse levels of 16-bit
    // inputs go to the tensor cores below instead)
    const bool warp_leaf = level == 0 && a.method != PISA_METHOD_PISA1 && a.dense_off[0] < 0;
    const bool coarse_level = level > 0 || a.method == PISA_METHOD_PISA1;
    const bool mma_level = kMmaCoarse<T> && coarse_level && !(dense_row && a.dense_off[level] >= 0) &&
                           a.G <= 16 && (a.method == PISA_METHOD_PISA1 || a.br == 2 || a.br == 4) && !identity;
    for (int w = tid; w < width; w += NT) {
      const int f = fl[w];
      const bool valid = f & 1, forced = f & 2;
      const bool scoreable = valid && !forced && !identity;
      float v = 0.f;
      if (scoreable && !warp_leaf && dense_row && a.dense_off[level] >= 0) {
        v = dense_row[a.dense_off[level] + ids[w]];
      } else if (scoreable && !warp_leaf && !mma_level) {
        if (a.method == PISA_METHOD_PISA1) {
          v = coarse_score<T, GMAX>(a, summary + a.levels.offset[level] * node_stride, len, ids[w], qs);
        } else {
          v = coarse_score<T, GMAX>(a, summary + a.levels.offset[level - 1] * node_stride,
                                    a.levels.size[level - 1], ids[w], qs);
        }
      }
      sc[w] = !valid ? kNegFill : (forced ? kPosFill : v);
    }
    if constexpr (kMmaCoarse<T>) {
      if (mma_level) {
        __syncthreads();
        if (a.D <= 64) item_coarse_mma<T, 2, NT>(a, ids, fl, identity, width, level, b, t, h, warp, lane, sc);
        else if (a.D <= 128) item_coarse_mma<T, 4, NT>(a, ids, fl, identity, width, level, b, t, h, warp, lane, sc);
        else item_coarse_mma<T, 8, NT>(a, ids, fl, identity, width, level, b, t, h, warp, lane, sc);
      }
    }
    if (warp_leaf) {
      __syncthreads();
      for (int w = warp; w < width; w += NT / 32) {
        const int f = fl[w];
        const bool scoreable = (f & 1) && !(f & 2) && !identity;
        if (scoreable) {
          const float v = leaf_score_warp<T, GMAX>(a, key_base, ids[w], qs, lane);
          if (lane == 0) sc[w] = v;
        }
      }
    }
    __syncthreads();
    if (warp == 0) {
      int64_t* out = level == 0 ? a.out_ids + int64_t(item) * a.K : nullptr;
      switch (width) {
        case 16: network_step<16>(sc, ids, width, a.K, a.br, level, pos, a.C, lane, out, ids); break;
        case 32: network_step<32>(sc, ids, width, a.K, a.br, level, pos, a.C, lane, out, ids); break;
        case 64: network_step<64>(sc, ids, width, a.K, a.br, level, pos, a.C, lane, out, ids); break;
        case 128: network_step<128>(sc, ids, width, a.K, a.br, level, pos, a.C, lane, out, ids); break;
        default: network_step<256>(sc, ids, width, a.K, a.br, level, pos, a.C, lane, out, ids); break;
      }
    }
    __syncthreads();
    width = a.K * a.br;
    span /= a.br;
    div /= a.br;
  }
  if constexpr (ATTEND) {
    // the final ids are in ids[0 .. K); attention scratch after the router's
    // arrays (the launcher admits G * Dv / 32 <= 64 accumulators per lane)
    float* scratch = reinterpret_cast<float*>(fl + ((kMaxWidth + 15) / 16) * 16);
    switch (a.Dv / 32) {
      case 2: decode_attend<T, GMAX, 2, NT>(a, ids, qs, b, t, h, pos, scratch); break;
      case 4:
        if constexpr (GMAX <= 16) decode_attend<T, GMAX, 4, NT>(a, ids, qs, b, t, h, pos, scratch);
        break;
      default:
        if constexpr (GMAX <= 8) decode_attend<T, GMAX, 8, NT>(a, ids, qs, b, t, h, pos, scratch);
        break;
    }
  }
}

// The comparison network over the first WP elements of E register slots
// (element i in lane i%32, slot i/32).
template <int WP, int E>
__device__ __forceinline__ void warp_sort(float (&s)[E], int (&id)[E], int lane) {
  float ss[Network<WP>::E];
  int ii[Network<WP>::E];
#pragma unroll
  for (int e = 0; e < Network<WP>::E; ++e) { ss[e] = s[e]; ii[e] = id[e]; }
  Network<WP>::sort(ss, ii, lane);
#pragma unroll
  for (int e = 0; e < Network<WP>::E; ++e) { s[e] = ss[e]; id[e] = ii[e]; }
}

// The network of the level's width (a power of two from 16 to 32*E).
template <int E>
__device__ __forceinline__ void warp_sort_width(float (&s)[E], int (&id)[E], int lane, int width) {
  if (width <= 16) warp_sort<16, E>(s, id, lane);
  else if (width <= 32) warp_sort<32, E>(s, id, lane);
  else if constexpr (E >= 2) {
    if (width <= 64) warp_sort<64, E>(s, id, lane);
    else if constexpr (E >= 4) {
      if (width <= 128) warp_sort<128, E>(s, id, lane);
      else if constexpr (E >= 8) warp_sort<256, E>(s, id, lane);
    }
  }
}

// ---------------------------------------------------------------------------
// Per-row scoring of a coarse level inside the warp router.
//
// Dense scoring (dense.cu) scores every node of a level for every token:
// its work grows with the square of the sequence length, and each level
// reloads the rows' queries.  A row-scored level instead takes the row's own
// candidates: their children summaries (at most 64 columns) against the
// row's G <= 16 query heads, S = Q X^T as a 16 x 8 x 16 warp MMA per column
// tile (mma.sync; bf16/fp16 in, fp32 accumulate), then the score equations
// of block_scores (top_k_pyramid_torch.py:48-80) per candidate, summed over
// the heads -- the reference descent's own O(K) work per level.  (tcgen05
// needs M >= 64 rows per MMA; one row's G heads give 16.)
//
// Fragment layout (m16n8k16, g = lane/4, c = lane%4).  The dot product sums
// over all head dims, so any one-to-one map of the MMA's k index onto the
// dims, shared by A and B, gives the same sums; the map used here lets each
// lane fetch its part of a row with one 16-byte load per 32 dims: for the
// dim pair-step p (dims 32p .. 32p+31) lane c holds dims 32p+8c .. 32p+8c+7,
// whose words 0,1 are (k0..1, k8..9) of k-step 2p and words 2,3 those of
// k-step 2p+1, with k0 = 2c.
//   A (row-major 16 x 16): a0/a2 = Q[g] words, a1/a3 = Q[g+8] words
//   B (column n = g of the tile): b0/b1 = X[n] words
//   C: c0, c1 = S[g][2c + {0,1}], c2, c3 = S[g+8][same]
// ---------------------------------------------------------------------------
constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;

// log2 on the MUFU unit (lg2.approx: relative error about 2^-22)
__device__ __forceinline__ float lg2f(float x) {
  float r;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// 16 bytes of a query / summary row (read-only path), zero when absent.
__device__ __forceinline__ uint4 ld_row16(const void* p, bool ok) {
  return ok ? __ldg(static_cast<const uint4*>(p)) : make_uint4(0u, 0u, 0u, 0u);
}

// The row's query heads as A fragments: KP pair-steps of 32 dims, rows g and
// g+8 (zero past D and past G heads).
template <typename T, int KP>
__device__ __forceinline__ void load_q_frags(const RouteArgs& a, int b, int t, int h, int lane,
                                             uint4 (&q0)[KP], uint4 (&q1)[KP]) {
  const int g = lane >> 2, c = lane & 3;
  const T* base = static_cast<const T*>(a.q) + int64_t(b) * a.q_sb + int64_t(t) * a.q_st;
  const T* r0 = base + int64_t(h * a.G + g) * a.q_sh;
  const T* r1 = base + int64_t(h * a.G + g + 8) * a.q_sh;
#pragma unroll
  for (int p = 0; p < KP; ++p) {
    const int d = 32 * p + 8 * c;
    q0[p] = ld_row16(r0 + d, g < a.G && d < a.D);
    q1[p] = ld_row16(r1 + d, g + 8 < a.G && d < a.D);
  }
}

// Scores of the scoreable candidates of one level (element i in lane i%32,
// slot i/32; sid = the id when scoreable, else -1) into sc_out[i] (shared
// memory of this warp, `width` <= 64 entries; unscored entries are left alone).
template <typename T, int KP>
__device__ void row_level_scores(const RouteArgs& a, const uint4 (&q0)[KP], const uint4 (&q1)[KP],
                                 int sid0, int sid1, int width, int level, int b, int h, int lane,
                                 float* sc_out) {
  constexpr int NG = KP >= 4 ? 1 : 4 / KP;        // column tiles whose loads are in flight together
  const bool self = a.method == PISA_METHOD_PISA1;
  const int sup = self ? 1 : a.br;                 // columns per candidate: 1, 2 or 4
  const int lgs = sup == 1 ? 0 : (sup == 2 ? 1 : 2);
  const int child_level = self ? level : level - 1;
  const int child_len = a.levels.size[child_level];
  const int64_t node_stride = int64_t(a.H) * a.D;
  const T* base = static_cast<const T*>(a.summary) + int64_t(b) * a.s_sb +
                  a.levels.offset[child_level] * node_stride + int64_t(h) * a.D;
  const int ncols = width << lgs;
  const int g = lane >> 2, c = lane & 3;
  const bool row0 = g < a.G, row1 = g + 8 < a.G;
  for (int nt0 = 0; nt0 * 8 < ncols; nt0 += NG) {
    // this group's B rows: column nt*8 + g of each tile, one 16-byte load per pair-step
    uint4 xv[NG][KP];
    bool any[NG];
#pragma unroll
    for (int u = 0; u < NG; ++u) {
      const int colb = (nt0 + u) * 8 + g;
      const int cb = colb >> lgs, jb = colb & (sup - 1);
      const int i0 = __shfl_sync(kFull, sid0, cb & 31), i1 = __shfl_sync(kFull, sid1, cb & 31);
      const int idb = colb < ncols ? (cb < 32 ? i0 : i1) : -1;
      const int node = idb < 0 ? -1 : (self ? idb : idb * a.br + jb);
      const bool have = node >= 0 && node < child_len;
      any[u] = __ballot_sync(kFull, idb >= 0) != 0;
      const T* xr = base + int64_t(have ? node : 0) * node_stride;
#pragma unroll
      for (int p = 0; p < KP; ++p) {
        const int d = 32 * p + 8 * c;
        xv[u][p] = ld_row16(xr + d, have && d < a.D);
      }
    }
#pragma unroll
    for (int u = 0; u < NG; ++u) {
      const int nt = nt0 + u;
      if (nt * 8 >= ncols || !any[u]) continue;    // warp-uniform
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < KP; ++p) {
        mma16816<T>(acc, q0[p].x, q1[p].x, q0[p].y, q1[p].y, xv[u][p].x, xv[u][p].y);
        mma16816<T>(acc, q0[p].z, q1[p].z, q0[p].w, q1[p].w, xv[u][p].z, xv[u][p].w);
      }
      // this lane's C columns: 2c and 2c + 1 of the tile
      const int col0 = nt * 8 + 2 * c;
      if (sup == 1) {
        // pisa1: q . node mean (scale 1); columns col0 and col0 + 1 are two candidates
        float p0 = (row0 ? acc[0] : 0.f) + (row1 ? acc[2] : 0.f);
        float p1 = (row0 ? acc[1] : 0.f) + (row1 ? acc[3] : 0.f);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          p0 += __shfl_xor_sync(kFull, p0, o);
          p1 += __shfl_xor_sync(kFull, p1, o);
        }
        if (g == 0) {
          if (col0 < ncols) sc_out[col0] = p0;
          if (col0 + 1 < ncols) sc_out[col0 + 1] = p1;
        }
        continue;
      }
      // children of candidate `cand` that exist at the child level
      const int cand = col0 >> lgs;
      const int c0 = __shfl_sync(kFull, sid0, cand & 31), c1 = __shfl_sync(kFull, sid1, cand & 31);
      const int cid = col0 < ncols ? (cand < 32 ? c0 : c1) : -1;
      const int nchild = cid < 0 ? 0 : max(0, min(sup, child_len - cid * a.br));
      float part = 0.f;   // this lane's heads' contribution to the candidate score
      if (sup == 2) {
        // both children in this lane: (c0, c1) for head g, (c2, c3) for head g+8
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          if (!(r == 0 ? row0 : row1)) continue;
          const float z0 = acc[2 * r] * a.scale, z1 = acc[2 * r + 1] * a.scale;
          float v;
          if (a.method == PISA_METHOD_PISA) {
            // log(e^z0 + e^z1) = m + ln2 * log2(1 + 2^(-|z0 - z1| * log2 e))
            v = nchild >= 2 ? fmaxf(z0, z1) + kLn2 * lg2f(1.f + tc::ex2f(-fabsf(z0 - z1) * kLog2e)) : z0;
          } else {
            const float diff = z0 - z1;
            v = nchild >= 2 ? 0.5f * (z0 + z1) + 0.125f * diff * diff : z0;
          }
          part += v;
        }
      } else {
        // four children over a lane pair (c = 2m, 2m+1): exchange with the partner
        float o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = __shfl_xor_sync(kFull, acc[i], 1);
        const bool low = (lane & 1) == 0;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          if (!(r == 0 ? row0 : row1)) continue;
          float x[4];   // children 0..3 of the candidate, in column order
          x[0] = low ? acc[2 * r] : o[2 * r];
          x[1] = low ? acc[2 * r + 1] : o[2 * r + 1];
          x[2] = low ? o[2 * r] : acc[2 * r];
          x[3] = low ? o[2 * r + 1] : acc[2 * r + 1];
          float v;
          if (a.method == PISA_METHOD_PISA) {
            // base 2: y = x * scale * log2 e; LSE = ln2 * (max y + log2 sum 2^(y - max y))
            const float k2 = a.scale * kLog2e;
            float m = -INFINITY;
#pragma unroll
            for (int i = 0; i < 4; ++i) if (i < nchild) m = fmaxf(m, x[i] * k2);
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) if (i < nchild) s += tc::ex2f(fmaf(x[i], k2, -m));
            v = nchild > 0 ? kLn2 * (m + lg2f(s)) : 0.f;
          } else {
            float s1 = 0.f, s2 = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) if (i < nchild) { s1 += x[i]; s2 += x[i] * x[i]; }
            const float cnt = float(nchild > 0 ? nchild : 1);
            const float mean = s1 / cnt;
            const float var = fmaxf(s2 / cnt - mean * mean, 0.f);
            v = a.scale * mean + a.c2 * var;
          }
          part += v;
        }
      }
      // sum over the heads: lanes with the same lane%4 hold the other head rows
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) part += __shfl_xor_sync(kFull, part, o);
      if (g == 0 && cid >= 0 && (sup == 2 || (lane & 1) == 0)) sc_out[cand] = part;
    }
  }
}

// Warp-per-item router for descents whose every scored level has precomputed
// scores (dense.cu) or is row-scored here (KP > 0 pair-steps of head dims):
// levels >= 1 for pisa/pisa2 when the leaf level is left to the grouped
// tensor-core scorer (coarse_only), every level for pisa1.  The candidates
// and scores live in registers (element i in lane i%32, slot i/32; E slots,
// widths up to 32*E), validity is counted with ballots, and the same
// comparison network picks the K survivors; their children are expanded
// through shared memory.
template <typename T, int KP, int E>
__global__ void __launch_bounds__(128, (KP > 0 && KP <= 4) ? 6 : 1) route_warp_kernel(const RouteArgs a) {
  __shared__ int kept[4][64];
  __shared__ float s_row[4][64];   // row-scored level: candidate scores of each warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t local = int64_t(blockIdx.x) * 4 + warp;
  if (local >= int64_t(a.B) * a.t_count * a.H) return;
  // items < 2^31 (checked by the launcher)
  const uint32_t l1 = a.fH.div(uint32_t(local)), l2 = a.ftc.div(l1);
  const int h = int(uint32_t(local) - l1 * uint32_t(a.H));
  const int tl = int(l1 - l2 * uint32_t(a.t_count));
  const int b = int(l2);
  const int t = a.t_begin + tl;
  const int64_t item = (int64_t(b) * a.T + t) * a.H + h;
  const int64_t pos = a.positions ? a.positions[int64_t(b) * a.T + t] : a.pos_offset + t;
  const float* dense_row = a.dense ? a.dense + local * a.dense_stride : nullptr;
  const int64_t leaf = pos / a.C;
  uint4 q0[KP > 0 ? KP : 1], q1[KP > 0 ? KP : 1];
  if constexpr (KP > 0) load_q_frags<T, KP>(a, b, t, h, lane, q0, q1);
  // forced-recent leaves leaf-r (r < force_recent, leaf-r >= 0) have, at any
  // level, ancestors forming the contiguous id range [lo_leaf / div, leaf / div]
  const int64_t lo_leaf = leaf - a.force_recent + 1 > 0 ? leaf - a.force_recent + 1 : 0;
  // branching is a power of two (2 or 4): ancestors by shifts
  const int lgb = 31 - __clz(a.br);
  int64_t span = int64_t(a.C) << (lgb * a.top);
  int sh = lgb * a.top;   // log2 of br^level

  int id[E];
  float sc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) id[e] = e * 32 + lane;   // top level: 0..first_width-1
  int width = a.first_width;
  for (int level = a.top; level >= 0; --level) {
    const int len = a.levels.size[level];
    const int64_t f_hi = leaf >= 0 ? leaf >> sh : -1, f_lo = leaf >= 0 ? lo_leaf >> sh : 0;
    bool valid[E], forced[E];
    int nvalid = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int i = e * 32 + lane;
      int v = i < width ? id[e] : -1;
      if (v >= len) v = -1;
      id[e] = v;
      valid[e] = v >= 0 && int64_t(v) * span <= pos;
      bool f = false;
      if (valid[e]) {
        if (a.force_first && v == 0) f = true;
        if (a.force_recent > 0 && v >= f_lo && v <= f_hi) f = true;
      }
      forced[e] = f;
      nvalid += __popc(__ballot_sync(kFull, valid[e]));
    }
    const bool identity = a.method != PISA_METHOD_PISA1 && nvalid <= a.K;
    if (level == 0 && a.coarse_only) {
      int32_t* dst = a.candidates + item * a.W0;
      uint8_t* fdst = a.flags + item * a.W0;
      // families are br consecutive slots (br divides 32): the first slot's
      // lane counts the family's request when any child is scoreable
      const int bucket0 = a.fam_counts ? ((b * a.nwin + t / a.TW) * a.H + h) * a.NP : 0;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = e * 32 + lane;
        const bool scoreable = i < width && valid[e] && !forced[e] && !identity;
        if (i < width) {
          dst[i] = id[e];
          fdst[i] = uint8_t((valid[e] ? 1 : 0) | (forced[e] ? 2 : 0) | (scoreable ? 4 : 0));
        }
        if (a.fam_counts && e * 32 < width) {
          const unsigned bits = __ballot_sync(kFull, scoreable);
          const int q = int(a.fbr.div(uint32_t(lane)));
          if (lane == q * a.br && ((bits >> lane) & ((1u << a.br) - 1u)) != 0)
            atomicAdd(a.fam_counts + bucket0 + int(a.fbr.div(uint32_t(id[e]))), 1);
        }
      }
      return;
    }
    const int off = a.dense_off[level];
    bool row_scored = false;
    if constexpr (KP > 0) {
      if (((a.row_levels >> level) & 1u) && !identity) {
        int sid[2];
#pragma unroll
        for (int e = 0; e < 2; ++e)
          sid[e] = (e < E && e * 32 + lane < width && valid[e] && !forced[e]) ? id[e < E ? e : 0] : -1;
        row_level_scores<T, KP>(a, q0, q1, sid[0], sid[1], width, level, b, h, lane, s_row[warp]);
        __syncwarp();
        row_scored = true;
      }
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const bool scoreable = valid[e] && !forced[e] && !identity;
      float v = 0.f;
      if (scoreable) v = row_scored ? s_row[warp][e * 32 + lane] : dense_row[off + id[e]];
      sc[e] = !valid[e] ? kNegFill : (forced[e] ? kPosFill : v);
      if (e * 32 + lane >= width) { sc[e] = kNegFill; id[e] = -1; }
    }
    __syncwarp();
    warp_sort_width<E>(sc, id, lane, width);
    if (level == 0) {
      int64_t* out = a.out_ids + item * a.K;
#pragma unroll
      for (int e = 0; e < (E < 2 ? E : 2); ++e) {
        const int i = e * 32 + lane;
        if (i < a.K) out[i] = (id[e] < 0 || int64_t(id[e]) * a.C > pos) ? -1 : id[e];
      }
      return;
    }
    // survivors -> shared memory -> children in network order
#pragma unroll
    for (int e = 0; e < (E < 2 ? E : 2); ++e) {
      const int i = e * 32 + lane;
      if (i < a.K) kept[warp][i] = id[e];
    }
    __syncwarp();
    width = a.K * a.br;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int i = e * 32 + lane;
      const int q = int(a.fbr.div(uint32_t(i)));
      const int parent = i < width ? kept[warp][q] : -1;
      id[e] = parent < 0 ? -1 : parent * a.br + (i - q * a.br);
    }
    __syncwarp();
    span >>= lgb;
    sh -= lgb;
  }
}

template <typename T, int GMAX, bool ATTEND, int NT>
int launch_route_nt(const RouteArgs& a, cudaStream_t stream) {
  size_t smem = size_t(a.G) * a.D * sizeof(float) + kMaxWidth * (2 * sizeof(int) + 1);
  if (ATTEND) {
    // fused decode attention: probabilities, per-warp (m, l) and partial outputs
    const int W = NT / 32;
    smem = size_t(a.G) * a.D * sizeof(float) + kMaxWidth * 2 * sizeof(int) + (kMaxWidth + 15) / 16 * 16 +
           sizeof(float) * (size_t(W) * a.G * 32 + 2 * W * a.G + size_t(W) * a.G * a.Dv);
  }
  auto kernel = route_kernel<T, GMAX, ATTEND, NT>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return fail_cuda(e, "route smem attribute");
  }
  const int64_t items = int64_t(a.B) * a.t_count * a.H;
  if (items == 0) return PISA_OK;
  TimedLaunch timed(PISA_KERNEL_ROUTER, stream);
  kernel<<<unsigned(items), NT, smem, stream>>>(a);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

// The router keeps four warps per item; the fused decode kernel takes more
// warps per item when there are few items (a CTA's leaf scoring and attention
// are latency bound, so more warps read more key blocks at once), four when
// the items fill the GPU (fewer, wider CTAs would leave items waiting for a
// second wave: at 512 items sixteen warps measured 911 us against 742 us,
// at 128 items 219 us against 548 us).
template <typename T, int GMAX>
int launch_route(const RouteArgs& a, cudaStream_t stream) {
  if (!a.attend) return launch_route_nt<T, GMAX, false, kThreads>(a, stream);
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = int64_t(a.B) * a.t_count * a.H;
  if (items <= sms) return launch_route_nt<T, GMAX, true, kAttendThreads>(a, stream);
  if (items <= 2 * int64_t(sms)) return launch_route_nt<T, GMAX, true, kAttendThreads / 2>(a, stream);
  return launch_route_nt<T, GMAX, true, kThreads>(a, stream);
}

template <typename T>
int route_t(const RouteArgs& a, cudaStream_t stream) {
  if (a.attend && (a.G > 16 || a.G * (a.Dv / 32) > 64))
    return fail(PISA_ERR_UNSUPPORTED, "fused decode needs G <= 16 and G * value head_dim <= 2048");
  if (a.G <= 1) return launch_route<T, 1>(a, stream);
  if (a.G <= 2) return launch_route<T, 2>(a, stream);
  if (a.G <= 4) return launch_route<T, 4>(a, stream);
  if (a.G <= 8) return launch_route<T, 8>(a, stream);
  if (a.G <= 16) return launch_route<T, 16>(a, stream);
  return launch_route<T, 32>(a, stream);
}

}  // namespace

int route(const RouteArgs& a, int dtype, cudaStream_t stream, bool* counted) {
  if (counted) *counted = false;
  // every scored level precomputed or row-scored: the warp-per-item router
  bool warp_ok = true;
  for (int l = a.top; l >= 0 && warp_ok; --l) {
    if (l == 0 && a.coarse_only) break;
    const bool dense = a.dense != nullptr && a.dense_off[l] >= 0;
    const bool rowl = (a.row_levels >> l) & 1u;
    if (!dense && !rowl) {
      // unscored levels are fine only when every row takes the all-fit shortcut
      if (a.method == PISA_METHOD_PISA1 || a.levels.size[l] > a.K) warp_ok = false;
    }
  }
  if (a.attend) warp_ok = false;   // the fused decode attention lives in the per-item router
  const int64_t items = int64_t(a.B) * a.t_count * a.H;
  if (warp_ok && items < (int64_t(1) << 31)) {
    if (items == 0) return PISA_OK;
    RouteArgs w = a;
    w.fbr = FastDiv::make(uint32_t(a.br));
    w.fH = FastDiv::make(uint32_t(a.H));
    w.ftc = FastDiv::make(uint32_t(a.t_count));
    const unsigned grid = unsigned((items + 3) / 4);
    TimedLaunch timed(PISA_KERNEL_ROUTER, stream);
    const int max_width = std::max(a.first_width, a.K * a.br);
    if (a.row_levels == 0) {
      // register slots per lane for the widest network of the descent
      if (max_width <= 32) route_warp_kernel<float, 0, 1><<<grid, 128, 0, stream>>>(w);
      else if (max_width <= 64) route_warp_kernel<float, 0, 2><<<grid, 128, 0, stream>>>(w);
      else if (max_width <= 128) route_warp_kernel<float, 0, 4><<<grid, 128, 0, stream>>>(w);
      else route_warp_kernel<float, 0, 8><<<grid, 128, 0, stream>>>(w);
    } else {
      // row-scored levels (planned only for 16-bit inputs, G <= 16 and widths
      // up to 64): pair-steps of 32 head dims
      if (dtype == PISA_F32 || max_width > 64 || a.G > 16)
        return fail(PISA_ERR_UNSUPPORTED, "row-scored levels need fp16/bf16, G <= 16 and widths up to 64");
      const int kp = (a.D + 31) / 32;
      const bool bf = dtype == PISA_BF16;
      if (kp <= 2) {
        if (bf) route_warp_kernel<__nv_bfloat16, 2, 2><<<grid, 128, 0, stream>>>(w);
        else route_warp_kernel<__half, 2, 2><<<grid, 128, 0, stream>>>(w);
      } else if (kp <= 4) {
        if (bf) route_warp_kernel<__nv_bfloat16, 4, 2><<<grid, 128, 0, stream>>>(w);
        else route_warp_kernel<__half, 4, 2><<<grid, 128, 0, stream>>>(w);
      } else {
        if (bf) route_warp_kernel<__nv_bfloat16, 8, 2><<<grid, 128, 0, stream>>>(w);
        else route_warp_kernel<__half, 8, 2><<<grid, 128, 0, stream>>>(w);
      }
    }
    PISA_CHECK_LAUNCH();
    if (counted) *counted = a.fam_counts != nullptr;
    return PISA_OK;
  }
  RouteArgs plain = a;
  plain.fam_counts = nullptr;   // the SIMT router leaves the counting to family_count_kernel
  switch (dtype) {
    case PISA_F32: return route_t<float>(plain, stream);
    case PISA_BF16: return route_t<__nv_bfloat16>(plain, stream);
    case PISA_F16: return route_t<__half>(plain, stream);
  }
  return fail(PISA_ERR_UNSUPPORTED, "unsupported dtype");
}

}  // namespace pisa
