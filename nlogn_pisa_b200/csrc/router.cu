// K2: coarse-to-fine router (and, in the fused schedule, leaf scoring + top-K).
//
// One CTA of four warps routes one (batch, query token, KV head) item through
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
#include "internal.h"
#include "score.cuh"

namespace pisa {

namespace {

constexpr int kThreads = 128;
constexpr int kMaxWidth = 256;

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
      } else if (out) {
        out[i] = (v < 0 || int64_t(v) * C > pos) ? -1 : v;
      }
    }
  }
}

template <typename T, int GMAX>
__global__ void __launch_bounds__(kThreads) route_kernel(const RouteArgs a) {
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
  for (int e = tid; e < a.G * a.D; e += kThreads) {
    const int g = e / a.D, d = e % a.D;
    qs[e] = to_f32<T>(qp[g * a.q_sh + d]);
  }
  int width = a.first_width;
  for (int w = tid; w < width; w += kThreads) ids[w] = w;
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
    for (int w = tid; w < width; w += kThreads) {
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
      for (int w = tid; w < width; w += kThreads) {
        const int f = fl[w];
        const bool scoreable = (f & 1) && !(f & 2) && !identity;
        dst[w] = ids[w];
        fdst[w] = uint8_t(f | (scoreable ? 4 : 0));
      }
      return;
    }

    // fill values and thread-per-candidate scoring
    const bool warp_leaf = level == 0 && a.method != PISA_METHOD_PISA1 && a.dense_off[0] < 0;
    for (int w = tid; w < width; w += kThreads) {
      const int f = fl[w];
      const bool valid = f & 1, forced = f & 2;
      const bool scoreable = valid && !forced && !identity;
      float v = 0.f;
      if (scoreable && !warp_leaf && dense_row && a.dense_off[level] >= 0) {
        v = dense_row[a.dense_off[level] + ids[w]];
      } else if (scoreable && !warp_leaf) {
        if (a.method == PISA_METHOD_PISA1) {
          v = coarse_score<T, GMAX>(a, summary + a.levels.offset[level] * node_stride, len, ids[w], qs);
        } else {
          v = coarse_score<T, GMAX>(a, summary + a.levels.offset[level - 1] * node_stride,
                                    a.levels.size[level - 1], ids[w], qs);
        }
      }
      sc[w] = !valid ? kNegFill : (forced ? kPosFill : v);
    }
    if (warp_leaf) {
      __syncthreads();
      for (int w = warp; w < width; w += kThreads / 32) {
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
}

// Warp-per-item router for descents whose every scored level has precomputed
// scores (dense.cu): levels >= 1 for pisa/pisa2 when the leaf level is left to
// the grouped tensor-core scorer (coarse_only), every level for pisa1.  The
// candidates and scores live in registers (element i in lane i%32, slot
// i/32), validity is counted with ballots, and the same comparison network
// picks the K survivors; their children are expanded through shared memory.
template <int WP>
__device__ __forceinline__ void warp_sort(float (&s)[8], int (&id)[8], int lane) {
  float ss[Network<WP>::E];
  int ii[Network<WP>::E];
#pragma unroll
  for (int e = 0; e < Network<WP>::E; ++e) { ss[e] = s[e]; ii[e] = id[e]; }
  Network<WP>::sort(ss, ii, lane);
#pragma unroll
  for (int e = 0; e < Network<WP>::E; ++e) { s[e] = ss[e]; id[e] = ii[e]; }
}

__global__ void __launch_bounds__(128) route_warp_kernel(const RouteArgs a) {
  __shared__ int kept[4][64];
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
  const float* dense_row = a.dense + local * a.dense_stride;
  const int64_t leaf = pos / a.C;
  // forced-recent leaves leaf-r (r < force_recent, leaf-r >= 0) have, at any
  // level, ancestors forming the contiguous id range [lo_leaf / div, leaf / div]
  const int64_t lo_leaf = leaf - a.force_recent + 1 > 0 ? leaf - a.force_recent + 1 : 0;
  int64_t span = a.C, div = 1;
  for (int l = 0; l < a.top; ++l) { span *= a.br; div *= a.br; }

  int id[8];
  float sc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) id[e] = e * 32 + lane;   // top level: 0..first_width-1
  int width = a.first_width;
  for (int level = a.top; level >= 0; --level) {
    const int len = a.levels.size[level];
    const int64_t f_hi = leaf >= 0 ? leaf / div : -1, f_lo = leaf >= 0 ? lo_leaf / div : 0;
    bool valid[8], forced[8];
    int nvalid = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
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
      for (int e = 0; e < 8; ++e) {
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
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const bool scoreable = valid[e] && !forced[e] && !identity;
      float v = scoreable ? dense_row[off + id[e]] : 0.f;
      sc[e] = !valid[e] ? kNegFill : (forced[e] ? kPosFill : v);
      if (e * 32 + lane >= width) { sc[e] = kNegFill; id[e] = -1; }
    }
    switch (width) {
      case 16: warp_sort<16>(sc, id, lane); break;
      case 32: warp_sort<32>(sc, id, lane); break;
      case 64: warp_sort<64>(sc, id, lane); break;
      case 128: warp_sort<128>(sc, id, lane); break;
      default: warp_sort<256>(sc, id, lane); break;
    }
    if (level == 0) {
      int64_t* out = a.out_ids + item * a.K;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = e * 32 + lane;
        if (i < a.K) out[i] = (id[e] < 0 || int64_t(id[e]) * a.C > pos) ? -1 : id[e];
      }
      return;
    }
    // survivors -> shared memory -> children in network order
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int i = e * 32 + lane;
      if (i < a.K) kept[warp][i] = id[e];
    }
    __syncwarp();
    width = a.K * a.br;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int i = e * 32 + lane;
      const int q = int(a.fbr.div(uint32_t(i)));
      const int parent = i < width ? kept[warp][q] : -1;
      id[e] = parent < 0 ? -1 : parent * a.br + (i - q * a.br);
    }
    __syncwarp();
    span /= a.br;
    div /= a.br;
  }
}

template <typename T, int GMAX>
int launch_route(const RouteArgs& a, cudaStream_t stream) {
  const size_t smem = size_t(a.G) * a.D * sizeof(float) + kMaxWidth * (2 * sizeof(int) + 1);
  auto kernel = route_kernel<T, GMAX>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return fail_cuda(e, "route smem attribute");
  }
  const int64_t items = int64_t(a.B) * a.t_count * a.H;
  if (items == 0) return PISA_OK;
  TimedLaunch timed(PISA_KERNEL_ROUTER, stream);
  kernel<<<unsigned(items), kThreads, smem, stream>>>(a);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

template <typename T>
int route_t(const RouteArgs& a, cudaStream_t stream) {
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
  // every scored level precomputed: the warp-per-item router
  bool all_dense = a.dense != nullptr;
  for (int l = a.top; l >= 0 && all_dense; --l) {
    if (l == 0 && a.coarse_only) break;
    if (a.dense_off[l] < 0) {
      // unscored levels are fine only when every row takes the all-fit shortcut
      if (a.method == PISA_METHOD_PISA1 || a.levels.size[l] > a.K) all_dense = false;
    }
  }
  const int64_t items = int64_t(a.B) * a.t_count * a.H;
  if (all_dense && items < (int64_t(1) << 31)) {
    if (items == 0) return PISA_OK;
    RouteArgs w = a;
    w.fbr = FastDiv::make(uint32_t(a.br));
    w.fH = FastDiv::make(uint32_t(a.H));
    w.ftc = FastDiv::make(uint32_t(a.t_count));
    TimedLaunch timed(PISA_KERNEL_ROUTER, stream);
    route_warp_kernel<<<unsigned((items + 3) / 4), 128, 0, stream>>>(w);
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
