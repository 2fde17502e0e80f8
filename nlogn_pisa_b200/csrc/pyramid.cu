// K1: mean-pooled key pyramid (leaf means, then pools of `branching` nodes).
//
// Semantics follow torch_mean_pool (pisa/pisa/ops/compress/mean_pooling/
// mean_pooling_torch.py:7-14) and build_pyramid (mean_pooling.py:45-52):
// fp32 sums over the valid tokens of a block, divided by the real count
// (a tail block divides by what it has), rounded to the key dtype after every
// level, so level l+1 pools the *rounded* level l exactly as the reference.
//
// Layout: all levels live in one storage [B, total, H, D] (node stride H*D),
// level l starting at node offset level_offsets[l].
//
// A full build is two launches.  pyramid_group_kernel reads every key byte
// once (16-byte vector loads) and writes the leaves and the lowest k levels:
// one CTA per (group of L = br^k leaves, batch), one thread per (leaf,
// 16-byte column of the whole node row, all KV heads) walking the leaf's
// tokens with sixteen loads in flight, so warps read whole contiguous key rows
// and no cross-thread reduction is needed; the group's upper nodes are pooled
// from the rounded leaf means held in shared memory.
// pyramid_top_kernel then pools the remaining levels per (batch, KV head),
// launched with programmatic dependent launch so that its launch overlaps the
// group pass (it waits on griddepcontrol.wait for the group grid to finish).
// Incremental updates (first_token > 0) recompute only the touched leaves and
// their ancestors with one launch per level (leaf_mean_kernel,
// parent_mean_kernel).
#include <algorithm>

#include "internal.h"

namespace pisa {

template <typename T>
__global__ void __launch_bounds__(256)
leaf_mean_kernel(const T* __restrict__ keys, int64_t sb, int64_t st, int64_t sh, int N, int H,
                 int D, int size, int first_leaf, T* __restrict__ out, int64_t out_sb,
                 int64_t out_off) {
  constexpr int V = Vec<T>::N;
  const int leaf = first_leaf + blockIdx.x;
  const int b = blockIdx.y;
  const int chunks = H * D / V;
  const int64_t t0 = int64_t(leaf) * size;
  const int64_t t1 = min64(t0 + size, N);
  const float count = float(t1 - t0);
  const T* base = keys + b * sb;
  T* dst = out + b * out_sb + (out_off + leaf) * int64_t(H) * D;
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
    const int e = c * V;
    const int h = e / D, d = e % D;
    const T* p = base + h * sh + d;
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
    int64_t t = t0;
    for (; t + 8 <= t1; t += 8) {
      float x[8][V];
#pragma unroll
      for (int u = 0; u < 8; ++u) load_vec<T>(p + (t + u) * st, x[u]);
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] += x[u][i];
    }
    for (; t < t1; ++t) {
      float x[V];
      load_vec<T>(p + t * st, x);
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] += x[i];
    }
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = acc[i] / count;
    store_vec<T>(dst + e, acc);
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
parent_mean_kernel(T* storage, int64_t sb, int64_t child_off, int child_len, int64_t parent_off,
                   int first_parent, int branching, int HD) {
  constexpr int V = Vec<T>::N;
  const int node = first_parent + blockIdx.x;
  const int b = blockIdx.y;
  const int c0 = node * branching;
  const int c1 = min(c0 + branching, child_len);
  const float count = float(c1 - c0);
  T* base = storage + b * sb;
  for (int c = threadIdx.x; c < HD / V; c += blockDim.x) {
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
    for (int ch = c0; ch < c1; ++ch) {
      float x[V];
      load_vec_cg<T>(base + (child_off + ch) * HD + c * V, x);
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] += x[i];
    }
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = acc[i] / count;
    store_vec<T>(base + (parent_off + node) * HD + c * V, acc);
  }
}

constexpr int kTopThreads = 1024;
constexpr int kLeafThreads = 512;   // threads of a group CTA (wider node rows take the per-level launches)

// acc[i] += element i of a raw 16-byte vector of T.
template <typename T>
__device__ __forceinline__ void add_raw(uint4 raw, float (&acc)[Vec<T>::N]) {
  if constexpr (sizeof(T) == 4) {
    acc[0] += __uint_as_float(raw.x); acc[1] += __uint_as_float(raw.y);
    acc[2] += __uint_as_float(raw.z); acc[3] += __uint_as_float(raw.w);
  } else {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < Vec<T>::N; ++i) acc[i] += to_f32<T>(e[i]);
  }
}

// Leaves and the lowest k_local levels of one group of L leaves of one batch
// row: thread (leaf lane, 16-byte column of the whole [H*D] node row) sums a
// leaf's tokens for its column, so every warp reads whole contiguous key rows
// (all heads of a token are adjacent) and no cross-thread reduction is needed.
template <typename T>
__global__ void __launch_bounds__(kLeafThreads)
pyramid_group_kernel(const T* __restrict__ keys, int64_t sb, int64_t st, int64_t sh, int N, int H, int D, int C,
                     int br, int L, int k_local, T* __restrict__ out, int64_t out_sb, const LevelTable lv) {
  constexpr int V = Vec<T>::N;
  // let the dependent top-level launch start; it waits for this grid to finish
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ float pool[];   // rounded node values of the group: levels 0..k_local, [node][H*D]
  const int HD = H * D;
  const int CH = HD / V;            // 16-byte columns of one node row
  const int TL = blockDim.x / CH;   // leaf lanes
  const int col = threadIdx.x % CH, lane_leaf = threadIdx.x / CH;
  const int group = blockIdx.x;
  const int b = blockIdx.y;
  const int n_leaves = lv.size[0];
  const int e = col * V, h = e / D, d = e - h * D;
  const T* src_base = keys + b * sb + h * sh + d;
  T* out_b = out + b * out_sb;
  if (lane_leaf < TL) {
    for (int li = lane_leaf; li < L; li += TL) {
      const int leaf = group * L + li;
      if (leaf >= n_leaves) break;
      const int64_t t0 = int64_t(leaf) * C;
      const int64_t t1 = min64(t0 + C, N);
      float acc[V];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = 0.f;
      int64_t t = t0;
      // sixteen raw 16-byte loads in flight, summed in token order
      for (; t + 16 <= t1; t += 16) {
        uint4 raw[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) raw[u] = __ldg(reinterpret_cast<const uint4*>(src_base + (t + u) * st));
#pragma unroll
        for (int u = 0; u < 16; ++u) add_raw<T>(raw[u], acc);
      }
      for (; t < t1; ++t) add_raw<T>(__ldg(reinterpret_cast<const uint4*>(src_base + t * st)), acc);
      const float count = float(t1 - t0);
      float* keep = pool + li * HD + e;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        acc[i] = to_f32<T>(from_f32<T>(acc[i] / count));   // rounded as the stored level
        keep[i] = acc[i];
      }
      store_vec<T>(out_b + (lv.offset[0] + leaf) * int64_t(HD) + e, acc);
    }
  }
  // levels 1 .. k_local of this group from the rounded values below them
  int child_base = 0, width = L;
  for (int l = 1; l <= k_local; ++l) {
    __syncthreads();
    const int nodes = width / br;
    const int parent_base = child_base + width;
    const int first = group * nodes;               // global index of the group's first node at level l
    for (int item = threadIdx.x; item < nodes * CH; item += blockDim.x) {
      const int j = item / CH, c = item - j * CH;
      const int node = first + j;
      if (node >= lv.size[l]) continue;
      const int c0 = node * br, c1 = min(c0 + br, lv.size[l - 1]);
      float acc[V];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = 0.f;
      for (int ch = c0; ch < c1; ++ch) {
        const float* x = pool + (child_base + (ch - group * width)) * HD + c * V;
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] += x[i];
      }
      const float count = float(c1 - c0);
      float* keep = pool + (parent_base + j) * HD + c * V;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        acc[i] = to_f32<T>(from_f32<T>(acc[i] / count));
        keep[i] = acc[i];
      }
      store_vec<T>(out_b + (lv.offset[l] + node) * int64_t(HD) + c * V, acc);
    }
    child_base = parent_base;
    width = nodes;
  }
}

// Levels first_level .. levels-1 of one (batch, KV head), level by level from
// the stored level below (read through L2: written by the group grid or by
// this CTA's previous level).
template <typename T>
__global__ void __launch_bounds__(kTopThreads)
pyramid_top_kernel(T* storage, int64_t sb, int H, int D, int br, int first_level, int levels, const LevelTable lv) {
  constexpr int V = Vec<T>::N;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int CH = D / V;
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  T* base = storage + b * sb + int64_t(h) * D;
  const int64_t node_stride = int64_t(H) * D;
  for (int l = first_level; l < levels; ++l) {
    if (l > first_level) __syncthreads();
    for (int item = threadIdx.x; item < lv.size[l] * CH; item += blockDim.x) {
      const int node = item / CH, c = item % CH;
      const int c0 = node * br, c1 = min(c0 + br, lv.size[l - 1]);
      float acc[V];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = 0.f;
      for (int ch = c0; ch < c1; ++ch) {
        float x[V];
        load_vec_cg<T>(base + (lv.offset[l - 1] + ch) * node_stride + c * V, x);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] += x[i];
      }
      const float count = float(c1 - c0);
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = acc[i] / count;
      store_vec<T>(base + (lv.offset[l] + node) * node_stride + c * V, acc);
    }
  }
}

// Full build (first_token == 0) in two launches; *done stays false when the
// shape is outside the group kernel (the per-level launches then run).
template <typename T>
static int pyramid_full(const void* keys, int64_t B, int64_t N, int64_t H, int64_t D, int64_t sb, int64_t st,
                        int64_t sh, int64_t C, int64_t br, int64_t levels, void* storage, int64_t ssb,
                        const int64_t* offs, cudaStream_t stream, bool* done) {
  *done = false;
  constexpr int V = Vec<T>::N;
  const int64_t CH = H * D / V;     // 16-byte columns of a node row
  if (D % V || CH < 1 || CH > kLeafThreads || B > 65535) return PISA_OK;
  const int TL = int(std::max<int64_t>(1, kLeafThreads / CH));
  // local levels: groups of L = br^k leaves with L <= TL (one leaf per lane)
  // and the group's nodes within 64 KB of shared memory
  int k = 0, L = 1, pool_nodes = 1;
  while (k + 1 < levels && L * br <= TL && size_t(pool_nodes + L * br) * H * D * sizeof(float) <= 64 * 1024) {
    L *= int(br);
    pool_nodes = 0;
    for (int w = L; w >= 1; w /= int(br)) pool_nodes += w;
    ++k;
  }
  if (k == 0) { L = TL; pool_nodes = TL; }   // leaves only in this pass: one per lane
  const size_t smem = size_t(pool_nodes) * H * D * sizeof(float);
  if (smem > 96 * 1024) return PISA_OK;
  LevelTable lv{};
  int64_t n = (N + C - 1) / C;
  for (int64_t l = 0; l < levels; ++l) {
    lv.offset[l] = offs[l];
    lv.size[l] = int32_t(n);
    n = (n + br - 1) / br;
  }
  const int64_t groups = (int64_t(lv.size[0]) + L - 1) / L;
  if (groups > INT32_MAX) return PISA_OK;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(pyramid_group_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(smem));
    if (e != cudaSuccess) return fail_cuda(e, "pyramid smem attribute");
  }
  *done = true;
  TimedLaunch timed(PISA_KERNEL_PYRAMID, stream);
  const dim3 grid(static_cast<unsigned>(groups), static_cast<unsigned>(B), 1u);
  const int threads = int(std::min<int64_t>(kLeafThreads, int64_t(TL) * CH));
  pyramid_group_kernel<T><<<grid, threads, smem, stream>>>(
      static_cast<const T*>(keys), sb, st, sh, int(N), int(H), int(D), int(C), int(br), L, k,
      static_cast<T*>(storage), ssb, lv);
  PISA_CHECK_LAUNCH();
  if (k + 1 < levels) {
    if (B * H > 65535) return fail(PISA_ERR_UNSUPPORTED, "batch x heads too large for the pyramid's top levels");
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(B * H));
    cfg.blockDim = dim3(kTopThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, pyramid_top_kernel<T>, static_cast<T*>(storage), ssb, int(H),
                                       int(D), int(br), k + 1, int(levels), lv);
    if (e != cudaSuccess) return fail_cuda(e, "pyramid top levels");
    PISA_CHECK_LAUNCH();
  }
  return PISA_OK;
}

template <typename T>
static int pyramid_impl(const void* keys, int64_t B, int64_t N, int64_t H, int64_t D, int64_t sb,
                        int64_t st, int64_t sh, int64_t C, int64_t br, int64_t levels,
                        void* storage, int64_t ssb, const int64_t* offs, int64_t first_token,
                        cudaStream_t stream) {
  if (first_token == 0 && levels <= kMaxLevels) {
    bool done = false;
    int rc = pyramid_full<T>(keys, B, N, H, D, sb, st, sh, C, br, levels, storage, ssb, offs, stream, &done);
    if (rc || done) return rc;
  }
  const int threads = 128;
  TimedLaunch timed(PISA_KERNEL_PYRAMID, stream);
  int64_t n = (N + C - 1) / C;
  int64_t first = first_token / C;
  if (n - first > 0) {
    dim3 grid(unsigned(n - first), unsigned(B));
    leaf_mean_kernel<T><<<grid, threads, 0, stream>>>(
        static_cast<const T*>(keys), sb, st, sh, int(N), int(H), int(D), int(C), int(first),
        static_cast<T*>(storage), ssb, offs[0]);
    PISA_CHECK_LAUNCH();
  }
  for (int64_t l = 1; l < levels; ++l) {
    const int64_t parents = (n + br - 1) / br;
    const int64_t pfirst = first / br;
    if (parents - pfirst > 0) {
      dim3 grid(unsigned(parents - pfirst), unsigned(B));
      parent_mean_kernel<T><<<grid, threads, 0, stream>>>(
          static_cast<T*>(storage), ssb, offs[l - 1], int(n), offs[l], int(pfirst), int(br),
          int(H * D));
      PISA_CHECK_LAUNCH();
    }
    n = parents;
    first = pfirst;
  }
  return PISA_OK;
}

int build_pyramid(const void* keys, int dtype, int64_t B, int64_t N, int64_t H, int64_t D,
                  int64_t sb, int64_t st, int64_t sh, int64_t C, int64_t br, int64_t levels,
                  void* storage, int64_t ssb, const int64_t* offs, int64_t first_token,
                  cudaStream_t stream) {
  switch (dtype) {
    case PISA_F32: return pyramid_impl<float>(keys, B, N, H, D, sb, st, sh, C, br, levels, storage, ssb, offs, first_token, stream);
    case PISA_BF16: return pyramid_impl<__nv_bfloat16>(keys, B, N, H, D, sb, st, sh, C, br, levels, storage, ssb, offs, first_token, stream);
    case PISA_F16: return pyramid_impl<__half>(keys, B, N, H, D, sb, st, sh, C, br, levels, storage, ssb, offs, first_token, stream);
  }
  return fail(PISA_ERR_UNSUPPORTED, "unsupported dtype");
}

}  // namespace pisa
