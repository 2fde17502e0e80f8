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
// The leaf pass is HBM-bound: every key byte is read once with 16-byte
// vector loads, one CTA per (leaf block, batch), each thread owning 16-byte
// columns of the [H*D] row and walking the block's tokens with eight loads in
// flight.  Upper levels are <1% of the traffic (a few MB at 256K tokens).
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

template <typename T>
static int pyramid_impl(const void* keys, int64_t B, int64_t N, int64_t H, int64_t D, int64_t sb,
                        int64_t st, int64_t sh, int64_t C, int64_t br, int64_t levels,
                        void* storage, int64_t ssb, const int64_t* offs, int64_t first_token,
                        cudaStream_t stream) {
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
