// Backward of the selected-block attention for callers that cannot allocate
// device memory.
//
// pisa_sparse_attn_bwd needs caller-provided scratch: fp32 accumulators for
// dK and dV (B*N*H*(D+Dv)*4 bytes) that start at zero.  Some callers cannot
// hand it over: a host runtime reached only through this C ABI that owns the
// tensors it passes but has no CUDA allocator of its own, or a framework
// whose device memory is fully planned in advance, where an extra
// cudaMalloc would fail or break the plan.  For them this file keeps the
// accumulators in one fixed device array that lives in the library image:
// kScratchBytes (32 MiB) per GPU, held until the process exits.  With lazy
// module loading (the CUDA default since 12.2) the array is reserved on a
// device when the first call there looks up its address, not when the
// library is loaded.  The entry point itself calls no allocator.
#include <cstdio>
#include <mutex>

#include "internal.h"

namespace pisa {
namespace {

constexpr int64_t kScratchBytes = int64_t(32) << 20;
constexpr int kMaxDevices = 64;

// Device-side accumulators of the no-allocation backward.  In host code this
// name is only a stand-in for the symbol, never a usable device address:
// the address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_bwd_scratch[kScratchBytes];

std::mutex g_setup_lock;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_bwd_scratch on the current device, looked up once per
// device (the first call on a device does this set-up).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "pisa_sparse_attn_bwd_noalloc: current device");
  if (dev < 0 || dev >= kMaxDevices) return fail(PISA_ERR_UNSUPPORTED, "pisa_sparse_attn_bwd_noalloc: device index above 63");
  std::lock_guard<std::mutex> hold(g_setup_lock);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bwd_scratch);
    if (e != cudaSuccess || !p) return fail_cuda(e, "pisa_sparse_attn_bwd_noalloc: scratch symbol address");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return PISA_OK;
}

}  // namespace
}  // namespace pisa

extern "C" {

int64_t pisa_sparse_attn_bwd_noalloc_max_bytes(void) { return pisa::kScratchBytes; }

int pisa_sparse_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* out,
                                 const void* dout, const float* lse, const void* indices, int index_bytes,
                                 const int64_t* positions, int64_t position_offset, int dtype, int64_t B,
                                 int64_t Tq, int64_t Hq, int64_t H, int64_t D, int64_t Dv, int64_t N,
                                 int64_t S, int64_t block_size, float scale, int causal, void* dq,
                                 void* dk, void* dv, pisa_stream_t stream) {
  const int64_t need = pisa_sparse_attn_bwd_workspace_bytes(B, Tq, Hq, H, D, Dv, N);
  if (need > pisa::kScratchBytes) {
    char msg[200];
    snprintf(msg, sizeof msg,
             "pisa_sparse_attn_bwd_noalloc: these shapes need %lld bytes of dK/dV accumulators "
             "(pisa_sparse_attn_bwd_workspace_bytes), above the fixed %lld-byte scratch "
             "(pisa_sparse_attn_bwd_noalloc_max_bytes); use pisa_sparse_attn_bwd",
             static_cast<long long>(need), static_cast<long long>(pisa::kScratchBytes));
    return pisa::fail(PISA_ERR_UNSUPPORTED, msg);
  }
  // The array is looked up for the current device while the kernels run on
  // the stream's device: the two must be the same GPU.
  {
    int cur = 0, sdev = 0;
    cudaError_t e = cudaGetDevice(&cur);
    if (e == cudaSuccess) e = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev);
    if (e != cudaSuccess) return pisa::fail_cuda(e, "pisa_sparse_attn_bwd_noalloc: stream device");
    if (cur != sdev)
      return pisa::fail(PISA_ERR_INVALID, "pisa_sparse_attn_bwd_noalloc: the current device must be the stream's device");
  }
  void* scratch = nullptr;
  const int rc = pisa::scratch_address(&scratch);
  if (rc != PISA_OK) return rc;
  // The backward clears the accumulators it uses on `stream` before its kernels run.
  return pisa_sparse_attn_bwd(q, k, v, out, dout, lse, indices, index_bytes, positions, position_offset,
                              dtype, B, Tq, Hq, H, D, Dv, N, S, block_size, scale, causal, dq, dk, dv,
                              scratch, pisa::kScratchBytes, stream);
}

}  // extern "C"
