// Device status words: how a bounded device-side wait that expired reaches
// the caller.
//
// Every kernel that waits on an mbarrier (the tile pipelines, the dense
// coarse-level scorer) waits a bounded number of tries; when a wait gives up,
// the kernel records PISA_ERR_TIMEOUT in the status word at byte offset 0 of
// the call's workspace, releases what it holds and returns.  The entry point
// clears that word on the stream before its kernels run, so after the stream
// reaches the end of the call the word holds the call's outcome.
// pisa_workspace_status reads it back (one 4-byte copy and a stream
// synchronisation); pisa_wait_selftest exercises the whole path with a wait
// on a barrier that nothing ever arrives on.
#include "internal.h"
#include "tc.cuh"

namespace pisa {

namespace {

// One warp: an mbarrier expecting one arrival.  With `arrive` the barrier
// completes before the wait; without it nothing arrives and the bounded wait
// gives up after `max_tries` tries and records the timeout.  No asynchronous
// copy or tensor-core operation is issued, so an expired wait leaves nothing
// in flight.
__global__ void wait_selftest_kernel(int arrive, uint32_t max_tries, int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
  }
  __syncwarp();
  if (arrive && threadIdx.x == 0) tc::mbar_arrive(&bar);
  __syncwarp();
  bool ok = true;
  if (threadIdx.x == 0) ok = tc::mbar_wait(&bar, 0, max_tries);
  if (!ok) atomicExch(status, PISA_ERR_TIMEOUT);
}

// Both exponentials of the leaf epilogue on the same inputs: the polynomial
// form (tc::ex2_poly2) and ex2.approx.
__global__ void ex2_selftest_kernel(const float* x, float* poly, float* mufu, int64_t n) {
  const int64_t i = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) * 2;
  if (i >= n) return;
  const float2 v = make_float2(x[i], i + 1 < n ? x[i + 1] : 0.f);
  const float2 p = tc::ex2_poly2(v);
  poly[i] = p.x;
  mufu[i] = tc::ex2f(v.x);
  if (i + 1 < n) {
    poly[i + 1] = p.y;
    mufu[i + 1] = tc::ex2f(v.y);
  }
}

}  // namespace

}  // namespace pisa

extern "C" {

int pisa_ex2_selftest(const float* x, float* poly, float* mufu, int64_t n, pisa_stream_t stream) {
  if (n < 0 || (n > 0 && (!x || !poly || !mufu))) return pisa::fail(PISA_ERR_INVALID, "x, poly and mufu are required");
  if (n == 0) return PISA_OK;
  const int64_t pairs = (n + 1) / 2;
  pisa::ex2_selftest_kernel<<<unsigned((pairs + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, poly, mufu, n);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

int pisa_workspace_status(const void* workspace, pisa_stream_t stream) {
  if (!workspace) return pisa::fail(PISA_ERR_INVALID, "workspace is required");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int word = 0;
  cudaError_t e = cudaMemcpyAsync(&word, workspace, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return pisa::fail_cuda(e, "status read");
  if (word == PISA_OK) return PISA_OK;
  if (word == PISA_ERR_TIMEOUT)
    return pisa::fail(PISA_ERR_TIMEOUT, "a bounded device-side wait expired; the call's results are not valid");
  return pisa::fail(PISA_ERR_CUDA, "unexpected device status word");
}

int pisa_wait_selftest(int arrive, int64_t max_tries, void* workspace, int64_t workspace_bytes,
                       pisa_stream_t stream) {
  if (!workspace || workspace_bytes < 256) return pisa::fail(PISA_ERR_INVALID, "a 256-byte workspace is required");
  if (max_tries < 1 || max_tries > (int64_t(1) << 30)) return pisa::fail(PISA_ERR_INVALID, "max_tries out of range");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(workspace, 0, 256, s);
  if (e != cudaSuccess) return pisa::fail_cuda(e, "status clear");
  pisa::wait_selftest_kernel<<<1, 32, 0, s>>>(arrive ? 1 : 0, uint32_t(max_tries), static_cast<int*>(workspace));
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

}  // extern "C"
