// Per-kernel device timing: CUDA events recorded on the launch stream around
// the launches of the tile kernels, summed on read.  Used by the benchmark to
// put a measured duration under the roofline of one kernel.
#include <atomic>
#include <mutex>
#include <vector>

#include "internal.h"

namespace pisa {

namespace {

struct Pool {
  std::vector<cudaEvent_t> start, stop;
  size_t used = 0;
  int64_t launches = 0;
};

std::mutex g_lock;
bool g_on = false;
Pool g_pool[PISA_KERNEL_COUNT];
std::atomic<int64_t> g_launches{0};

}  // namespace

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

TimedLaunch::TimedLaunch(int kernel, cudaStream_t stream) : kernel_(kernel), slot_(-1), stream_(stream) {
  std::lock_guard<std::mutex> hold(g_lock);
  if (!g_on || kernel < 0 || kernel >= PISA_KERNEL_COUNT) return;
  Pool& p = g_pool[kernel];
  if (p.used == p.start.size()) {
    cudaEvent_t a = nullptr, b = nullptr;
    if (cudaEventCreate(&a) != cudaSuccess) return;
    if (cudaEventCreate(&b) != cudaSuccess) {
      cudaEventDestroy(a);
      return;
    }
    p.start.push_back(a);
    p.stop.push_back(b);
  }
  if (cudaEventRecord(p.start[p.used], stream) != cudaSuccess) return;
  slot_ = int(p.used++);
}

TimedLaunch::~TimedLaunch() {
  if (slot_ < 0) return;
  std::lock_guard<std::mutex> hold(g_lock);
  Pool& p = g_pool[kernel_];
  cudaEventRecord(p.stop[slot_], stream_);
  ++p.launches;
}

}  // namespace pisa

extern "C" {

int64_t pisa_launch_count(void) { return pisa::g_launches.load(std::memory_order_relaxed); }

int pisa_kernel_timing(int enable) {
  std::lock_guard<std::mutex> hold(pisa::g_lock);
  pisa::g_on = enable != 0;
  return PISA_OK;
}

int pisa_kernel_time(int kernel, double* total_ms, int64_t* launches) {
  if (kernel < 0 || kernel >= PISA_KERNEL_COUNT || !total_ms || !launches)
    return pisa::fail(PISA_ERR_INVALID, "pisa_kernel_time: unknown kernel or null output");
  std::lock_guard<std::mutex> hold(pisa::g_lock);
  pisa::Pool& p = pisa::g_pool[kernel];
  double sum = 0.0;
  for (size_t i = 0; i < p.used; ++i) {
    cudaError_t e = cudaEventSynchronize(p.stop[i]);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, p.start[i], p.stop[i]);
    if (e != cudaSuccess) {
      p.used = 0;
      p.launches = 0;
      return pisa::fail_cuda(e, "pisa_kernel_time");
    }
    sum += ms;
  }
  *total_ms = sum;
  *launches = p.launches;
  p.used = 0;
  p.launches = 0;
  return PISA_OK;
}

}  // extern "C"
