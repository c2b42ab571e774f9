// Library-wide entry points: version, error reporting, device attribute cache.
#include "ak_common.cuh"

#include <mutex>

namespace ak {

static thread_local char g_last_error[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = 0; }

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace ak

extern "C" int ak_version(void) { return (0 << 16) | (1 << 8) | 0; }

extern "C" const char* ak_last_error(void) { return ak::g_last_error; }

// ---------------------------------------------------------------------------
// Device status words
// ---------------------------------------------------------------------------
namespace ak {
namespace {

// One thread arms an mbarrier that expects one arrival, then waits on it with
// the given poll limit.  Nothing ever arrives, so the wait runs out, the status
// word receives AK_ERR_TIMEOUT and the kernel returns.  No copy is in flight on
// the barrier, so abandoning it is harmless.
__global__ void bounded_wait_probe(int* status, uint32_t max_spins) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  mbar_fence_init();
  mbar_wait_bounded(&bar, 0u, status, max_spins);
}

}  // namespace
}  // namespace ak

extern "C" int ak_status_device_pointer(void* host_word, void** dev_ptr) {
  ak::clear_error();
  AK_REQUIRE(host_word != nullptr && dev_ptr != nullptr, AK_ERR_ARG, "ak_status_device_pointer: null pointer");
  AK_CUDA_TRY(cudaHostGetDevicePointer(dev_ptr, host_word, 0), "ak_status_device_pointer");
  return AK_OK;
}

extern "C" int ak_test_bounded_wait(int* status, int max_spins, void* stream) {
  ak::clear_error();
  AK_REQUIRE(max_spins >= 1 && max_spins <= (1 << 20), AK_ERR_ARG,
             "ak_test_bounded_wait: max_spins must be in [1, 2^20], got %d", max_spins);
  cudaStream_t st = (cudaStream_t)stream;
  ak::bounded_wait_probe<<<1, 32, 0, st>>>(status, (uint32_t)max_spins);
  AK_CHECK_LAUNCH("ak_test_bounded_wait");
  return AK_OK;
}
