// Host-side utilities of the C ABI: error strings, launch accounting, device
// attributes.
#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "tsc_common.cuh"

namespace tsc {

static thread_local char g_err[1024] = "";
static std::atomic<unsigned long long> g_launches{0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("launch of %s failed: %s", what, cudaGetErrorString(e));
    return TSC_ERR_CUDA;
  }
  return TSC_OK;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace tsc

extern "C" {

int tsc_abi_version(void) { return TSC_ABI_VERSION; }

const char* tsc_last_error(void) { return tsc::g_err; }

unsigned long long tsc_launch_count(void) {
  return tsc::g_launches.load(std::memory_order_relaxed);
}

}  // extern "C"
