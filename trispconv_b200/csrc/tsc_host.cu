// Host-side utilities of the C ABI: error strings, launch accounting, device
// attributes.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>

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

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("TRISPCONV_B200_PDL");
    return !(e != nullptr && e[0] == '0' && e[1] == '\0');
  }();
  return on;
}

namespace {

// one index space over both ranges; 16-byte stores where a range allows them
__global__ void __launch_bounds__(256) k_fill_words(uint32_t* __restrict__ p1, uint32_t v1, int64_t n1,
                                                    uint32_t* __restrict__ p2, uint32_t v2, int64_t n2) {
  pdl_wait();
  pdl_trigger();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int r = 0; r < 2; ++r) {
    uint32_t* p = r ? p2 : p1;
    const uint32_t v = r ? v2 : v1;
    const int64_t n = r ? n2 : n1;
    if (p == nullptr || n <= 0) continue;
    int64_t head = 0;
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
      const int64_t nv = n / 4;
      const uint4 q = make_uint4(v, v, v, v);
      for (int64_t i = t0; i < nv; i += stride) reinterpret_cast<uint4*>(p)[i] = q;
      head = nv * 4;
    }
    for (int64_t i = head + t0; i < n; i += stride) p[i] = v;
  }
}

}  // namespace

int fill_words(void* p1, uint32_t v1, int64_t n1, void* p2, uint32_t v2, int64_t n2, cudaStream_t stream) {
  const int64_t work = (n1 > 0 ? (n1 + 3) / 4 : 0) + (n2 > 0 ? (n2 + 3) / 4 : 0);
  if (work == 0) return TSC_OK;
  int64_t blocks = ceil_div(work, 256);
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  TSC_LAUNCH_PDL("k_fill_words", k_fill_words, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                 static_cast<uint32_t*>(p1), v1, n1, static_cast<uint32_t*>(p2), v2, n2);
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
