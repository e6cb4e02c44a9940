// Shared device/host helpers for the trispconv_b200 CUDA library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "trispconv_b200.h"

namespace tsc {

// ---- host-side error reporting ------------------------------------------------
void set_error(const char* fmt, ...);
void count_launch();
// Checks cudaGetLastError() after a launch; records `what` on failure.
int check_launch(const char* what);

#define TSC_CHECK_ARG(cond, ...)                                             \
  do {                                                                       \
    if (!(cond)) {                                                           \
      ::tsc::set_error(__VA_ARGS__);                                         \
      return TSC_ERR_INVALID_ARG;                                            \
    }                                                                        \
  } while (0)

#define TSC_CUDA(call)                                                       \
  do {                                                                       \
    cudaError_t e_ = (call);                                                 \
    if (e_ != cudaSuccess) {                                                 \
      ::tsc::set_error("%s failed: %s", #call, cudaGetErrorString(e_));      \
      return TSC_ERR_CUDA;                                                   \
    }                                                                        \
  } while (0)

#define TSC_LAUNCH_CHECK(what)                                               \
  do {                                                                       \
    ::tsc::count_launch();                                                   \
    int rc_ = ::tsc::check_launch(what);                                     \
    if (rc_ != TSC_OK) return rc_;                                           \
  } while (0)

// ---- programmatic dependent launch -------------------------------------------
// Kernels launched with launch_pdl may be scheduled while the previous kernel
// of the stream is still running, which hides the launch gap between
// dependent kernels.  Every kernel that launch_pdl starts calls pdl_wait()
// before it touches global memory (it then sees everything the previous grid
// wrote, and that grid has finished reading) and pdl_trigger() to let the next
// kernel be scheduled once all of its own CTAs have started.  Both are no-ops
// for a kernel launched the ordinary way.  TRISPCONV_B200_PDL=0 turns the
// attribute off (ordinary launches).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Launches through launch_pdl and checks the result like TSC_LAUNCH_CHECK.
#define TSC_LAUNCH_PDL(what, kern, grid, block, smem, stream, ...)                   \
  do {                                                                              \
    cudaError_t e_ = ::tsc::launch_pdl(kern, grid, block, smem, stream, __VA_ARGS__); \
    if (e_ != cudaSuccess) {                                                        \
      ::tsc::set_error("launch of %s failed: %s", what, cudaGetErrorString(e_));    \
      return TSC_ERR_CUDA;                                                          \
    }                                                                               \
    TSC_LAUNCH_CHECK(what);                                                         \
  } while (0)

// Fills n1 32-bit words at p1 with v1 and n2 words at p2 with v2 (p2 may be
// NULL) in one PDL launch: the stream's memsets of the hot path, as a kernel
// that joins the dependent-launch chain.
int fill_words(void* p1, uint32_t v1, int64_t n1, void* p2, uint32_t v2, int64_t n2, cudaStream_t stream);

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Cached multiprocessor count of the current device.
int sm_count();

// ---- device helpers -------------------------------------------------------------
constexpr unsigned long long kEmptySlot = ~0ull;
constexpr unsigned kFullMask = 0xffffffffu;

__device__ __forceinline__ void raise_status(int64_t* status, long long bits) {
  atomicOr(reinterpret_cast<unsigned long long*>(status), static_cast<unsigned long long>(bits));
}

// Slot of a 32-bit linear cell key in a power-of-two table (log2cap >= 8):
// Fibonacci hashing of key >> 3, keeping the low 3 bits, so 8 cells that are
// consecutive along x land in 8 consecutive slots (one or two cache sectors
// for a warp querying neighbouring voxels).
__device__ __forceinline__ uint32_t hash_slot(uint32_t key, int log2cap) {
  const uint32_t hi = static_cast<uint32_t>((static_cast<unsigned long long>(key >> 3) * 0x9E3779B97F4A7C15ull) >>
                                            (64 - (log2cap - 3)));
  return (hi << 3) | (key & 7u);
}

// Kernel offset decomposition, k = (kz*kH + ky)*kW + kx.
struct KOffset {
  int kz, ky, kx;
};
__device__ __forceinline__ KOffset split_k(int k, int kH, int kW) {
  KOffset r;
  r.kx = k % kW;
  int t = k / kW;
  r.ky = t % kH;
  r.kz = t / kH;
  return r;
}

// Element conversions.
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// ---- convolution epilogue ------------------------------------------------------
// Per output channel n: out = act(acc * scale[n] + shift[n]) when scale is set
// (an eval-mode BatchNorm folded into the store, the conv bias inside shift),
// else act(acc + bias[n]).  Computed in fp32 and rounded once to the output
// type.
struct EpiParams {
  const float* scale;
  const float* shift;
  int act;      // TSC_ACT_*
  float alpha;  // negative slope of TSC_ACT_LEAKY_RELU
};

__device__ __forceinline__ float activate(float x, int act, float alpha) {
  switch (act) {
    case TSC_ACT_RELU: return fmaxf(x, 0.f);
    case TSC_ACT_LEAKY_RELU: return x >= 0.f ? x : x * alpha;
    // x * sigmoid(x) from the fast exponential and division intrinsics (a
    // few ulp in fp32; -0 for very negative x)
    case TSC_ACT_SILU: return __fdividef(x, 1.f + __expf(-x));
    default: return x;
  }
}

template <typename T>
__device__ __forceinline__ float epi_apply(float v, int n, const EpiParams& e, const T* __restrict__ bias) {
  if (e.scale != nullptr)
    v = fmaf(v, __ldg(&e.scale[n]), __ldg(&e.shift[n]));
  else if (bias != nullptr)
    v += to_f32(bias[n]);
  return activate(v, e.act, e.alpha);
}

// Eight consecutive output channels n..n+7 of one row: the common bias (+
// ReLU) store as its own loop, the general epilogue otherwise (one uniform
// branch per eight values).
template <typename T>
__device__ __forceinline__ void epi_store8(const float* v, int n, const EpiParams& e, const T* __restrict__ bias,
                                           T (&h)[8]) {
  if (e.scale == nullptr && e.act <= TSC_ACT_RELU) {
    const bool relu = e.act == TSC_ACT_RELU;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float x = v[i];
      if (bias != nullptr) x += to_f32(bias[n + i]);
      if (relu) x = fmaxf(x, 0.f);
      h[i] = from_f32<T>(x);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = from_f32<T>(epi_apply(v[i], n + i, e, bias));
  }
}

// Block-wide exclusive scan of one uint32 per thread (blockDim.x multiple of 32,
// at most 1024).  `warp_sums` must hold 32 entries.  Returns the exclusive prefix
// and writes the block total to *total.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_sums,
                                                         uint32_t* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    uint32_t y = __shfl_up_sync(kFullMask, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < nwarps ? warp_sums[lane] : 0u;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      uint32_t y = __shfl_up_sync(kFullMask, w, d);
      if (lane >= d) w += y;
    }
    if (lane < nwarps) warp_sums[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  uint32_t warp_off = warp > 0 ? warp_sums[warp - 1] : 0u;
  uint32_t tot = warp_sums[nwarps - 1];
  __syncthreads();  // warp_sums may be reused by the caller right after
  *total = tot;
  return warp_off + x - v;
}

// 64-bit variant for offsets that may exceed 2^32 (pair lists).
__device__ __forceinline__ unsigned long long block_exclusive_scan64(unsigned long long v,
                                                                     unsigned long long* warp_sums,
                                                                     unsigned long long* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  unsigned long long x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    unsigned long long y = __shfl_up_sync(kFullMask, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    unsigned long long w = lane < nwarps ? warp_sums[lane] : 0ull;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      unsigned long long y = __shfl_up_sync(kFullMask, w, d);
      if (lane >= d) w += y;
    }
    if (lane < nwarps) warp_sums[lane] = w;
  }
  __syncthreads();
  unsigned long long warp_off = warp > 0 ? warp_sums[warp - 1] : 0ull;
  unsigned long long tot = warp_sums[nwarps - 1];
  __syncthreads();
  *total = tot;
  return warp_off + x - v;
}

}  // namespace tsc
