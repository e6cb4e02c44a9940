// Output-stationary sparse convolution (implicit GEMM over a gather map).
//
// Replaces sparse_conv_forward (trispconv/pytorch/functional.py:14-51) and
// the per-offset Triton gather-GEMM-scatter (triton_kernels.py:31-92): one
// launch covers all K offsets, each output tile accumulates in fp32 in k
// order (the ConvAlgo.Native order of functional.py:40-46) and is stored
// once with bias (and optionally ReLU) fused; no atomics, no zero-fill pass.
#include <cstdint>

#include "conv_launch.h"
#include "tsc_common.cuh"

namespace tsc {
namespace {

constexpr int kConvThreads = 256;
constexpr int kChunkC = 16;  // input channels staged per shared-memory round

// Element (k, c, n) of the weight: internal (K, Cin, Cout) layout
// (weight.py:36 of the reference) or spconv KRSC (Cout, kD, kH, kW, Cin),
// which the kernels read in place.
__device__ __forceinline__ int64_t w_index(int krsc, int k, int c, int n, int K, int c_in, int c_out) {
  return krsc ? (static_cast<int64_t>(n) * K + k) * c_in + c
              : (static_cast<int64_t>(k) * c_in + c) * c_out + n;
}

// Generic SIMT tile: TM output rows x TN output channels per CTA, 4x4 outputs
// per thread, fp32 FFMA.  Works for any dtype and channel count; used for
// fp32 (where TF32 would break the 1e-4 parity bound) and as the fallback.
template <typename T, int TN>
__global__ void __launch_bounds__(kConvThreads)
k_conv_simt(const T* __restrict__ F, int64_t n_in, int c_in, const T* __restrict__ Wt, int w_krsc,
            const T* __restrict__ bias, const int32_t* __restrict__ gmap, int K, int64_t n_out,
            int c_out, const int32_t* __restrict__ ovf, int64_t ovf_cap, const int64_t* __restrict__ meta,
            T* __restrict__ out, int flags, EpiParams epi, int64_t* __restrict__ status) {
  constexpr int CT = TN / 4;              // threads along output channels
  constexpr int RT = kConvThreads / CT;   // threads along rows
  constexpr int TM = RT * 4;              // rows per CTA
  __shared__ float As[kChunkC][TM + 4];   // gathered rows, transposed [c][m]
  __shared__ __align__(16) float Bs[kChunkC][TN];
  __shared__ int rows[TM];

  const int tx = threadIdx.x % CT;
  const int ty = threadIdx.x / CT;
  const int64_t o0 = static_cast<int64_t>(blockIdx.x) * TM;
  const int n0 = blockIdx.y * TN;
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[r][q] = 0.f;

  for (int k = 0; k < K; ++k) {
    int has = 0;
    for (int m = threadIdx.x; m < TM; m += kConvThreads) {
      const int64_t o = o0 + m;
      int j = -1;
      if (o < n_out) {
        j = gmap != nullptr ? __ldg(&gmap[static_cast<int64_t>(k) * n_out + o]) : static_cast<int>(o);
        if (j >= n_in) {
          raise_status(status, TSC_STATUS_KEY_RANGE);
          j = -1;
        }
      }
      rows[m] = j;
      has |= (j >= 0);
    }
    if (!__syncthreads_or(has)) continue;  // no row of this tile has a pair at offset k
    for (int c0 = 0; c0 < c_in; c0 += kChunkC) {
      for (int e = threadIdx.x; e < TM * kChunkC; e += kConvThreads) {
        const int m = e / kChunkC, c = e % kChunkC;
        const int j = rows[m];
        float v = 0.f;
        if (j >= 0 && c0 + c < c_in) v = to_f32(F[static_cast<int64_t>(j) * c_in + c0 + c]);
        As[c][m] = v;
      }
      for (int e = threadIdx.x; e < kChunkC * TN; e += kConvThreads) {
        int c, nn;
        if (w_krsc) {  // (Cout, K, Cin): consecutive threads walk Cin
          nn = e / kChunkC;
          c = e % kChunkC;
        } else {       // (K, Cin, Cout): consecutive threads walk Cout
          c = e / TN;
          nn = e % TN;
        }
        float v = 0.f;
        if (c0 + c < c_in && n0 + nn < c_out) v = to_f32(Wt[w_index(w_krsc, k, c0 + c, n0 + nn, K, c_in, c_out)]);
        Bs[c][nn] = v;
      }
      __syncthreads();
#pragma unroll
      for (int c = 0; c < kChunkC; ++c) {
        float a[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) a[r] = As[c][ty * 4 + r];
        const float4 b = *reinterpret_cast<const float4*>(&Bs[c][tx * 4]);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          acc[r][0] = fmaf(a[r], b.x, acc[r][0]);
          acc[r][1] = fmaf(a[r], b.y, acc[r][1]);
          acc[r][2] = fmaf(a[r], b.z, acc[r][2]);
          acc[r][3] = fmaf(a[r], b.w, acc[r][3]);
        }
      }
      __syncthreads();
    }
  }

  // Pairs that did not fit the gather map (duplicate input coordinates only);
  // their count is read on the device so the host never has to synchronise.
  int64_t n_ovf = 0;
  if (ovf != nullptr && meta != nullptr) {
    n_ovf = static_cast<int64_t>(__ldg(&meta[TSC_META_N_OVERFLOW]));
    if (n_ovf > ovf_cap) n_ovf = ovf_cap;
  }
  for (int64_t e = 0; e < n_ovf; ++e) {
    const int k = __ldg(&ovf[3 * e + 0]);
    const int64_t o = __ldg(&ovf[3 * e + 1]);
    const int j = __ldg(&ovf[3 * e + 2]);
    const int64_t m = o - o0;
    if (m < ty * 4 || m >= ty * 4 + 4 || k < 0 || k >= K || j < 0 || j >= n_in) continue;
    const int r = static_cast<int>(m - ty * 4);
    for (int c = 0; c < c_in; ++c) {
      const float f = to_f32(F[static_cast<int64_t>(j) * c_in + c]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int n = n0 + tx * 4 + q;
        if (n < c_out) acc[r][q] = fmaf(f, to_f32(Wt[w_index(w_krsc, k, c, n, K, c_in, c_out)]), acc[r][q]);
      }
    }
  }

#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t o = o0 + ty * 4 + r;
    if (o >= n_out) continue;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int n = n0 + tx * 4 + q;
      if (n >= c_out) continue;
      out[o * c_out + n] = from_f32<T>(epi_apply(acc[r][q], n, epi, bias));
    }
  }
}

template <typename T>
int launch_simt(const void* F, int64_t n_in, int c_in, const void* W, int w_krsc, const void* bias,
                const int32_t* gmap, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
                const int64_t* meta, void* out, int flags, const EpiParams& epi, int64_t* status, cudaStream_t stream) {
  const T* f = static_cast<const T*>(F);
  const T* w = static_cast<const T*>(W);
  const T* bs = static_cast<const T*>(bias);
  T* o = static_cast<T*>(out);
  if (c_out <= 16) {
    constexpr int TN = 16, TM = (kConvThreads / (TN / 4)) * 4;
    dim3 grid(static_cast<unsigned>(ceil_div(n_out, TM)), static_cast<unsigned>(ceil_div(c_out, TN)));
    k_conv_simt<T, TN><<<grid, kConvThreads, 0, stream>>>(f, n_in, c_in, w, w_krsc, bs, gmap, K, n_out, c_out,
                                                          ovf, ovf_cap, meta, o, flags, epi, status);
  } else if (c_out <= 32) {
    constexpr int TN = 32, TM = (kConvThreads / (TN / 4)) * 4;
    dim3 grid(static_cast<unsigned>(ceil_div(n_out, TM)), static_cast<unsigned>(ceil_div(c_out, TN)));
    k_conv_simt<T, TN><<<grid, kConvThreads, 0, stream>>>(f, n_in, c_in, w, w_krsc, bs, gmap, K, n_out, c_out,
                                                          ovf, ovf_cap, meta, o, flags, epi, status);
  } else {
    constexpr int TN = 64, TM = (kConvThreads / (TN / 4)) * 4;
    dim3 grid(static_cast<unsigned>(ceil_div(n_out, TM)), static_cast<unsigned>(ceil_div(c_out, TN)));
    k_conv_simt<T, TN><<<grid, kConvThreads, 0, stream>>>(f, n_in, c_in, w, w_krsc, bs, gmap, K, n_out, c_out,
                                                          ovf, ovf_cap, meta, o, flags, epi, status);
  }
  TSC_LAUNCH_CHECK("k_conv_simt");
  return TSC_OK;
}

template <typename T>
__global__ void __launch_bounds__(256)
k_to_dense(const T* __restrict__ F, const int4* __restrict__ idx, int64_t n, int C, int B, int D, int H,
           int W, int channels_first, T* __restrict__ out, int64_t* __restrict__ status) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= n * C) return;
  const int64_t i = t / C;
  const int ch = static_cast<int>(t - i * C);
  const int4 c = __ldg(&idx[i]);
  if (static_cast<unsigned>(c.x) >= static_cast<unsigned>(B) ||
      static_cast<unsigned>(c.y) >= static_cast<unsigned>(D) ||
      static_cast<unsigned>(c.z) >= static_cast<unsigned>(H) ||
      static_cast<unsigned>(c.w) >= static_cast<unsigned>(W)) {
    if (ch == 0) raise_status(status, TSC_STATUS_KEY_RANGE);
    return;
  }
  size_t off;
  if (channels_first) {
    off = ((((static_cast<size_t>(c.x) * C + ch) * D + c.y) * H + c.z) * W) + c.w;
  } else {
    off = ((((static_cast<size_t>(c.x) * D + c.y) * H + c.z) * W + c.w) * C) + ch;
  }
  out[off] = F[t];
}

template <typename T>
int launch_dense(const void* F, const int32_t* indices, int64_t n, int C, int B, const int32_t* s,
                 int cf, void* out, int64_t* status, cudaStream_t stream) {
  const int64_t total = n * C;
  k_to_dense<T><<<static_cast<unsigned>(ceil_div(total, 256)), 256, 0, stream>>>(
      static_cast<const T*>(F), reinterpret_cast<const int4*>(indices), n, C, B, s[0], s[1], s[2], cf,
      static_cast<T*>(out), status);
  TSC_LAUNCH_CHECK("k_to_dense");
  return TSC_OK;
}

size_t dtype_size(int dtype) {
  switch (dtype) {
    case TSC_F32: return 4;
    case TSC_F16: return 2;
    case TSC_BF16: return 2;
    case TSC_F64: return 8;
    default: return 0;
  }
}

}  // namespace
}  // namespace tsc

using namespace tsc;

namespace {

// Argument checks and kernel choice shared by tsc_conv_forward and
// tsc_conv_forward_halo.
int conv_forward(ConvArgs a, int32_t dtype, int32_t weight_layout) {
  const int64_t n_in = a.n_in, n_out = a.n_out;
  const int c_in = a.c_in, c_out = a.c_out, k_vol = a.k_vol, flags = a.flags;
  TSC_CHECK_ARG(c_in > 0 && c_out > 0, "channel counts must be positive (c_in=%d, c_out=%d)", c_in, c_out);
  TSC_CHECK_ARG(k_vol > 0 && k_vol <= 4096, "kernel volume %d out of range", k_vol);
  TSC_CHECK_ARG(n_in >= 0 && n_in <= 0x7fffffffLL && n_out >= 0 && n_out <= 0x7fffffffLL,
                "row counts out of range");
  TSC_CHECK_ARG(a.status != nullptr, "status is NULL");
  TSC_CHECK_ARG(a.gather_map != nullptr || (k_vol == 1 && n_in == n_out),
                "identity map requires K == 1 and n_in == n_out");
  if (n_out == 0) return TSC_OK;
  TSC_CHECK_ARG(a.out != nullptr && a.weight != nullptr, "NULL buffer");
  TSC_CHECK_ARG(n_in == 0 || a.features != nullptr, "features is NULL");
  TSC_CHECK_ARG(aligned(a.weight, 16) && aligned(a.out, 16) && (a.features == nullptr || aligned(a.features, 16)),
                "features/weight/out must be 16-byte aligned");
  TSC_CHECK_ARG(weight_layout == TSC_W_KCC || weight_layout == TSC_W_KRSC, "bad weight layout %d",
                weight_layout);
  TSC_CHECK_ARG(a.bias == nullptr || aligned(a.bias, 4), "bias must be 4-byte aligned");
  TSC_CHECK_ARG(a.overflow == nullptr || (a.meta != nullptr && a.overflow_cap >= 0),
                "overflow list needs its meta buffer");
  TSC_CHECK_ARG(a.epi.act >= TSC_ACT_NONE && a.epi.act <= TSC_ACT_SILU, "unknown activation %d", a.epi.act);
  TSC_CHECK_ARG((a.epi.scale == nullptr) == (a.epi.shift == nullptr), "epilogue scale and shift go together");
  TSC_CHECK_ARG(a.epi.scale == nullptr || (aligned(a.epi.scale, 4) && aligned(a.epi.shift, 4)),
                "epilogue scale/shift must be 4-byte aligned");
  if ((flags & TSC_CONV_RELU) != 0) {
    TSC_CHECK_ARG(a.epi.act == TSC_ACT_NONE || a.epi.act == TSC_ACT_RELU,
                  "TSC_CONV_RELU and activation %d both requested", a.epi.act);
    a.epi.act = TSC_ACT_RELU;
  }
  const int w_krsc = weight_layout == TSC_W_KRSC;
  const bool force_simt = (flags & TSC_CONV_FORCE_SIMT) != 0;
  const bool f16 = dtype == TSC_F16;
  if (!force_simt && (flags & TSC_CONV_USE_TC) != 0) {
    // the one-tile-per-CTA kernel only on request (testing); otherwise the
    // persistent kernels where their tile shapes apply, else mma.sync below
    if ((flags & TSC_CONV_TC_SIMPLE) != 0 && tc_eligible(dtype, w_krsc, c_in, c_out, k_vol))
      return f16 ? launch_tc_f16(a) : launch_tc_bf16(a);
    if (n_in > 0 && (flags & TSC_CONV_TC_SIMPLE) == 0 && a.halo_map != nullptr && a.gather_map != nullptr &&
        a.row_order == nullptr && a.overflow == nullptr && a.halo_planes == 3 &&
        tmh_eligible(dtype, w_krsc, c_in, c_out, k_vol) && a.halo_capacity == tmh_capacity(c_out))
      return f16 ? launch_tmh_f16(a) : launch_tmh_bf16(a);
    if (n_in > 0 && tcp_eligible(dtype, w_krsc, c_in, c_out, k_vol) && (flags & TSC_CONV_TC_SIMPLE) == 0)
      return f16 ? launch_tcp_f16(a) : launch_tcp_bf16(a);
  }
  if (!force_simt && (flags & TSC_CONV_NO_RG) == 0 && rg_eligible(dtype, w_krsc, c_in, c_out, k_vol) &&
      n_out <= 0x7fffff00LL)
    return f16 ? launch_rg_f16(a) : launch_rg_bf16(a);
  if (!force_simt && mma_eligible(dtype, w_krsc, c_in, c_out, k_vol))
    return f16 ? launch_mma_f16(a) : launch_mma_bf16(a);
  // the CUDA-core kernel walks rows in index order; results do not depend on
  // the row order, so it is ignored here
  switch (dtype) {
    case TSC_F32:
      return launch_simt<float>(a.features, n_in, c_in, a.weight, w_krsc, a.bias, a.gather_map, k_vol, n_out, c_out,
                                a.overflow, a.overflow_cap, a.meta, a.out, flags, a.epi, a.status, a.stream);
    case TSC_F16:
      return launch_simt<__half>(a.features, n_in, c_in, a.weight, w_krsc, a.bias, a.gather_map, k_vol, n_out, c_out,
                                 a.overflow, a.overflow_cap, a.meta, a.out, flags, a.epi, a.status, a.stream);
    case TSC_BF16:
      return launch_simt<__nv_bfloat16>(a.features, n_in, c_in, a.weight, w_krsc, a.bias, a.gather_map, k_vol, n_out,
                                        c_out, a.overflow, a.overflow_cap, a.meta, a.out, flags, a.epi, a.status, a.stream);
    default:
      set_error("unsupported dtype code %d for the convolution", dtype);
      return TSC_ERR_UNSUPPORTED;
  }
}

}  // namespace

extern "C" {

int tsc_conv_forward(const void* features, int32_t dtype, int64_t n_in, int32_t c_in, const void* weight,
                     int32_t weight_layout, const void* bias, const int32_t* gather_map, const int32_t* row_order,
                     int32_t k_vol, int64_t n_out, int32_t c_out, const int32_t* overflow, int64_t overflow_cap,
                     const int64_t* meta, void* out, int32_t flags, int64_t* status, uint32_t* tile_counter,
                     void* stream) {
  const ConvArgs a{features, n_in,     c_in,  weight, bias,   gather_map,   row_order,
                   k_vol,    n_out,    c_out, overflow, overflow_cap, meta, out,
                   flags,    status,   tile_counter, static_cast<cudaStream_t>(stream)};
  return conv_forward(a, dtype, weight_layout);
}

int tsc_conv_forward_ex(const void* features, int32_t dtype, int64_t n_in, int32_t c_in, const void* weight,
                        int32_t weight_layout, const void* bias, const int32_t* gather_map, const int32_t* row_order,
                        int32_t k_vol, int64_t n_out, int32_t c_out, const int32_t* overflow, int64_t overflow_cap,
                        const int64_t* meta, void* out, int32_t flags, int64_t* status, uint32_t* tile_counter,
                        const tsc_conv_extras* extras, void* stream) {
  ConvArgs a{features, n_in,     c_in,  weight, bias,   gather_map,   row_order,
             k_vol,    n_out,    c_out, overflow, overflow_cap, meta, out,
             flags,    status,   tile_counter, static_cast<cudaStream_t>(stream)};
  if (extras != nullptr) {
    const tsc_conv_extras& x = *extras;
    TSC_CHECK_ARG(x.halo_map == nullptr || (x.halo_rows != nullptr && x.halo_count != nullptr &&
                                            x.plane_kmask != nullptr && aligned(x.halo_rows, 16)),
                  "halo_map needs halo_rows (16-byte aligned), halo_count and plane_kmask");
    a.halo_rows = x.halo_rows;
    a.halo_count = x.halo_count;
    a.plane_kmask = x.plane_kmask;
    a.halo_map = x.halo_map;
    a.halo_planes = x.halo_planes;
    a.halo_capacity = x.halo_capacity;
    a.epi = EpiParams{x.scale, x.shift, x.act, x.act_alpha};
  }
  return conv_forward(a, dtype, weight_layout);
}

int32_t tsc_conv_halo_capacity(int32_t dtype, int32_t c_in, int32_t c_out, int32_t k_vol, int32_t flags) {
  if ((flags & TSC_CONV_USE_TC) == 0 || (flags & (TSC_CONV_TC_SIMPLE | TSC_CONV_FORCE_SIMT)) != 0) return 0;
  if (!tmh_eligible(dtype, 1, c_in, c_out, k_vol)) return 0;
  return tmh_capacity(c_out);
}

int tsc_to_dense(const void* features, int32_t dtype, const int32_t* indices, int64_t n, int32_t c,
                 int32_t batch, const int32_t* shape3, int32_t channels_first, void* out, int64_t* status,
                 void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  TSC_CHECK_ARG(c > 0 && batch > 0 && shape3 != nullptr, "bad dense() arguments");
  TSC_CHECK_ARG(shape3[0] > 0 && shape3[1] > 0 && shape3[2] > 0, "spatial_shape must be positive");
  TSC_CHECK_ARG(status != nullptr && out != nullptr, "NULL buffer");
  const size_t es = dtype_size(dtype);
  TSC_CHECK_ARG(es != 0, "unsupported dtype code %d", dtype);
  const size_t total = static_cast<size_t>(batch) * c * shape3[0] * shape3[1] * shape3[2];
  TSC_CUDA(cudaMemsetAsync(out, 0, total * es, stream));
  if (n == 0) return TSC_OK;
  TSC_CHECK_ARG(indices != nullptr && aligned(indices, 16), "indices must be 16-byte aligned");
  TSC_CHECK_ARG(features != nullptr, "features is NULL");
  switch (dtype) {
    case TSC_F32: return launch_dense<float>(features, indices, n, c, batch, shape3, channels_first, out, status, stream);
    case TSC_F16: return launch_dense<__half>(features, indices, n, c, batch, shape3, channels_first, out, status, stream);
    case TSC_BF16: return launch_dense<__nv_bfloat16>(features, indices, n, c, batch, shape3, channels_first, out, status, stream);
    case TSC_F64: return launch_dense<double>(features, indices, n, c, batch, shape3, channels_first, out, status, stream);
    default: return TSC_ERR_UNSUPPORTED;
  }
}

}  // extern "C"
