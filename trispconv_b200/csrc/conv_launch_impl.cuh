// Template launchers of the tensor-core conv kernels.  Each
// conv_launch_*.cu translation unit instantiates one kernel family for one
// element type, so the library compiles in parallel.
#pragma once

#include <cuda.h>
#include <type_traits>

#include "conv_launch.h"
#include "conv_mma.cuh"
#include "conv_tc.cuh"
#include "conv_tmh.cuh"
#include <cstdlib>
#include "conv_tcp.cuh"
#include "tsc_common.cuh"

namespace tsc {
namespace detail {

static_assert(tcp::KMAX == kPersistentKMax, "persistent kernel K limit");

// The general store epilogue is needed for a folded BatchNorm or an
// activation other than ReLU.
inline bool epi_general(const EpiParams& e) { return e.scale != nullptr || e.act > TSC_ACT_RELU; }
static_assert(mma::KMAX == kMmaKMax && tc::KMAX == kMmaKMax, "kernel K limits");

// ---- tensor-core (mma.sync) path -------------------------------------------

// Persistent mma.sync kernel with the column tile's weights resident in
// shared memory (one channel chunk, weights <= mma::kMaxResidentWeightBytes).
template <typename T, int TN, int KC, int CH>
int launch_mmaw_cfg(const T* f, int64_t n_in, int c_in, const T* w, const T* bias, const int32_t* gmap,
                    const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
                    const int64_t* meta, T* out, int flags, const EpiParams& epi, int64_t* status, cudaStream_t stream) {
  using C = mma::CfgW<TN, KC>;
  auto kern = mma::k_conv_mmaw<T, TN, KC, CH>;
  constexpr int kMaxSmem = C::MAIN + mma::kMaxResidentWeightBytes + (mma::KMAX * mma::BM + mma::BM + mma::KMAX + 8) * 4;
  static unsigned long long configured = 0;
  static int ctas_per_sm[mma::KMAX + 1][64] = {};  // [K][device]: 0 = not computed yet
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (!(configured & (1ull << dev))) {
    TSC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
    configured |= 1ull << dev;
  }
  const int smem = C::bytes(K);
  int& occ = ctas_per_sm[K][dev];
  if (occ == 0) {
    TSC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, mma::NT, smem));
    if (occ < 1) occ = 1;
  }
  const int64_t row_tiles = ceil_div(n_out, mma::BM);
  const int64_t cap = static_cast<int64_t>(sm_count()) * occ;
  dim3 grid(static_cast<unsigned>(row_tiles < cap ? row_tiles : cap), static_cast<unsigned>(ceil_div(c_out, TN)));
  TSC_LAUNCH_PDL("k_conv_mmaw", kern, grid, dim3(mma::NT), smem, stream, f, n_in, c_in, w, bias, gmap, perm, K,
                 n_out, c_out, ovf, ovf_cap, meta, out, flags, epi, status);
  return TSC_OK;
}

// Streamed-weight mma.sync kernel with RB output rows per CTA.
template <typename T, int TN, int KC, int CH, int RB>
int launch_mma_rows(const T* f, int64_t n_in, int c_in, const T* w, const T* bias, const int32_t* gmap,
                    const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
                    const int64_t* meta, T* out, int flags, const EpiParams& epi, int64_t* status, cudaStream_t stream) {
  using C = mma::Cfg<TN, KC, RB>;
  auto kern = mma::k_conv_mma<T, TN, KC, CH, RB>;
  static unsigned long long configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    TSC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::TOTAL));
    configured |= 1ull << (dev & 63);
  }
  dim3 grid(static_cast<unsigned>(ceil_div(n_out, RB)), static_cast<unsigned>(ceil_div(c_out, TN)));
  TSC_LAUNCH_PDL("k_conv_mma", kern, grid, dim3(mma::NT), C::bytes(K), stream, f, n_in, c_in, w, bias, gmap, perm,
                 K, n_out, c_out, ovf, ovf_cap, meta, out, flags, epi, status);
  return TSC_OK;
}

template <typename T, int TN, int KC, int CH>
int launch_mma_cfg(const T* f, int64_t n_in, int c_in, const T* w, const T* bias, const int32_t* gmap,
                   const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
                   const int64_t* meta, T* out, int flags, const EpiParams& epi, int64_t* status, cudaStream_t stream) {
  if ((flags & TSC_CONV_NO_RESIDENT_W) == 0 && c_in <= KC && K <= mma::KMAX &&
      static_cast<int64_t>(K) * TN * KC * 2 <= mma::kMaxResidentWeightBytes)
    return launch_mmaw_cfg<T, TN, KC, CH>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta,
                                          out, flags, epi, status, stream);
  // 16-channel chunks with narrow column tiles take 2 * BM rows per CTA (each
  // weight slice then serves twice the rows).  Measured on the config-3 maps:
  // 16->32 71.0 -> 68.5 us; 32-channel layers got slower (32->32 102 -> 113
  // us, 32->64 123 -> 132 us) because the larger tile halves the CTAs per SM.
  if constexpr (KC == 16 && TN <= 32) {
    if (n_out >= 4096)
      return launch_mma_rows<T, TN, KC, CH, 2 * mma::BM>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf,
                                                         ovf_cap, meta, out, flags, epi, status, stream);
  }
  return launch_mma_rows<T, TN, KC, CH, mma::BM>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap,
                                                 meta, out, flags, epi, status, stream);
}

// ---- tcgen05 path ------------------------------------------------------------

template <typename T, int TN, int KC>
int launch_tc_cfg(const T* f, int64_t n_in, int c_in, const T* w, const T* bias, const int32_t* gmap,
                  const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
                  const int64_t* meta, T* out, int flags, const EpiParams& epi, int64_t* status, cudaStream_t stream) {
  using C = tc::Cfg<TN, KC>;
  auto kern = tc::k_conv_tc<T, TN, KC>;
  const int smem = C::TOTAL_FIXED + K * tc::BM * 4;
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    TSC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  C::TOTAL_FIXED + tc::KMAX * tc::BM * 4));
    configured |= 1ull << (dev & 63);
  }
  dim3 grid(static_cast<unsigned>(ceil_div(n_out, tc::BM)), static_cast<unsigned>(ceil_div(c_out, TN)));
  kern<<<grid, tc::NT, smem, stream>>>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta,
                                       out, flags, epi, status);
  TSC_LAUNCH_CHECK("k_conv_tc");
  return TSC_OK;
}

template <typename T, int TN>
int launch_tc_tn(const T* f, int64_t n_in, int c_in, const T* w, const T* bias, const int32_t* gmap,
                 const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
                 const int64_t* meta, T* out, int flags, const EpiParams& epi, int64_t* status, cudaStream_t stream) {
  if (c_in <= 16)
    return launch_tc_cfg<T, TN, 16>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, out,
                                    flags, epi, status, stream);
  if (c_in <= 32)
    return launch_tc_cfg<T, TN, 32>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, out,
                                    flags, epi, status, stream);
  return launch_tc_cfg<T, TN, 64>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, out,
                                  flags, epi, status, stream);
}

// ---- persistent tcgen05 path ---------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library does not link libcuda directly).
inline int encode_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
      set_error("cuTensorMapEncodeTiled is not available from the driver");
      return TSC_ERR_CUDA;
    }
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  *out = fn;
  return TSC_OK;
}

template <typename T>
constexpr CUtensorMapDataType tma_dtype() {
  return std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

template <int KC>
constexpr CUtensorMapSwizzle tma_swizzle() {
  return KC == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : (KC == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// Features [n_in][c_in] as a 2-D tensor {c_in, n_in}, box {KC, 1} (gather4),
// and KRSC weights [c_out][K][c_in] as a 3-D tensor {c_in, K, c_out}, box
// {KC, 1, TN}; both swizzled like the UMMA K-major operand tiles.  The
// kernel issues only boxes and gather rows that lie inside the tensors.
template <typename T, int TN, int KC>
int encode_maps(const T* f, int64_t n_in, int c_in, const T* w, int K, int c_out, CUtensorMap* mf, CUtensorMap* mw) {
  EncodeTiledFn enc;
  int rc = encode_fn(&enc);
  if (rc != TSC_OK) return rc;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(c_in), static_cast<cuuint64_t>(n_in)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(c_in) * sizeof(T)};
    cuuint32_t box[2] = {KC, 1};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(mf, tma_dtype<T>(), 2, const_cast<T*>(f), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     tma_swizzle<KC>(), CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled(features) failed with %d", static_cast<int>(r));
      return TSC_ERR_CUDA;
    }
  }
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(c_in), static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(c_out)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(c_in) * sizeof(T),
                             static_cast<cuuint64_t>(K) * c_in * sizeof(T)};
    cuuint32_t box[3] = {KC, 1, TN};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(mw, tma_dtype<T>(), 3, const_cast<T*>(w), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     tma_swizzle<KC>(), CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled(weights) failed with %d", static_cast<int>(r));
      return TSC_ERR_CUDA;
    }
  }
  return TSC_OK;
}

template <typename T, int TN, int KC>
int launch_tcp_cfg(const T* f, int64_t n_in, int c_in, const T* w, const T* bias, const int32_t* gmap,
                   const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
                   const int64_t* meta, T* out, int flags, const EpiParams& epi, int64_t* status, uint32_t* tile_counter,
                   cudaStream_t stream) {
  using C = tcp::Cfg<TN, KC>;
  auto kern = epi_general(epi) ? tcp::k_conv_tcp<T, TN, KC, true> : tcp::k_conv_tcp<T, TN, KC, false>;
  CUtensorMap mf, mw;
  int rc = encode_maps<T, TN, KC>(f, n_in, c_in, w, K, c_out, &mf, &mw);
  if (rc != TSC_OK) return rc;
  static unsigned long long configured[2] = {0, 0};
  int dev = 0;
  cudaGetDevice(&dev);
  const int gen = epi_general(epi) ? 1 : 0;
  if (!(configured[gen] & (1ull << (dev & 63)))) {
    TSC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::TOTAL));
    configured[gen] |= 1ull << (dev & 63);
  }
  const int64_t tiles = ceil_div(n_out, tcp::BMT) * ceil_div(c_out, TN);
  const int64_t grid = tiles < sm_count() ? tiles : sm_count();
  if (tile_counter != nullptr) {
    rc = fill_words(tile_counter, 0u, 1, nullptr, 0u, 0, stream);
    if (rc != TSC_OK) return rc;
  }
  TSC_LAUNCH_PDL("k_conv_tcp", kern, dim3(static_cast<unsigned>(grid)), dim3(tcp::NT), C::TOTAL, stream, mf, mw, f,
                 n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, out, flags, epi, status,
                 tile_counter);
  return TSC_OK;
}

template <typename T, int TN>
int launch_tcp_tn(const T* f, int64_t n_in, int c_in, const T* w, const T* bias, const int32_t* gmap,
                  const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
                  const int64_t* meta, T* out, int flags, const EpiParams& epi, int64_t* status, uint32_t* tile_counter,
                   cudaStream_t stream) {
  // KC = 64 divides c_in (tcp_eligible): every feature and weight box lies inside its tensor
  return launch_tcp_cfg<T, TN, 64>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, out,
                                   flags, epi, status, tile_counter, stream);
}

template <typename T>
int launch_tcp(const void* F, int64_t n_in, int c_in, const void* W, const void* bias, const int32_t* gmap,
               const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
               const int64_t* meta, void* out, int flags, const EpiParams& epi, int64_t* status, uint32_t* tile_counter,
               cudaStream_t stream) {
  const T* f = static_cast<const T*>(F);
  const T* w = static_cast<const T*>(W);
  const T* b = static_cast<const T*>(bias);
  T* o = static_cast<T*>(out);
  // the largest UMMA N that divides c_out (tcp_eligible: c_out % 32 == 0)
  if (c_out % 256 == 0)
    return launch_tcp_tn<T, 256>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                                 status, tile_counter, stream);
  if (c_out % 128 == 0)
    return launch_tcp_tn<T, 128>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                                 status, tile_counter, stream);
  if (c_out % 64 == 0)
    return launch_tcp_tn<T, 64>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                                 status, tile_counter, stream);
  return launch_tcp_tn<T, 32>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                                 status, tile_counter, stream);
}


// ---- persistent tcgen05 path with per-plane halos, A in tensor memory ---------

template <typename T, int TN, int NS>
int launch_tmh_tn(const ConvArgs& a) {
  using C = tmh::Cfg<TN, NS>;
  auto kern = epi_general(a.epi) ? tmh::k_conv_tmh<T, TN, NS, true> : tmh::k_conv_tmh<T, TN, NS, false>;
  const T* f = static_cast<const T*>(a.features);
  const T* w = static_cast<const T*>(a.weight);
  CUtensorMap mf, mw;
  // gather4 rows of 64 channels (the whole row) and weight boxes {64, 1, TN}
  int rc = encode_maps<T, TN, tmh::KC>(f, a.n_in, a.c_in, w, a.k_vol, a.c_out, &mf, &mw);
  if (rc != TSC_OK) return rc;
  static unsigned long long configured[2] = {0, 0};
  int dev = 0;
  cudaGetDevice(&dev);
  const int gen = epi_general(a.epi) ? 1 : 0;
  if (!(configured[gen] & (1ull << (dev & 63)))) {
    TSC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::TOTAL));
    configured[gen] |= 1ull << (dev & 63);
  }
  const int64_t tiles = ceil_div(a.n_out, tmh::BMT);
  const int64_t grid = tiles < sm_count() ? tiles : sm_count();
  TSC_LAUNCH_PDL("k_conv_tmh", kern, dim3(static_cast<unsigned>(grid)), dim3(tmh::NT), C::TOTAL, a.stream, mf, mw, f,
                 a.n_in, static_cast<const T*>(a.bias), a.gather_map, a.n_out, a.halo_rows, a.halo_count,
                 a.plane_kmask, a.halo_map, a.halo_capacity, static_cast<T*>(a.out), a.flags, a.epi, a.status);
  return TSC_OK;
}

inline int tmh_capacity_of(int c_out) {
  return c_out == 64 ? tmh::Cfg<64, 4>::HALO : (c_out == 128 ? tmh::Cfg<128, 4>::HALO : 0);
}

// Stage count of the 64-channel halo kernel: TRISPCONV_B200_TMH_STAGES (4 or
// 6; 6 leaves one accumulator buffer), read once.
inline int tmh_stages() {
  static int ns = [] {
    const char* e = std::getenv("TRISPCONV_B200_TMH_STAGES");
    return (e != nullptr && std::atoi(e) == 6) ? 6 : 4;
  }();
  return ns;
}

template <typename T>
int launch_tmh(const ConvArgs& a) {
  if (a.c_out == 64) return tmh_stages() == 6 ? launch_tmh_tn<T, 64, 6>(a) : launch_tmh_tn<T, 64, 4>(a);
  return launch_tmh_tn<T, 128, 4>(a);
}

template <typename T>
int launch_tc(const void* F, int64_t n_in, int c_in, const void* W, const void* bias, const int32_t* gmap,
              const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
              const int64_t* meta, void* out, int flags, const EpiParams& epi, int64_t* status, cudaStream_t stream) {
  const T* f = static_cast<const T*>(F);
  const T* w = static_cast<const T*>(W);
  const T* b = static_cast<const T*>(bias);
  T* o = static_cast<T*>(out);
  if (c_out <= 32)
    return launch_tc_tn<T, 32>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                               status, stream);
  if (c_out <= 64)
    return launch_tc_tn<T, 64>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                               status, stream);
  if (c_out <= 128)
    return launch_tc_tn<T, 128>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                                status, stream);
  return launch_tc_tn<T, 256>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                              status, stream);
}

template <typename T, int TN>
int launch_mma_tn(const T* f, int64_t n_in, int c_in, const T* w, const T* bias, const int32_t* gmap,
                  const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
                  const int64_t* meta, T* out, int flags, const EpiParams& epi, int64_t* status, cudaStream_t stream) {
  if (c_in <= 16) {
    if (c_in % 8 == 0)
      return launch_mma_cfg<T, TN, 16, 16>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta,
                                           out, flags, epi, status, stream);
    return launch_mma_cfg<T, TN, 16, 8>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta,
                                        out, flags, epi, status, stream);
  }
  if (c_in <= 32)
    return launch_mma_cfg<T, TN, 32, 16>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta,
                                         out, flags, epi, status, stream);
  return launch_mma_cfg<T, TN, 64, 16>(f, n_in, c_in, w, bias, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, out,
                                       flags, epi, status, stream);
}


template <typename T>
int launch_mma(const void* F, int64_t n_in, int c_in, const void* W, const void* bias, const int32_t* gmap,
               const int32_t* perm, int K, int64_t n_out, int c_out, const int32_t* ovf, int64_t ovf_cap,
               const int64_t* meta, void* out, int flags, const EpiParams& epi, int64_t* status, cudaStream_t stream) {
  const T* f = static_cast<const T*>(F);
  const T* w = static_cast<const T*>(W);
  const T* b = static_cast<const T*>(bias);
  T* o = static_cast<T*>(out);
  if (c_out <= 16)
    return launch_mma_tn<T, 16>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                                status, stream);
  if (c_out <= 32)
    return launch_mma_tn<T, 32>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                                status, stream);
  if (c_out <= 64)
    return launch_mma_tn<T, 64>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                                status, stream);
  return launch_mma_tn<T, 128>(f, n_in, c_in, w, b, gmap, perm, K, n_out, c_out, ovf, ovf_cap, meta, o, flags, epi,
                               status, stream);
}

// Dense scatter for SparseConvTensor.dense().

}  // namespace detail
}  // namespace tsc
