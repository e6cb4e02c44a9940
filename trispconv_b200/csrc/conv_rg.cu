// Launchers of the register-gather convolution kernel (conv_rg.cuh).

#include "conv_launch.h"
#include "conv_rg.cuh"

namespace tsc {
namespace {

constexpr size_t kMaxDynSmem = 227 * 1024;

template <typename T, int CIN, int TN, int MT, int G, int NT, int WN, int MINB>
int launch_cfg(const ConvArgs& a) {
  auto kern = rg::k_conv_rg<T, CIN, TN, MT, G, NT, WN, MINB>;
  const int K = a.k_vol;
  const size_t smem = rg::Smem<CIN, TN>::bytes(K);
  if (smem > kMaxDynSmem) {
    set_error("register-gather conv needs %zu bytes of shared memory", smem);
    return TSC_ERR_UNSUPPORTED;
  }
  static unsigned long long configured = 0;      // one bit per device
  static int ctas_per_sm[rg::KMAX + 1][64] = {};  // [K][device]: 0 = not computed yet
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (!(configured & (1ull << dev))) {
    TSC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kMaxDynSmem)));
    configured |= 1ull << dev;
  }
  int& occ = ctas_per_sm[K][dev];
  if (occ == 0) {
    TSC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, NT, smem));
    if (occ < 1) occ = 1;
  }
  constexpr int kGroups = NT / 32 / WN;  // row blocks per CTA at once
  const int64_t blocks = ceil_div(ceil_div(a.n_out, 16 * MT), kGroups);
  const int64_t cap = static_cast<int64_t>(sm_count()) * occ;
  const dim3 grid(static_cast<unsigned>(blocks < cap ? blocks : cap));
  TSC_LAUNCH_PDL("k_conv_rg", kern, grid, dim3(NT), smem, a.stream, static_cast<const T*>(a.features),
                 static_cast<int>(a.n_in), static_cast<const T*>(a.weight), static_cast<const T*>(a.bias),
                 a.gather_map, a.row_order, K, static_cast<int>(a.n_out), a.overflow, a.overflow_cap, a.meta,
                 static_cast<T*>(a.out), a.epi, a.status);
  return TSC_OK;
}

// Tile shape per channel pair: rows per warp (16*MT = 16), G = 4 units
// loaded per step, 256 threads, one warp per row block, and the register
// bound of 4 CTAs per SM (C_in <= 8) or 3 (C_in 16 and 32).  Chosen by a
// sweep on the config-3 layers against other shapes (32 rows per warp, 2 or
// 8 units per step, two warps per row block, 2-4 CTAs per SM).
template <typename T, int CIN, int TN>
int launch_shape(const ConvArgs& a) {
  if constexpr (CIN <= 8) {
    return launch_cfg<T, CIN, TN, 1, 4, 256, 1, 4>(a);
  } else {
    return launch_cfg<T, CIN, TN, 1, 4, 256, 1, 3>(a);
  }
}

template <typename T, int CIN>
int launch_cin(const ConvArgs& a) {
  switch (a.c_out) {
    case 16: return launch_shape<T, CIN, 16>(a);
    case 32: return launch_shape<T, CIN, 32>(a);
    default:
      if constexpr (CIN <= 8) return launch_shape<T, CIN, 64>(a);
      set_error("register-gather conv does not take %d -> %d", CIN, a.c_out);
      return TSC_ERR_UNSUPPORTED;
  }
}

template <typename T>
int launch_rg(const ConvArgs& a) {
  switch (a.c_in) {
    case 4: return launch_cin<T, 4>(a);
    case 8: return launch_cin<T, 8>(a);
    case 16: return launch_cin<T, 16>(a);
    default: return launch_cin<T, 32>(a);
  }
}

}  // namespace

size_t rg_smem_bytes(int c_in, int c_out, int K) {
  return static_cast<size_t>((K * c_in + 15) / 16) * (c_out / 16) * 32 * 16;
}

bool rg_fits(int c_in, int c_out, int K) { return rg_smem_bytes(c_in, c_out, K) <= kMaxDynSmem; }

int launch_rg_f16(const ConvArgs& a) { return launch_rg<__half>(a); }
int launch_rg_bf16(const ConvArgs& a) { return launch_rg<__nv_bfloat16>(a); }

}  // namespace tsc
