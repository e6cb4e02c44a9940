// Launch entry points of the tensor-core convolution kernels, one per kernel
// family and element type (each defined in its own conv_launch_*.cu so the
// heavy template instantiations compile in parallel).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "trispconv_b200.h"
#include "tsc_common.cuh"

namespace tsc {

struct ConvArgs {
  const void* features;
  int64_t n_in;
  int c_in;
  const void* weight;  // KRSC (C_out, K, C_in)
  const void* bias;
  const int32_t* gather_map;
  const int32_t* row_order;
  int k_vol;
  int64_t n_out;
  int c_out;
  const int32_t* overflow;
  int64_t overflow_cap;
  const int64_t* meta;
  void* out;
  int flags;
  int64_t* status;
  uint32_t* tile_counter;  // persistent kernel: dynamic tile hand-out (NULL = round robin)
  cudaStream_t stream;
  // per-plane input sub-halos (tsc_tile_halo); NULL = none
  const int32_t* halo_rows = nullptr;
  const int32_t* halo_count = nullptr;
  const uint32_t* plane_kmask = nullptr;
  const int16_t* halo_map = nullptr;
  int halo_planes = 0;
  int halo_capacity = 0;
  // store epilogue (folded BatchNorm scale/shift, activation); set by conv_forward
  EpiParams epi = {nullptr, nullptr, TSC_ACT_NONE, 0.f};
};

// Largest kernel volumes the tensor-core kernels take (gather-map slice in
// shared memory; one 32-bit active-offset mask for the persistent kernel).
constexpr int kMmaKMax = 64;
constexpr int kPersistentKMax = 27;

// mma.sync path: 16-bit types, KRSC weights, C_in % 8 == 0 (or C_in % 4 == 0
// and C_in <= 16), C_out % 8 == 0.
inline bool mma_eligible(int dtype, int w_krsc, int c_in, int c_out, int K) {
  if (dtype != TSC_F16 && dtype != TSC_BF16) return false;
  if (!w_krsc || K > kMmaKMax || c_out % 8 != 0) return false;
  if (c_in % 8 == 0) return true;
  return c_in % 4 == 0 && c_in <= 16;
}

// tcgen05 paths: 16-bit types, KRSC weights, C_in % 8 == 0, C_out % 8 == 0.
inline bool tc_eligible(int dtype, int w_krsc, int c_in, int c_out, int K) {
  if (dtype != TSC_F16 && dtype != TSC_BF16) return false;
  return w_krsc && K <= kMmaKMax && c_in % 8 == 0 && c_out % 8 == 0;
}

// persistent tcgen05 path (TMA gathers): additionally C_in % 64 == 0,
// C_out % 32 == 0 and K <= 27, so that channel chunks (64) and column tiles
// (32..256) divide the tensors exactly and no TMA box reaches outside them.
// Measured on the config-3 maps, 64-channel rows are where the TMA gather
// beats the mma.sync kernel (32-channel layers run faster on mma.sync).
// 32-byte feature rows (C_in = 16) and N = 16 tiles are not built at all:
// that configuration made an illegal memory access on a 280k-row map
// although every coordinate it issued was checked in range.
inline bool tcp_eligible(int dtype, int w_krsc, int c_in, int c_out, int K) {
  return tc_eligible(dtype, w_krsc, c_in, c_out, K) && c_in % 64 == 0 && c_out % 32 == 0 && K <= kPersistentKMax;
}

// halo kernel (persistent tcgen05, per-plane sub-halos staged once in shared
// memory, A operand in tensor memory): 3x3x3 kernels (3 planes of 9
// offsets), exactly 64 input channels and 64 or 128 output channels, maps
// without duplicate-coordinate overflow pairs.
inline bool tmh_eligible(int dtype, int w_krsc, int c_in, int c_out, int K) {
  return tcp_eligible(dtype, w_krsc, c_in, c_out, K) && c_in == 64 && (c_out == 64 || c_out == 128) && K == 27;
}

// Rows per (tile, plane) sub-halo the halo kernel holds for c_out output
// channels (0 when it does not take c_out).
int tmh_capacity(int c_out);

// Register-gather kernel (conv_rg.cu): mma.sync with the A fragments loaded
// straight from the gathered rows into registers and all weights resident in
// shared memory.  16-bit types, KRSC weights, K <= 64 where the weights fit
// in shared memory, C_in in {4, 8} with C_out in {16, 32, 64}, or C_in in
// {16, 32} with C_out in {16, 32}.  Measured on the config-3 layers, the
// shared-memory mma.sync kernel is faster for 32 -> 64 (131 against 144-300
// us over the shapes tried), where the 110 KB of resident weights leave room
// for too few warps per SM.
size_t rg_smem_bytes(int c_in, int c_out, int K);
bool rg_fits(int c_in, int c_out, int K);
inline bool rg_eligible(int dtype, int w_krsc, int c_in, int c_out, int K) {
  if (dtype != TSC_F16 && dtype != TSC_BF16) return false;
  if (!w_krsc || K < 1 || K > 64) return false;
  if (c_in != 4 && c_in != 8 && c_in != 16 && c_in != 32) return false;
  if (c_out != 16 && c_out != 32 && (c_out != 64 || c_in > 8)) return false;
  return rg_fits(c_in, c_out, K);
}

int launch_rg_f16(const ConvArgs& a);
int launch_rg_bf16(const ConvArgs& a);
int launch_mma_f16(const ConvArgs& a);
int launch_mma_bf16(const ConvArgs& a);
int launch_tc_f16(const ConvArgs& a);
int launch_tc_bf16(const ConvArgs& a);
int launch_tcp_f16(const ConvArgs& a);
int launch_tcp_bf16(const ConvArgs& a);
int launch_tmh_f16(const ConvArgs& a);
int launch_tmh_bf16(const ConvArgs& a);

}  // namespace tsc
