// Per-tile input halos for the halo convolution kernel (conv_tch.cuh).
//
// A tile is 256 consecutive output rows of a k-major gather map.  Its halo
// is the list of distinct input rows that any (offset, row) pair of the tile
// reads.  For every pair the halo map holds the input row's position in that
// list, so the convolution kernel can fetch each distinct input row of a tile
// once into shared memory and build all of the tile's A operands from there.
//
// One CTA per tile:
//   1. insert the tile's valid gather entries into an open-addressing table
//      in shared memory (8192 slots > 256 rows x 27 offsets, so an insert
//      always finds a slot);
//   2. number the occupied slots (block-wide prefix sum of per-thread
//      counts); the first `capacity` numbers form the halo list, padded to a
//      multiple of 4 rows with copies of its last row (TMA gathers 4 rows);
//   3. rewrite every entry of the tile as its halo position, kOutsideHalo
//      when the position is >= capacity (the kernel reads those rows from
//      global memory), or kNoPair.
// Halo positions depend on the order of the atomic inserts; the
// convolution's results do not (each output row still accumulates its pairs
// in offset order from the same input values).
#include <cstdint>

#include "tsc_common.cuh"

namespace tsc {
namespace {

constexpr int kTileRows = TSC_HALO_TILE_ROWS;
constexpr int kLog2Slots = 13;
constexpr int kSlots = 1 << kLog2Slots;
constexpr int kMaxK = 27;  // kTileRows * kMaxK < kSlots
static_assert(kTileRows * kMaxK < kSlots, "halo table must never fill");
constexpr int kThreads = kTileRows;
constexpr int kSlotsPerThread = kSlots / kThreads;  // 32
static_assert(kSlotsPerThread == 32, "slot ownership assumes 32 slots per thread");
constexpr int kNoPair = -1;
constexpr int kOutsideHalo = -2;

__device__ __forceinline__ uint32_t slot_of(int32_t key) {
  return (static_cast<uint32_t>(key) * 2654435761u) >> (32 - kLog2Slots);
}

__device__ __forceinline__ void table_insert(int32_t* keys, int32_t key) {
  uint32_t h = slot_of(key);
  for (int p = 0; p < kSlots; ++p) {
    const int32_t prev = atomicCAS(&keys[h], 0, key);
    if (prev == 0 || prev == key) return;
    h = (h + 1) & (kSlots - 1);
  }
}

__device__ __forceinline__ int table_find(const int32_t* keys, const int32_t* ids, int32_t key) {
  uint32_t h = slot_of(key);
  for (int p = 0; p < kSlots; ++p) {
    const int32_t k = keys[h];
    if (k == key) return ids[h];
    if (k == 0) return -1;
    h = (h + 1) & (kSlots - 1);
  }
  return -1;
}

__global__ void __launch_bounds__(kThreads) k_tile_halo(const int32_t* __restrict__ gmap, int K, int64_t n_in,
                                                        int64_t n_out, int cap, int32_t* __restrict__ halo_rows,
                                                        int32_t* __restrict__ halo_count,
                                                        int16_t* __restrict__ hmap, int64_t* __restrict__ status) {
  extern __shared__ int32_t sh[];
  int32_t* keys = sh;           // input row + 1; 0 = empty
  int32_t* ids = sh + kSlots;   // halo position of the slot's row
  __shared__ int32_t s_warp[kThreads / 32];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t tile = blockIdx.x;
  const int64_t o = tile * kTileRows + tid;
  const bool row_ok = o < n_out;

  for (int i = tid; i < kSlots; i += kThreads) keys[i] = 0;
  __syncthreads();
  for (int k = 0; k < K; ++k) {
    int v = row_ok ? __ldg(&gmap[static_cast<int64_t>(k) * n_out + o]) : -1;
    if (v >= n_in) {
      raise_status(status, TSC_STATUS_KEY_RANGE);
      v = -1;
    }
    if (v >= 0) table_insert(keys, v + 1);
  }
  __syncthreads();

  // thread tid owns slots 32*tid .. 32*tid+31, visited in a lane-rotated
  // order so that a warp's reads fall into distinct banks
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < kSlotsPerThread; ++i) cnt += keys[tid * kSlotsPerThread + ((i + lane) & 31)] != 0;
  int incl = cnt;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(kFullMask, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  int before = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    before += w < warp ? s_warp[w] : 0;
    total += s_warp[w];
  }
  int id = before + incl - cnt;
  int32_t* list = halo_rows + tile * static_cast<int64_t>(cap);
#pragma unroll
  for (int i = 0; i < kSlotsPerThread; ++i) {
    const int s = tid * kSlotsPerThread + ((i + lane) & 31);
    const int32_t key = keys[s];
    if (key != 0) {
      ids[s] = id;
      if (id < cap) list[id] = key - 1;
      ++id;
    }
  }
  __syncthreads();
  const int hc = total < cap ? total : cap;
  if (tid < 3 && hc > 0) {
    const int i = hc + tid;
    if (i < ((hc + 3) & ~3)) list[i] = list[hc - 1];
  }
  if (tid == 0) halo_count[tile] = hc;

  for (int k = 0; k < K; ++k) {
    if (!row_ok) break;
    const int v = __ldg(&gmap[static_cast<int64_t>(k) * n_out + o]);
    int hv = kNoPair;
    if (v >= 0 && v < n_in) {
      const int p = table_find(keys, ids, v + 1);
      hv = p < 0 ? kNoPair : (p < cap ? p : kOutsideHalo);
      if (p < 0) raise_status(status, TSC_STATUS_INTERNAL);
    }
    hmap[static_cast<int64_t>(k) * n_out + o] = static_cast<int16_t>(hv);
  }
}

constexpr int kSmemBytes = 2 * kSlots * static_cast<int>(sizeof(int32_t));

}  // namespace
}  // namespace tsc

using namespace tsc;

extern "C" {

int tsc_tile_halo(const int32_t* gather_map, int32_t k_vol, int64_t n_in, int64_t n_out, int32_t capacity,
                  int32_t* halo_rows, int32_t* halo_count, int16_t* halo_map, int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  TSC_CHECK_ARG(k_vol >= 1 && k_vol <= kMaxK, "halo maps take 1..%d kernel offsets, got %d", kMaxK, k_vol);
  TSC_CHECK_ARG(capacity >= 4 && capacity % 4 == 0 && capacity <= 32767,
                "halo capacity must be a multiple of 4 in [4, 32767], got %d", capacity);
  TSC_CHECK_ARG(n_in >= 0 && n_in <= 0x7fffffffLL && n_out >= 0 && n_out <= 0x7fffffffLL, "row counts out of range");
  TSC_CHECK_ARG(status != nullptr, "status is NULL");
  if (n_out == 0) return TSC_OK;
  TSC_CHECK_ARG(gather_map != nullptr && halo_rows != nullptr && halo_count != nullptr && halo_map != nullptr,
                "NULL buffer");
  TSC_CHECK_ARG(aligned(halo_rows, 16), "halo_rows must be 16-byte aligned");
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    TSC_CUDA(cudaFuncSetAttribute(k_tile_halo, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    configured |= 1ull << (dev & 63);
  }
  const int64_t tiles = ceil_div(n_out, kTileRows);
  k_tile_halo<<<static_cast<unsigned>(tiles), kThreads, kSmemBytes, stream>>>(
      gather_map, k_vol, n_in, n_out, capacity, halo_rows, halo_count, halo_map, status);
  TSC_LAUNCH_CHECK("k_tile_halo");
  return TSC_OK;
}

}  // extern "C"
