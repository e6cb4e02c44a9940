// Row order for the convolution kernels: output rows grouped by neighbour
// mask.
//
// The convolution kernels process tiles of consecutive rows of a row order
// and, per tile, only the kernel offsets that have a pair in it.  With rows
// in coordinate order a 256-row tile touches ~20 of 27 offsets and, at each
// of them, leaves many rows without a pair (gather slots that still cost a
// fetch or an MMA row).  Grouping rows by their neighbour mask (bit k set
// when gather_map[k][o] >= 0), masks in ascending order, makes the rows of a
// tile share their offsets: on the config-3 level-3 map the offsets per tile
// drop from 19.5 to 12.5 and the fetched rows from 1.47x to 1.01x the pairs.
// Results do not depend on the order (each output row is still accumulated
// over its offsets in k order), only the speed does.
//
// Three launches:
//   k_mask_insert   mask of each row; distinct masks counted in an
//                   open-addressing table (warp-aggregated atomics)
//   k_mask_order    one CTA: gathers the distinct masks, bitonic-sorts them
//                   in shared memory, prefix-sums their counts into each
//                   mask's first position
//   k_mask_scatter  each row claims the next position of its mask
// Rows of one mask land in arbitrary order (atomics); more than kMaxGroups
// distinct masks, or an insert that finds no slot within kMaxProbe probes,
// leave the identity order.
#include <cstdint>

#include "tsc_common.cuh"

namespace tsc {
namespace {

constexpr int kThreads = 256;
constexpr int kLog2Slots = 16;
constexpr uint32_t kSlots = 1u << kLog2Slots;
constexpr uint32_t kEmptyKey = 0xFFFFFFFFu;
constexpr int kMaxGroups = 16384;  // distinct masks sorted in one CTA
// Probes per insert or lookup.  A map with more distinct masks than the
// table holds (a config-5 LiDAR sample has ~232k) then gives up after a
// bounded walk and leaves the identity order; an unbounded walk over a full
// table cost 0.45 s on an 8M-row map.
constexpr uint32_t kMaxProbe = 128;
constexpr int kOrderThreads = 1024;
constexpr int kMaxK = 32;

struct RowSortWs {
  size_t masks, keys, counts, bases, cursors, flags, bytes;
};

RowSortWs rowsort_ws(int64_t n) {
  RowSortWs w;
  size_t off = 0;
  auto take = [&](size_t b) {
    const size_t o = off;
    off += (b + 255) / 256 * 256;
    return o;
  };
  w.masks = take(sizeof(uint32_t) * static_cast<size_t>(n < 1 ? 1 : n));
  w.keys = take(sizeof(uint32_t) * kSlots);
  w.counts = take(sizeof(uint32_t) * kSlots);
  w.bases = take(sizeof(uint32_t) * kSlots);
  w.cursors = take(sizeof(uint32_t) * kSlots);
  w.flags = take(sizeof(uint32_t) * 4);  // [0] table full, [1] use identity
  w.bytes = off;
  return w;
}

__device__ __forceinline__ uint32_t mask_slot(uint32_t m) { return (m * 0x9E3779B1u) >> (32 - kLog2Slots); }

__global__ void __launch_bounds__(kThreads)
k_mask_insert(const int32_t* __restrict__ gmap, int K, int64_t n, uint32_t* __restrict__ masks,
              uint32_t* __restrict__ keys, uint32_t* __restrict__ counts, uint32_t* __restrict__ flags) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool row = i < n;
  uint32_t m = 0;
  if (row) {
    for (int k = 0; k < K; ++k)
      if (__ldg(&gmap[static_cast<int64_t>(k) * n + i]) >= 0) m |= 1u << k;
    masks[i] = m;
  }
  uint32_t slot = mask_slot(m);
  bool placed = !row;
  for (uint32_t probe = 0; probe < kMaxProbe && !placed; ++probe) {
    uint32_t cur = keys[slot];
    if (cur == kEmptyKey) cur = atomicCAS(&keys[slot], kEmptyKey, m);
    if (cur == kEmptyKey || cur == m) {
      placed = true;
    } else {
      slot = (slot + 1u) & (kSlots - 1u);
    }
  }
  if (row && !placed) atomicOr(&flags[0], 1u);
  // one atomic per (warp, slot)
  const unsigned act = __ballot_sync(kFullMask, row && placed);
  if (row && placed) {
    const unsigned same = __match_any_sync(act, slot);
    if ((threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&counts[slot], static_cast<uint32_t>(__popc(same)));
  }
}

// One CTA.  Shared memory: keys and slots of up to kMaxGroups distinct masks.
__global__ void __launch_bounds__(kOrderThreads)
k_mask_order(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ counts, uint32_t* __restrict__ bases,
             uint32_t* __restrict__ flags) {
  extern __shared__ uint32_t sm[];
  uint32_t* s_key = sm;                 // [kMaxGroups]
  uint32_t* s_slot = sm + kMaxGroups;   // [kMaxGroups]
  __shared__ uint32_t s_n;
  __shared__ uint32_t s_part[kOrderThreads];
  const int tid = threadIdx.x;
  if (tid == 0) s_n = 0;
  __syncthreads();
  for (uint32_t s = tid; s < kSlots; s += kOrderThreads) {
    const uint32_t k = keys[s];
    if (k != kEmptyKey) {
      const uint32_t p = atomicAdd(&s_n, 1u);
      if (p < kMaxGroups) {
        s_key[p] = k;
        s_slot[p] = s;
      }
    }
  }
  __syncthreads();
  const uint32_t n = s_n;
  if (n > kMaxGroups || flags[0] != 0) {
    if (tid == 0) flags[1] = 1u;  // too many groups or a full table: identity order
    return;
  }
  uint32_t np2 = 1;
  while (np2 < n) np2 <<= 1;
  for (uint32_t p = n + tid; p < np2; p += kOrderThreads) {
    s_key[p] = kEmptyKey;
    s_slot[p] = 0;
  }
  __syncthreads();
  // bitonic sort of (key, slot) by key, ascending
  for (uint32_t size = 2; size <= np2; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t t = tid; t < np2 / 2; t += kOrderThreads) {
        const uint32_t lo = 2 * t - (t & (stride - 1));
        const uint32_t hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint32_t a = s_key[lo], b = s_key[hi];
        if ((a > b) == up) {
          s_key[lo] = b;
          s_key[hi] = a;
          const uint32_t ts = s_slot[lo];
          s_slot[lo] = s_slot[hi];
          s_slot[hi] = ts;
        }
      }
      __syncthreads();
    }
  }
  // exclusive prefix sum of the counts in key order -> first position of each mask
  constexpr int PER = kMaxGroups / kOrderThreads;
  uint32_t loc[PER];
  uint32_t sum = 0;
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const uint32_t p = tid * PER + q;
    loc[q] = p < n ? counts[s_slot[p]] : 0u;
    sum += loc[q];
  }
  s_part[tid] = sum;
  __syncthreads();
  for (int off = 1; off < kOrderThreads; off <<= 1) {
    const uint32_t v = tid >= off ? s_part[tid - off] : 0u;
    __syncthreads();
    s_part[tid] += v;
    __syncthreads();
  }
  uint32_t run = s_part[tid] - sum;
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const uint32_t p = tid * PER + q;
    if (p < n) bases[s_slot[p]] = run;
    run += loc[q];
  }
}

__global__ void __launch_bounds__(kThreads)
k_mask_scatter(const uint32_t* __restrict__ masks, int64_t n, const uint32_t* __restrict__ keys,
               const uint32_t* __restrict__ bases, uint32_t* __restrict__ cursors,
               const uint32_t* __restrict__ flags, int32_t* __restrict__ order, int64_t* __restrict__ status) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool row = i < n;
  if (flags[1] != 0) {
    if (row) order[i] = static_cast<int32_t>(i);
    return;
  }
  const uint32_t m = row ? masks[i] : 0u;
  uint32_t slot = mask_slot(m);
  bool found = !row;
  for (uint32_t probe = 0; probe < kMaxProbe && !found; ++probe) {
    const uint32_t k = __ldg(&keys[slot]);
    if (k == m) {
      found = true;
    } else if (k == kEmptyKey) {
      break;
    } else {
      slot = (slot + 1u) & (kSlots - 1u);
    }
  }
  const unsigned act = __ballot_sync(kFullMask, row && found);
  if (row && !found) {
    raise_status(status, TSC_STATUS_INTERNAL);  // every row's mask was inserted
    return;
  }
  if (!row) return;
  const unsigned same = __match_any_sync(act, slot);
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(same) - 1;
  uint32_t off = 0;
  if (lane == leader) off = atomicAdd(&cursors[slot], static_cast<uint32_t>(__popc(same)));
  off = __shfl_sync(same, off, leader);
  const uint32_t rank = __popc(same & ((1u << lane) - 1u));
  const int64_t pos = static_cast<int64_t>(bases[slot]) + off + rank;
  if (pos >= 0 && pos < n) {
    order[pos] = static_cast<int32_t>(i);
  } else {
    raise_status(status, TSC_STATUS_INTERNAL);
  }
}

}  // namespace
}  // namespace tsc

using namespace tsc;

extern "C" {

size_t tsc_row_order_workspace(int64_t n_out) { return rowsort_ws(n_out).bytes; }

int tsc_row_order(const int32_t* gather_map, int32_t k_vol, int64_t n_out, void* workspace, size_t workspace_bytes,
                  int32_t* row_order, int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  TSC_CHECK_ARG(k_vol > 0 && k_vol <= kMaxK, "row order needs 1 <= K <= %d (got %d)", kMaxK, k_vol);
  TSC_CHECK_ARG(n_out >= 0 && n_out <= 0x7fffffffLL, "n_out out of range");
  TSC_CHECK_ARG(status != nullptr, "status is NULL");
  if (n_out == 0) return TSC_OK;
  TSC_CHECK_ARG(gather_map != nullptr && row_order != nullptr, "NULL buffer");
  const RowSortWs w = rowsort_ws(n_out);
  if (workspace == nullptr || workspace_bytes < w.bytes || !aligned(workspace, 256)) {
    set_error("row-order workspace needs %zu bytes (256-byte aligned), got %zu", w.bytes, workspace_bytes);
    return TSC_ERR_WORKSPACE;
  }
  unsigned char* base = static_cast<unsigned char*>(workspace);
  auto* masks = reinterpret_cast<uint32_t*>(base + w.masks);
  auto* keys = reinterpret_cast<uint32_t*>(base + w.keys);
  auto* counts = reinterpret_cast<uint32_t*>(base + w.counts);
  auto* bases = reinterpret_cast<uint32_t*>(base + w.bases);
  auto* cursors = reinterpret_cast<uint32_t*>(base + w.cursors);
  auto* flags = reinterpret_cast<uint32_t*>(base + w.flags);
  TSC_CUDA(cudaMemsetAsync(keys, 0xFF, sizeof(uint32_t) * kSlots, stream));
  // counts, bases, cursors and flags are contiguous
  TSC_CUDA(cudaMemsetAsync(counts, 0, w.bytes - w.counts, stream));
  const unsigned grid = static_cast<unsigned>(ceil_div(n_out, kThreads));
  k_mask_insert<<<grid, kThreads, 0, stream>>>(gather_map, k_vol, n_out, masks, keys, counts, flags);
  TSC_LAUNCH_CHECK("k_mask_insert");
  constexpr int smem = 2 * kMaxGroups * sizeof(uint32_t);
  static unsigned long long configured = 0;
  int dev = 0;
  TSC_CUDA(cudaGetDevice(&dev));
  if (!(configured & (1ull << (dev & 63)))) {
    TSC_CUDA(cudaFuncSetAttribute(k_mask_order, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured |= 1ull << (dev & 63);
  }
  k_mask_order<<<1, kOrderThreads, smem, stream>>>(keys, counts, bases, flags);
  TSC_LAUNCH_CHECK("k_mask_order");
  k_mask_scatter<<<grid, kThreads, 0, stream>>>(masks, n_out, keys, bases, cursors, flags, row_order, status);
  TSC_LAUNCH_CHECK("k_mask_scatter");
  return TSC_OK;
}

}  // extern "C"
