// Per-plane input sub-halos for the tensor-memory halo convolution
// (conv_tmh.cuh).
//
// A tile is TSC_HALO_TILE_ROWS (256) consecutive output rows of a k-major
// gather map; a plane is one kz of the kernel (offsets
// k = plane*kH*kW .. +kH*kW-1).  The sub-halo of (tile, plane) is the list of
// distinct input rows that the plane's pairs of the tile read, in ascending
// row order.  For every pair the halo map holds the input row's position in
// that list, so the convolution fetches each distinct input row of a
// (tile, plane) once and builds the A operands of the plane's offsets from it.
//
// One CTA per (tile, plane), one thread per tile row:
//   1. the smallest and largest input row the (tile, plane) reads (each
//      thread keeps its row's entries of the plane in registers);
//   2. when they lie within kWindow rows of each other (spatially ordered
//      maps: the outputs of strided maps and the submanifold maps built on
//      them span a few hundred rows per plane), one bit per row of the span
//      in shared memory, set by every pair; a prefix popcount over the
//      span's words ranks the distinct rows in ascending order.  The first
//      `capacity` ranks form the list, padded to a multiple of 4 with copies
//      of its last row (TMA gathers 4 rows);
//   3. every pair's entry becomes its rank, kOutsideHalo when the rank is
//      >= capacity or the rows span more than the window (the convolution
//      reads those rows from global memory), or kNoPair.
// Also written: plane_kmask[tile][plane], bit k set when offset k of the
// plane has a pair in the tile.
#include <cstdint>

#include "tsc_common.cuh"

namespace tsc {
namespace {

constexpr int kTileRows = TSC_HALO_TILE_ROWS;
constexpr int kThreads = kTileRows;
constexpr int kWindowWords = 2048;            // bits for 65536 consecutive input rows
constexpr int kWindow = kWindowWords * 32;
constexpr int kWordsPerThread = kWindowWords / kThreads;  // 8
static_assert(kWordsPerThread * kThreads == kWindowWords, "window words per thread");
constexpr int kMaxK = 32;                     // plane_kmask is one 32-bit word
constexpr int kNoPair = -1;
constexpr int kOutsideHalo = -2;

__global__ void __launch_bounds__(kThreads) k_tile_plane_halo(const int32_t* __restrict__ gmap, int K, int kpg,
                                                              int planes, int64_t n_in, int64_t n_out, int cap,
                                                              int32_t* __restrict__ halo_rows,
                                                              int32_t* __restrict__ halo_count,
                                                              uint32_t* __restrict__ plane_kmask,
                                                              int16_t* __restrict__ hmap,
                                                              int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t bits[kWindowWords];
  __shared__ uint32_t word_pre[kWindowWords];
  __shared__ uint32_t warp_sums[32];
  __shared__ int s_lo, s_hi;
  __shared__ unsigned s_kmask;
  const int tid = threadIdx.x;
  const int64_t tile = blockIdx.x;
  const int plane = blockIdx.y;
  const int k0 = plane * kpg;
  const int64_t o = tile * kTileRows + tid;
  const bool row_ok = o < n_out;
  const int64_t hp = tile * planes + plane;  // (tile, plane) index

  if (tid == 0) {
    s_lo = 0x7fffffff;
    s_hi = -1;
    s_kmask = 0u;
  }
  __syncthreads();
  // the plane's gather entries of this row, read once
  int v[kMaxK];
  int lo = 0x7fffffff, hi = -1;
  unsigned km = 0u;
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    v[j] = -1;
    if (j < kpg) {
      int e = row_ok ? __ldg(&gmap[static_cast<int64_t>(k0 + j) * n_out + o]) : -1;
      if (e >= n_in) {
        raise_status(status, TSC_STATUS_KEY_RANGE);
        e = -1;
      }
      if (e >= 0) {
        lo = min(lo, e);
        hi = max(hi, e);
        km |= 1u << (k0 + j);
      }
      v[j] = e < 0 ? -1 : e;
    }
  }
  // warp-level reduction first, then one shared atomic per warp
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    lo = min(lo, __shfl_xor_sync(kFullMask, lo, d));
    hi = max(hi, __shfl_xor_sync(kFullMask, hi, d));
    km |= __shfl_xor_sync(kFullMask, km, d);
  }
  if ((tid & 31) == 0) {
    atomicMin(&s_lo, lo);
    atomicMax(&s_hi, hi);
    atomicOr(&s_kmask, km);
  }
  __syncthreads();
  const int base = s_lo;
  const bool any = s_hi >= 0;
  const bool windowed = any && static_cast<int64_t>(s_hi) - base < kWindow;
  if (tid == 0) plane_kmask[hp] = s_kmask;
  int32_t* list = halo_rows + hp * static_cast<int64_t>(cap);

  if (!windowed) {
    // no pair, or rows too far apart to rank in one window: empty list, and
    // every pair reads its row from global memory
    if (tid == 0) halo_count[hp] = 0;
    if (!row_ok) return;
#pragma unroll
    for (int j = 0; j < kMaxK; ++j)
      if (j < kpg)
        hmap[static_cast<int64_t>(k0 + j) * n_out + o] = static_cast<int16_t>(v[j] >= 0 ? kOutsideHalo : kNoPair);
    return;
  }

  // only the words the rows span: [base, s_hi]
  const int nwords = ((s_hi - base) >> 5) + 1;  // 1 .. kWindowWords
  for (int i = tid; i < nwords; i += kThreads) bits[i] = 0u;
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    if (j < kpg && v[j] >= 0) {
      const int b = v[j] - base;
      atomicOr(&bits[b >> 5], 1u << (b & 31));
    }
  }
  __syncthreads();
  // ranks: exclusive prefix of the popcounts; thread tid owns words
  // tid*wpt .. tid*wpt+wpt-1 of the span
  const int wpt = (nwords + kThreads - 1) / kThreads;  // 1 .. kWordsPerThread
  const int w0 = tid * wpt;
  uint32_t cnt = 0;
  for (int i = 0; i < wpt; ++i)
    if (w0 + i < nwords) cnt += __popc(bits[w0 + i]);
  uint32_t total = 0;
  uint32_t run = block_exclusive_scan(cnt, warp_sums, &total);
  for (int i = 0; i < wpt; ++i) {
    const int w = w0 + i;
    if (w >= nwords) break;
    word_pre[w] = run;
    uint32_t m = bits[w];
    while (m) {
      const int bit = __ffs(m) - 1;
      m &= m - 1;
      if (run < static_cast<uint32_t>(cap)) list[run] = base + w * 32 + bit;
      ++run;
    }
  }
  const int hc = total < static_cast<uint32_t>(cap) ? static_cast<int>(total) : cap;
  __syncthreads();
  // pad the list to a multiple of 4 rows with its last row (the thread that
  // ranked that row knows it: recompute from the window instead of reading
  // another thread's global write)
  if (tid == 0) halo_count[hp] = hc;
  if (tid < 3 && hc > 0) {
    const int i = hc + tid;
    if (i < ((hc + 3) & ~3)) {
      // find the row of rank hc-1
      const uint32_t want = static_cast<uint32_t>(hc - 1);
      int lo_w = 0, hi_w = nwords - 1;
      while (lo_w < hi_w) {  // last word whose prefix is <= want
        const int mid = (lo_w + hi_w + 1) >> 1;
        if (word_pre[mid] <= want) lo_w = mid; else hi_w = mid - 1;
      }
      uint32_t m = bits[lo_w];
      uint32_t r = word_pre[lo_w];
      int bit = 0;
      while (m) {
        bit = __ffs(m) - 1;
        m &= m - 1;
        if (r == want) break;
        ++r;
      }
      list[i] = base + lo_w * 32 + bit;
    }
  }
  if (!row_ok) return;
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    if (j >= kpg) break;
    int hv = kNoPair;
    if (v[j] >= 0) {
      const int b = v[j] - base;
      const uint32_t rank = word_pre[b >> 5] + __popc(bits[b >> 5] & ((1u << (b & 31)) - 1u));
      hv = rank < static_cast<uint32_t>(cap) ? static_cast<int>(rank) : kOutsideHalo;
    }
    hmap[static_cast<int64_t>(k0 + j) * n_out + o] = static_cast<int16_t>(hv);
  }
}

}  // namespace
}  // namespace tsc

using namespace tsc;

extern "C" {

int tsc_tile_halo(const int32_t* gather_map, int32_t k_vol, int32_t planes, int64_t n_in, int64_t n_out,
                  int32_t capacity, int32_t* halo_rows, int32_t* halo_count, uint32_t* plane_kmask,
                  int16_t* halo_map, int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  TSC_CHECK_ARG(k_vol >= 1 && k_vol <= kMaxK, "halo maps take 1..%d kernel offsets, got %d", kMaxK, k_vol);
  TSC_CHECK_ARG(planes >= 1 && k_vol % planes == 0, "%d planes do not divide %d kernel offsets", planes, k_vol);
  TSC_CHECK_ARG(capacity >= 4 && capacity % 4 == 0 && capacity <= 32767,
                "halo capacity must be a multiple of 4 in [4, 32767], got %d", capacity);
  TSC_CHECK_ARG(n_in >= 0 && n_in <= 0x7fffffffLL && n_out >= 0 && n_out <= 0x7fffffffLL, "row counts out of range");
  TSC_CHECK_ARG(status != nullptr, "status is NULL");
  if (n_out == 0) return TSC_OK;
  TSC_CHECK_ARG(gather_map != nullptr && halo_rows != nullptr && halo_count != nullptr && plane_kmask != nullptr &&
                    halo_map != nullptr,
                "NULL buffer");
  TSC_CHECK_ARG(aligned(halo_rows, 16), "halo_rows must be 16-byte aligned");
  const int64_t tiles = ceil_div(n_out, kTileRows);
  TSC_CHECK_ARG(tiles <= 0x7fffffffLL, "too many tiles");
  TSC_LAUNCH_PDL("k_tile_plane_halo", k_tile_plane_halo, dim3(static_cast<unsigned>(tiles), planes), dim3(kThreads), 0,
                 stream, gather_map, k_vol, k_vol / planes, planes, n_in, n_out, capacity, halo_rows, halo_count,
                 plane_kmask, halo_map, status);
  return TSC_OK;
}

}  // extern "C"
