// Kernel-map (indice-pair) generation on the GPU.
//
// Reference behaviour being replaced (mrpulford/trispconv):
//   trispconv/pytorch/indices.py:54-64    dense B*D*H*W int64 lookup table
//   trispconv/pytorch/indices.py:67-140   submanifold pairs, offset loop kz,ky,kx
//   trispconv/pytorch/indices.py:143-259  strided pairs, torch.unique(sorted=True)
//   trispconv/pytorch/modules.py:175-213  inverse pairs (participation + swap)
//
// Design (B200): the dense table becomes an open-addressing hash of packed
// 64-bit entries (cell key << 32 | row) built with atomicCAS; the strided
// output set becomes a 1-bit-per-cell occupancy bitmap whose prefix popcount
// gives every output cell its rank in sorted key order.  All maps are k-major
// int32 arrays so that per-offset reads and writes are coalesced.
#include <cstdint>
#include <mutex>

#include "tsc_common.cuh"

namespace tsc {
namespace {

constexpr int kThreads = 256;
constexpr int kItems = 8;                          // words / flags per thread in scans
constexpr int kTile = kThreads * kItems;           // 2048 per block
constexpr int kScanBlockThreads = 1024;
constexpr uint64_t kMaxCells = 0xFFFFFFFEull;      // 32-bit keys must stay below the empty sentinel
constexpr uint64_t kMaxCells64 = 1ull << 62;         // 64-bit keys (grids above kMaxCells)

struct GeoDev {
  int B, D, H, W;
  int oD, oH, oW;
  int kD, kH, kW;
  int sz, sy, sx;
  int pz, py, px;
  int dz, dy, dx;
};

GeoDev to_dev(const tsc_geometry& g) {
  GeoDev d;
  d.B = g.batch;
  d.D = g.in_shape[0]; d.H = g.in_shape[1]; d.W = g.in_shape[2];
  d.oD = g.out_shape[0]; d.oH = g.out_shape[1]; d.oW = g.out_shape[2];
  d.kD = g.ksize[0]; d.kH = g.ksize[1]; d.kW = g.ksize[2];
  d.sz = g.stride[0]; d.sy = g.stride[1]; d.sx = g.stride[2];
  d.pz = g.padding[0]; d.py = g.padding[1]; d.px = g.padding[2];
  d.dz = g.dilation[0]; d.dy = g.dilation[1]; d.dx = g.dilation[2];
  return d;
}

int log2_ceil(uint64_t v) {
  int l = 0;
  while ((1ull << l) < v) ++l;
  return l;
}

// Capacity of the submanifold hash: load factor <= 1/2.
// Smallest SubM hash: 2^ceil(log2 2n) slots (load factor <= 1/2).
int subm_log2cap(int64_t n) {
  int l = log2_ceil(static_cast<uint64_t>(n < 1 ? 1 : n) * 2);
  return l < 8 ? 8 : l;
}

// The workspace entry point takes up to 4x that (load factor <= 1/8) when the
// caller's workspace holds it: on the config-3 input map a lookup that misses
// then walks 1.14 slots on average instead of 2.03 (1.10 instead of 1.55 for a
// hit), one dependent L2 round trip each.
constexpr int kSubmSpread = 2;
int subm_ws_log2cap(int64_t n, size_t workspace_bytes, size_t slot_bytes) {
  const int lo = subm_log2cap(n);
  for (int l = lo + kSubmSpread; l > lo; --l)
    if ((slot_bytes << l) <= workspace_bytes) return l;
  return lo;
}

__device__ __forceinline__ bool in_grid(const int4& c, int B, int D, int H, int W) {
  return static_cast<unsigned>(c.x) < static_cast<unsigned>(B) &&
         static_cast<unsigned>(c.y) < static_cast<unsigned>(D) &&
         static_cast<unsigned>(c.z) < static_cast<unsigned>(H) &&
         static_cast<unsigned>(c.w) < static_cast<unsigned>(W);
}

// Linear cell key b*DHW + z*HW + y*W + x (indices.py:45-51).  The host checks
// B*D*H*W <= kMaxCells, so every partial product fits in 32 bits.
__device__ __forceinline__ uint32_t cell_key(unsigned b, unsigned z, unsigned y, unsigned x,
                                             unsigned D, unsigned H, unsigned W) {
  return ((b * D + z) * H + y) * W + x;
}

// The same key in KeyT: uint32_t for grids of at most kMaxCells cells,
// uint64_t above (the reference's int64 key, grids up to kMaxCells64).
template <typename KeyT>
__device__ __forceinline__ KeyT cell_key_t(unsigned b, unsigned z, unsigned y, unsigned x, unsigned D, unsigned H,
                                           unsigned W) {
  return ((static_cast<KeyT>(b) * D + z) * H + y) * W + x;
}

// Slot of a 64-bit cell key: Fibonacci hashing of key >> 3, keeping the low 3
// bits (the same neighbourhood-preserving layout as hash_slot).
__device__ __forceinline__ uint32_t hash_slot64(unsigned long long key, int log2cap) {
  const uint32_t hi = static_cast<uint32_t>(((key >> 3) * 0x9E3779B97F4A7C15ull) >> (64 - (log2cap - 3)));
  return (hi << 3) | static_cast<uint32_t>(key & 7u);
}

// ---------------------------------------------------------------------------
// Submanifold: hash build + per-offset query
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads)
k_hash_build(const int4* __restrict__ idx, int64_t n, int B, int D, int H, int W,
             unsigned long long* __restrict__ table, int log2cap, int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = idx[i];
  if (!in_grid(c, B, D, H, W)) {
    raise_status(status, TSC_STATUS_KEY_RANGE);
    return;
  }
  const uint32_t key = cell_key(c.x, c.y, c.z, c.w, D, H, W);
  const unsigned long long entry = (static_cast<unsigned long long>(key) << 32) |
                                   static_cast<uint32_t>(i);
  const uint32_t mask = (1u << log2cap) - 1u;
  uint32_t slot = hash_slot(key, log2cap);
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    unsigned long long cur = table[slot];
    if (cur == kEmptySlot) {
      cur = atomicCAS(&table[slot], kEmptySlot, entry);
      if (cur == kEmptySlot) return;
    }
    if (static_cast<uint32_t>(cur >> 32) == key) {
      // Duplicate coordinate: the highest row wins, like the reference's
      // in-order `table[encoded] = arange(N)` (indices.py:63).
      atomicMax(&table[slot], entry);
      return;
    }
    slot = (slot + 1u) & mask;
  }
  raise_status(status, TSC_STATUS_HASH_FULL);
}

__device__ __forceinline__ int hash_lookup(const unsigned long long* __restrict__ table,
                                           int log2cap, uint32_t key) {
  const uint32_t mask = (1u << log2cap) - 1u;
  uint32_t slot = hash_slot(key, log2cap);
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    const unsigned long long e = __ldg(&table[slot]);
    if (e == kEmptySlot) return -1;
    if (static_cast<uint32_t>(e >> 32) == key) return static_cast<int>(static_cast<uint32_t>(e));
    slot = (slot + 1u) & mask;
  }
  return -1;
}

// Grids above kMaxCells: keys and rows in two arrays of 2^log2cap slots
// (keys kEmptySlot and rows -1 when empty).  atomicCAS claims a key slot;
// atomicMax on its row keeps the largest row of a duplicated coordinate,
// the reference's last-write-wins `table[key] = arange(N)` (indices.py:63).
__global__ void __launch_bounds__(kThreads)
k_hash_build64(const int4* __restrict__ idx, int64_t n, int B, int D, int H, int W,
               unsigned long long* __restrict__ keys, int32_t* __restrict__ rows, int log2cap,
               int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = idx[i];
  if (!in_grid(c, B, D, H, W)) {
    raise_status(status, TSC_STATUS_KEY_RANGE);
    return;
  }
  const unsigned long long key = cell_key_t<unsigned long long>(c.x, c.y, c.z, c.w, D, H, W);
  const uint32_t mask = (1u << log2cap) - 1u;
  uint32_t slot = hash_slot64(key, log2cap);
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    unsigned long long cur = keys[slot];
    if (cur == kEmptySlot) cur = atomicCAS(&keys[slot], kEmptySlot, key);
    if (cur == kEmptySlot || cur == key) {
      atomicMax(&rows[slot], static_cast<int32_t>(i));
      return;
    }
    slot = (slot + 1u) & mask;
  }
  raise_status(status, TSC_STATUS_HASH_FULL);
}

// Lookups of a cell (b, z, y, x) of the (D, H, W) grid: in the 32-bit-key
// open-addressing hash, the 64-bit-key hash, or a direct-address table (one
// int32 row per cell, -1 = empty).
struct HashLookup {
  const unsigned long long* table;
  int log2cap;
  unsigned D, H, W;
  __device__ __forceinline__ int operator()(unsigned b, unsigned z, unsigned y, unsigned x) const {
    return hash_lookup(table, log2cap, cell_key(b, z, y, x, D, H, W));
  }
};

struct HashLookup64 {
  const unsigned long long* keys;
  const int32_t* rows;
  int log2cap;
  unsigned D, H, W;
  __device__ __forceinline__ int operator()(unsigned b, unsigned z, unsigned y, unsigned x) const {
    const unsigned long long key = cell_key_t<unsigned long long>(b, z, y, x, D, H, W);
    const uint32_t mask = (1u << log2cap) - 1u;
    uint32_t slot = hash_slot64(key, log2cap);
    for (uint32_t probe = 0; probe <= mask; ++probe) {
      const unsigned long long e = __ldg(&keys[slot]);
      if (e == kEmptySlot) return -1;
      if (e == key) return __ldg(&rows[slot]);
      slot = (slot + 1u) & mask;
    }
    return -1;
  }
};

// The output set of a strided map as its own lookup: a cell's row is the
// rank of its bit in the occupancy bitmap (the order the strided map emitted
// its output coordinates in), -1 when the bit is clear.
template <typename KeyT>
struct RankLookup {
  const uint32_t* bitmap;
  const uint32_t* word_prefix;
  unsigned D, H, W;
  __device__ __forceinline__ int operator()(unsigned b, unsigned z, unsigned y, unsigned x) const {
    const KeyT lin = cell_key_t<KeyT>(b, z, y, x, D, H, W);
    const KeyT w = lin >> 5;
    const uint32_t word = __ldg(&bitmap[w]);
    const uint32_t bit = 1u << static_cast<unsigned>(lin & 31u);
    if (!(word & bit)) return -1;
    return static_cast<int>(__ldg(&word_prefix[w]) + __popc(word & (bit - 1u)));
  }
};

struct DenseLookup {
  const int32_t* table;
  unsigned D, H, W;
  __device__ __forceinline__ int operator()(unsigned b, unsigned z, unsigned y, unsigned x) const {
    return __ldg(&table[cell_key(b, z, y, x, D, H, W)]);
  }
};

// One thread per (offset k = blockIdx.y, row i).  Writes gather_map[k][i] and
// accumulates pair_num[k].  Offsets follow indices.py:96-98:
// (k_dim - K_dim//2) * dilation.
template <class Lookup>
__global__ void __launch_bounds__(kThreads)
k_subm_query(const int4* __restrict__ idx, int64_t n, GeoDev g, Lookup look,
             int32_t* __restrict__ gmap, unsigned long long* __restrict__ meta) {
  pdl_wait();
  pdl_trigger();
  const int k = blockIdx.y;
  const KOffset ko = split_k(k, g.kH, g.kW);
  const int offz = (ko.kz - g.kD / 2) * g.dz;
  const int offy = (ko.ky - g.kH / 2) * g.dy;
  const int offx = (ko.kx - g.kW / 2) * g.dx;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int found = -1;
  if (i < n) {
    const int4 c = __ldg(&idx[i]);
    const int nz = c.y + offz, ny = c.z + offy, nx = c.w + offx;
    if (static_cast<unsigned>(c.x) < static_cast<unsigned>(g.B) &&
        static_cast<unsigned>(nz) < static_cast<unsigned>(g.D) &&
        static_cast<unsigned>(ny) < static_cast<unsigned>(g.H) &&
        static_cast<unsigned>(nx) < static_cast<unsigned>(g.W)) {
      found = look(c.x, nz, ny, nx);
    }
    gmap[static_cast<int64_t>(k) * n + i] = found;
  }
  const int cnt = __syncthreads_count(found >= 0);
  if (threadIdx.x == 0 && cnt) atomicAdd(&meta[TSC_META_COUNTS + k], static_cast<unsigned long long>(cnt));
}

// One thread per row i for all K offsets (K <= kRowQueryKMax): the row's
// coordinates are read once, the x-neighbour lookups of one (dz, dy) hit the
// same hash cache line (the hash keeps the low 3 key bits), and the writes
// gather_map[k][i] stay coalesced across the warp.  pair_num[k] is reduced
// per warp (ballot) and per block (shared memory) before one atomic per
// offset and block.
constexpr int kRowQueryKMax = 128;

template <class Lookup>
__global__ void __launch_bounds__(kThreads)
k_subm_query_rows(const int4* __restrict__ idx, int64_t n, GeoDev g, Lookup look,
                  int32_t* __restrict__ gmap, unsigned long long* __restrict__ meta) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned s_cnt[kRowQueryKMax];
  const int K = g.kD * g.kH * g.kW;
  for (int t = threadIdx.x; t < K; t += blockDim.x) s_cnt[t] = 0u;
  __syncthreads();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool row = i < n;
  int4 c = make_int4(-1, 0, 0, 0);
  if (row) c = __ldg(&idx[i]);
  const bool b_ok = row && static_cast<unsigned>(c.x) < static_cast<unsigned>(g.B);
  const int lane = threadIdx.x & 31;
  int k = 0;
  for (int kz = 0; kz < g.kD; ++kz) {
    const int nz = c.y + (kz - g.kD / 2) * g.dz;
    for (int ky = 0; ky < g.kH; ++ky) {
      const int ny = c.z + (ky - g.kH / 2) * g.dy;
      const bool zy_ok = b_ok && static_cast<unsigned>(nz) < static_cast<unsigned>(g.D) &&
                         static_cast<unsigned>(ny) < static_cast<unsigned>(g.H);
      for (int kx = 0; kx < g.kW; ++kx, ++k) {
        const int nx = c.w + (kx - g.kW / 2) * g.dx;
        int found = -1;
        if (zy_ok && static_cast<unsigned>(nx) < static_cast<unsigned>(g.W))
          found = look(c.x, nz, ny, nx);
        if (row) gmap[static_cast<int64_t>(k) * n + i] = found;
        const unsigned hits = __ballot_sync(kFullMask, found >= 0);
        if (lane == 0 && hits) atomicAdd(&s_cnt[k], static_cast<unsigned>(__popc(hits)));
      }
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < K; t += blockDim.x)
    if (s_cnt[t]) atomicAdd(&meta[TSC_META_COUNTS + t], static_cast<unsigned long long>(s_cnt[t]));
}

// Builds gather_map and pair_num from a filled hash or direct-address table
// (the workspace, allocation-free and dense entry points).
template <class Lookup>
int launch_subm_query(const int4* idx, int64_t n, const GeoDev& g, Lookup look, int32_t* gmap, int64_t* meta,
                      cudaStream_t stream) {
  const int K = g.kD * g.kH * g.kW;
  const unsigned grid = static_cast<unsigned>(ceil_div(n, kThreads));
  if (K <= kRowQueryKMax) {
    TSC_LAUNCH_PDL("k_subm_query_rows", k_subm_query_rows<Lookup>, dim3(grid), dim3(kThreads), 0, stream, idx, n, g,
                   look, gmap, reinterpret_cast<unsigned long long*>(meta));
  } else {
    TSC_LAUNCH_PDL("k_subm_query", k_subm_query<Lookup>, dim3(grid, K), dim3(kThreads), 0, stream, idx, n, g, look,
                   gmap, reinterpret_cast<unsigned long long*>(meta));
  }
  return TSC_OK;
}

int launch_subm_query(const int4* idx, int64_t n, const GeoDev& g, const unsigned long long* table, int log2cap,
                      int32_t* gmap, int64_t* meta, cudaStream_t stream) {
  return launch_subm_query(idx, n, g,
                           HashLookup{table, log2cap, static_cast<unsigned>(g.D), static_cast<unsigned>(g.H),
                                      static_cast<unsigned>(g.W)},
                           gmap, meta, stream);
}

// Direct-address table: the largest row of each cell (the reference's
// last-write-wins `table[key] = arange(N)`, indices.py:63) over cells that
// hold -1; k_dense_clear puts -1 back into the same cells afterwards.
__global__ void __launch_bounds__(kThreads)
k_dense_build(const int4* __restrict__ idx, int64_t n, int B, int D, int H, int W, int32_t* __restrict__ table,
              int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = idx[i];
  if (!in_grid(c, B, D, H, W)) {
    raise_status(status, TSC_STATUS_KEY_RANGE);
    return;
  }
  atomicMax(&table[cell_key(c.x, c.y, c.z, c.w, D, H, W)], static_cast<int32_t>(i));
}

__global__ void __launch_bounds__(kThreads)
k_dense_clear(const int4* __restrict__ idx, int64_t n, int B, int D, int H, int W, int32_t* __restrict__ table) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = idx[i];
  if (in_grid(c, B, D, H, W)) table[cell_key(c.x, c.y, c.z, c.w, D, H, W)] = -1;
}

// ---------------------------------------------------------------------------
// Strided: occupancy bitmap over the output grid
// ---------------------------------------------------------------------------

// o = c / s when c >= 0 is a multiple of s and c / s < lim (the candidate
// output position of one dimension); strides 1 and 2 avoid the division.
__device__ __forceinline__ bool exact_div(int c, int s, int lim, int& o) {
  if (c < 0) return false;
  if (s == 1) {
    o = c;
  } else if (s == 2) {
    if (c & 1) return false;
    o = c >> 1;
  } else {
    if (c % s) return false;
    o = c / s;
  }
  return o < lim;
}

// Per input row, walks the K offsets in reference order (indices.py:177-187):
// c = i + p - k*d is a valid output position iff c >= 0, c % s == 0 and
// c / s < out (for c >= 0 C and Python division agree).
template <typename KeyT>
__global__ void __launch_bounds__(kThreads)
k_strided_mark(const int4* __restrict__ idx, int64_t n, GeoDev g, uint32_t* __restrict__ bitmap,
               unsigned long long* __restrict__ meta, int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ unsigned int s_cnt[];  // K pair counters + 1 participation counter
  const int K = g.kD * g.kH * g.kW;
  for (int t = threadIdx.x; t <= K; t += blockDim.x) s_cnt[t] = 0u;
  __syncthreads();

  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  bool active = i < n;
  int4 c = make_int4(0, 0, 0, 0);
  if (active) {
    c = __ldg(&idx[i]);
    if (!in_grid(c, g.B, g.D, g.H, g.W)) {
      raise_status(status, TSC_STATUS_KEY_RANGE);
      active = false;
    }
  }
  const int lane = threadIdx.x & 31;
  bool any = false;
  int k = 0;
  for (int kz = 0; kz < g.kD; ++kz) {
    int oz = 0;
    const bool vz = exact_div(c.y + g.pz - kz * g.dz, g.sz, g.oD, oz);
    for (int ky = 0; ky < g.kH; ++ky) {
      int oy = 0;
      const bool vy = vz && exact_div(c.z + g.py - ky * g.dy, g.sy, g.oH, oy);
      for (int kx = 0; kx < g.kW; ++kx, ++k) {
        int ox = 0;
        const bool v = active && vy && exact_div(c.w + g.px - kx * g.dx, g.sx, g.oW, ox);
        const unsigned b = __ballot_sync(kFullMask, v);
        if (v) {
          // one fire-and-forget OR per candidate: combining the lanes of a
          // word first (__match_any_sync) saved only ~10 % of the atomics on
          // the config-3 maps and cost more instructions than it saved
          const KeyT lin = cell_key_t<KeyT>(c.x, oz, oy, ox, g.oD, g.oH, g.oW);
          atomicOr(&bitmap[lin >> 5], 1u << static_cast<unsigned>(lin & 31u));
          any = true;
        }
        if (lane == 0 && b) atomicAdd(&s_cnt[k], static_cast<unsigned>(__popc(b)));
      }
    }
  }
  const unsigned b = __ballot_sync(kFullMask, any);
  if (lane == 0 && b) atomicAdd(&s_cnt[K], static_cast<unsigned>(__popc(b)));
  __syncthreads();
  for (int t = threadIdx.x; t < K; t += blockDim.x)
    if (s_cnt[t]) atomicAdd(&meta[TSC_META_COUNTS + t], static_cast<unsigned long long>(s_cnt[t]));
  if (threadIdx.x == 0 && s_cnt[K])
    atomicAdd(&meta[TSC_META_N_PART], static_cast<unsigned long long>(s_cnt[K]));
}

// Popcount of each 2048-word tile of the (zero-padded) bitmap.
__global__ void __launch_bounds__(kThreads)
k_bitmap_tile_count(const uint4* __restrict__ bitmap, uint32_t* __restrict__ block_sums) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t ws[32];
  const size_t q = (static_cast<size_t>(blockIdx.x) * kTile + threadIdx.x * kItems) / 4;
  const uint4 a = bitmap[q], b = bitmap[q + 1];
  const uint32_t s = __popc(a.x) + __popc(a.y) + __popc(a.z) + __popc(a.w) + __popc(b.x) +
                     __popc(b.y) + __popc(b.z) + __popc(b.w);
  uint32_t total;
  block_exclusive_scan(s, ws, &total);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// Single-block exclusive scan of per-tile sums, in place; sums[nblocks] gets the
// total.  Optionally publishes the total and a status snapshot into meta.
template <typename U>
__global__ void __launch_bounds__(kScanBlockThreads)
k_scan_tile_sums(U* __restrict__ sums, int64_t nblocks, unsigned long long* __restrict__ meta,
                 int meta_slot, const int64_t* __restrict__ status,
                 unsigned long long* __restrict__ host_meta = nullptr, int meta_len = 0) {
  pdl_wait();
  pdl_trigger();
  __shared__ U ws[32];
  U carry = 0;
  for (int64_t base = 0; base < nblocks; base += blockDim.x) {
    const int64_t t = base + threadIdx.x;
    const U v = t < nblocks ? sums[t] : U(0);
    U tot;
    U ex;
    if constexpr (sizeof(U) == 8) {
      ex = block_exclusive_scan64(v, reinterpret_cast<unsigned long long*>(ws),
                                  reinterpret_cast<unsigned long long*>(&tot));
    } else {
      ex = block_exclusive_scan(v, reinterpret_cast<uint32_t*>(ws), reinterpret_cast<uint32_t*>(&tot));
    }
    if (t < nblocks) sums[t] = carry + ex;
    carry += tot;
  }
  if (threadIdx.x == 0) {
    sums[nblocks] = carry;
    if (meta != nullptr) {
      meta[meta_slot] = static_cast<unsigned long long>(carry);
      if (status != nullptr) meta[TSC_META_STATUS] = static_cast<unsigned long long>(*status);
    }
  }
  if (host_meta != nullptr && meta != nullptr) {
    // the whole meta block (earlier kernels wrote the rest) into mapped host
    // memory, visible to the host once this kernel has completed
    __syncthreads();
    for (int i = threadIdx.x; i < meta_len; i += blockDim.x) host_meta[i] = meta[i];
    __threadfence_system();
  }
}

// Exclusive prefix popcount of every bitmap word: the rank of a set bit is
// word_prefix[w] + popcount of the lower bits of its word, and rank order ==
// ascending cell key == the reference's unique(sorted=True) order
// (indices.py:219-229).
__global__ void __launch_bounds__(kThreads)
k_bitmap_prefix(const uint4* __restrict__ bitmap, const uint32_t* __restrict__ tile_off,
                uint32_t* __restrict__ word_prefix) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t ws[32];
  const size_t w0 = static_cast<size_t>(blockIdx.x) * kTile + threadIdx.x * kItems;
  const uint4 a = bitmap[w0 / 4], b = bitmap[w0 / 4 + 1];
  const uint32_t words[kItems] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j) s += __popc(words[j]);
  uint32_t total;
  uint32_t ex = block_exclusive_scan(s, ws, &total) + tile_off[blockIdx.x];
  uint32_t pre[kItems];
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    pre[j] = ex;
    ex += __popc(words[j]);
  }
  uint4* wp = reinterpret_cast<uint4*>(word_prefix + w0);
  wp[0] = make_uint4(pre[0], pre[1], pre[2], pre[3]);
  wp[1] = make_uint4(pre[4], pre[5], pre[6], pre[7]);
}

// One thread per bitmap word: decode its set bits to coordinates at their
// rank (a grid of one thread per word keeps sparse and dense grids alike
// fully parallel).
template <typename KeyT>
__global__ void __launch_bounds__(kThreads)
k_bitmap_coords(const uint32_t* __restrict__ bitmap, const uint32_t* __restrict__ word_prefix,
                int64_t nwords, GeoDev g, int4* __restrict__ out_idx, int64_t n_out) {
  pdl_wait();
  pdl_trigger();
  const int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (w >= nwords) return;
  uint32_t wv = __ldg(&bitmap[w]);
  if (wv == 0) return;
  uint32_t r = __ldg(&word_prefix[w]);
  const KeyT oW = g.oW, oH = g.oH, oD = g.oD;
  {
    while (wv) {
      const int bit = __ffs(wv) - 1;
      wv &= wv - 1u;
      const KeyT lin = static_cast<KeyT>(w) * 32 + static_cast<KeyT>(bit);
      const KeyT x = lin % oW;
      KeyT t = lin / oW;
      const KeyT y = t % oH;
      t /= oH;
      const KeyT z = t % oD;
      const KeyT bb = t / oD;
      if (r < n_out)
        out_idx[r] = make_int4(static_cast<int>(bb), static_cast<int>(z), static_cast<int>(y),
                               static_cast<int>(x));
      ++r;
    }
  }
}

__device__ __forceinline__ void push_overflow(int32_t* overflow, int64_t cap,
                                              unsigned long long* meta, int64_t* status, int k,
                                              int o, int i) {
  const unsigned long long slot = atomicAdd(&meta[TSC_META_N_OVERFLOW], 1ull);
  if (static_cast<int64_t>(slot) < cap) {
    overflow[3 * slot + 0] = k;
    overflow[3 * slot + 1] = o;
    overflow[3 * slot + 2] = i;
  } else {
    raise_status(status, TSC_STATUS_OVERFLOW_FULL);
  }
}

// Per input row and offset: rank of the output cell, written to the
// input-stationary scatter map and (first writer wins) to the
// output-stationary gather map.  A second input row for the same (k, o) can
// only come from duplicate input coordinates; it goes to the overflow list.
template <typename KeyT>
__global__ void __launch_bounds__(kThreads)
k_strided_pairs(const int4* __restrict__ idx, int64_t n, GeoDev g,
                const uint32_t* __restrict__ bitmap, const uint32_t* __restrict__ word_prefix,
                int64_t n_out, int32_t* __restrict__ gmap, int32_t* __restrict__ smap,
                int32_t* __restrict__ overflow, int64_t ovf_cap,
                unsigned long long* __restrict__ meta, int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int4 c = __ldg(&idx[i]);
  const bool active = in_grid(c, g.B, g.D, g.H, g.W);
  int k = 0;
  for (int kz = 0; kz < g.kD; ++kz) {
    int oz = 0;
    const bool vz = active && exact_div(c.y + g.pz - kz * g.dz, g.sz, g.oD, oz);
    for (int ky = 0; ky < g.kH; ++ky) {
      int oy = 0;
      const bool vy = vz && exact_div(c.z + g.py - ky * g.dy, g.sy, g.oH, oy);
      for (int kx = 0; kx < g.kW; ++kx, ++k) {
        int ox = 0;
        const bool v = vy && exact_div(c.w + g.px - kx * g.dx, g.sx, g.oW, ox);
        int o = -1;
        if (v) {
          const KeyT lin = cell_key_t<KeyT>(c.x, oz, oy, ox, g.oD, g.oH, g.oW);
          const KeyT w = lin >> 5;
          o = static_cast<int>(__ldg(&word_prefix[w]) +
                               __popc(__ldg(&bitmap[w]) & ((1u << static_cast<unsigned>(lin & 31u)) - 1u)));
          if (o >= n_out) {
            raise_status(status, TSC_STATUS_KEY_RANGE);
            smap[static_cast<int64_t>(k) * n + i] = -1;
            continue;
          }
          const int prev = atomicCAS(&gmap[static_cast<int64_t>(k) * n_out + o], -1,
                                     static_cast<int>(i));
          if (prev != -1) push_overflow(overflow, ovf_cap, meta, status, k, o, static_cast<int>(i));
        }
        smap[static_cast<int64_t>(k) * n + i] = o;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Row compaction (inverse convs): flags -> exclusive prefix
// ---------------------------------------------------------------------------

// Participation of input row i in a k-major map: any map[k][i] >= 0.
__device__ __forceinline__ bool row_participates(const int32_t* __restrict__ map, int K, int64_t n,
                                                 int64_t i) {
  for (int k = 0; k < K; ++k)
    if (__ldg(&map[static_cast<int64_t>(k) * n + i]) >= 0) return true;
  return false;
}

__global__ void __launch_bounds__(kThreads)
k_part_tile_count(const int32_t* __restrict__ map, int K, int64_t n, uint32_t* __restrict__ block_sums) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t ws[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile + threadIdx.x * kItems;
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t i = base + j;
    if (i < n && row_participates(map, K, n, i)) ++s;
  }
  uint32_t total;
  block_exclusive_scan(s, ws, &total);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// For participating rows (ascending): compact[i] = r, out_idx[r] = in_idx[i],
// inv_gather[k][r] = smap[k][i].
__global__ void __launch_bounds__(kThreads)
k_inverse_strided_emit(const int4* __restrict__ in_idx, const int32_t* __restrict__ smap, int K,
                       int64_t n, const uint32_t* __restrict__ tile_off, int64_t n_part,
                       int4* __restrict__ out_idx, int32_t* __restrict__ inv_gather,
                       int32_t* __restrict__ compact) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t ws[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile + threadIdx.x * kItems;
  bool flag[kItems];
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t i = base + j;
    flag[j] = i < n && row_participates(smap, K, n, i);
    s += flag[j] ? 1u : 0u;
  }
  uint32_t total;
  uint32_t r = block_exclusive_scan(s, ws, &total) + tile_off[blockIdx.x];
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t i = base + j;
    if (i >= n) break;
    if (compact != nullptr) compact[i] = flag[j] ? static_cast<int32_t>(r) : -1;
    if (flag[j] && r < n_part) {
      out_idx[r] = in_idx[i];
      for (int k = 0; k < K; ++k)
        inv_gather[static_cast<int64_t>(k) * n_part + r] = smap[static_cast<int64_t>(k) * n + i];
      ++r;
    }
  }
}

__global__ void __launch_bounds__(kThreads)
k_iota(int32_t* __restrict__ out, int64_t n) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = static_cast<int32_t>(i);
}

// Inverse of a submanifold map: flag every row j read by some pair.
__global__ void __launch_bounds__(kThreads)
k_flag_targets(const int32_t* __restrict__ gmap, int64_t total, int64_t n, int32_t* __restrict__ flags) {
  pdl_wait();
  pdl_trigger();
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= total) return;
  const int j = gmap[e];
  if (j >= 0 && j < n) flags[j] = 1;
}

__global__ void __launch_bounds__(kThreads)
k_flag_tile_count(const int32_t* __restrict__ flags, int64_t n, uint32_t* __restrict__ block_sums) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t ws[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile + threadIdx.x * kItems;
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t i = base + j;
    if (i < n && flags[i] != 0) ++s;
  }
  uint32_t total;
  block_exclusive_scan(s, ws, &total);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// flags (0/1) -> compact ids (r or -1), in place.
__global__ void __launch_bounds__(kThreads)
k_flag_compact(int32_t* __restrict__ flags, int64_t n, const uint32_t* __restrict__ tile_off) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t ws[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile + threadIdx.x * kItems;
  int32_t f[kItems];
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t i = base + j;
    f[j] = (i < n) ? flags[i] : 0;
    s += f[j] != 0 ? 1u : 0u;
  }
  uint32_t total;
  uint32_t r = block_exclusive_scan(s, ws, &total) + tile_off[blockIdx.x];
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t i = base + j;
    if (i < n) {
      flags[i] = f[j] != 0 ? static_cast<int32_t>(r) : -1;
      if (f[j] != 0) ++r;
    }
  }
}

__global__ void __launch_bounds__(kThreads)
k_gather_rows(const int4* __restrict__ in_idx, const int32_t* __restrict__ compact, int64_t n,
              int64_t n_part, int4* __restrict__ out_idx) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = compact[i];
  if (r >= 0 && r < n_part) out_idx[r] = in_idx[i];
}

// inv_gather[k][compact[j]] = i for gather_map[k][i] = j.
__global__ void __launch_bounds__(kThreads)
k_transpose_map(const int32_t* __restrict__ gmap, int K, int64_t n, const int32_t* __restrict__ compact,
                int64_t n_part, int32_t* __restrict__ inv_gather, int32_t* __restrict__ overflow,
                int64_t ovf_cap, unsigned long long* __restrict__ meta, int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= static_cast<int64_t>(K) * n) return;
  const int j = gmap[e];
  if (j < 0 || j >= n) return;
  const int k = static_cast<int>(e / n);
  const int i = static_cast<int>(e - static_cast<int64_t>(k) * n);
  const int r = compact[j];
  if (r < 0 || r >= n_part) return;
  const int prev = atomicCAS(&inv_gather[static_cast<int64_t>(k) * n_part + r], -1, i);
  if (prev != -1) push_overflow(overflow, ovf_cap, meta, status, k, r, i);
}

// ---------------------------------------------------------------------------
// Pair-list materialisation (k-major scan over a [K][n] map)
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads)
k_map_tile_count(const int32_t* __restrict__ map, int64_t total, unsigned long long* __restrict__ block_sums) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t ws[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile + threadIdx.x * kItems;
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t e = base + j;
    if (e < total && map[e] >= 0) ++s;
  }
  uint32_t t;
  block_exclusive_scan(s, ws, &t);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = t;
}

__global__ void __launch_bounds__(kThreads)
k_map_emit_pairs(const int32_t* __restrict__ map, int64_t total, int64_t n, int mode,
                 const int32_t* __restrict__ remap, const unsigned long long* __restrict__ tile_off,
                 int64_t* __restrict__ pairs_in, int64_t* __restrict__ pairs_out, int64_t capacity) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t ws[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile + threadIdx.x * kItems;
  int32_t v[kItems];
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t e = base + j;
    v[j] = e < total ? map[e] : -1;
    s += v[j] >= 0 ? 1u : 0u;
  }
  uint32_t t;
  unsigned long long pos = block_exclusive_scan(s, ws, &t) + tile_off[blockIdx.x];
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    if (v[j] < 0) continue;
    if (static_cast<int64_t>(pos) >= capacity) break;
    const int64_t e = base + j;
    const int64_t k = e / n;
    const int64_t idx = e - k * n;
    if (mode == 0) {
      pairs_in[pos] = v[j];
      pairs_out[pos] = idx;
    } else {
      pairs_in[pos] = idx;
      pairs_out[pos] = remap != nullptr ? static_cast<int64_t>(remap[v[j]]) : static_cast<int64_t>(v[j]);
    }
    ++pos;
  }
}

__global__ void __launch_bounds__(kThreads)
k_pairs_to_gather(const int64_t* __restrict__ pin, const int64_t* __restrict__ pout, int64_t count,
                  int k, int64_t n_out, int32_t* __restrict__ gmap, int32_t* __restrict__ overflow,
                  int64_t ovf_cap, unsigned long long* __restrict__ meta, int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= count) return;
  const int64_t o = pout[p];
  const int64_t i = pin[p];
  if (o < 0 || o >= n_out || i < 0 || i > 0x7fffffffLL) {
    raise_status(status, TSC_STATUS_KEY_RANGE);
    return;
  }
  const int prev = atomicCAS(&gmap[static_cast<int64_t>(k) * n_out + o], -1, static_cast<int>(i));
  if (prev != -1) push_overflow(overflow, ovf_cap, meta, status, k, static_cast<int>(o), static_cast<int>(i));
}

// ---------------------------------------------------------------------------
// Host-side validation helpers
// ---------------------------------------------------------------------------

int check_shape3(const int32_t* s, const char* what) {
  for (int d = 0; d < 3; ++d) {
    if (s[d] <= 0) {
      set_error("%s[%d] = %d must be positive", what, d, s[d]);
      return TSC_ERR_INVALID_ARG;
    }
  }
  return TSC_OK;
}

int check_geometry(const tsc_geometry* geo, bool strided) {
  TSC_CHECK_ARG(geo != nullptr, "geometry is NULL");
  TSC_CHECK_ARG(geo->batch > 0, "batch_size must be positive, got %d", geo->batch);
  int rc;
  if ((rc = check_shape3(geo->in_shape, "spatial_shape")) != TSC_OK) return rc;
  if ((rc = check_shape3(geo->ksize, "kernel_size")) != TSC_OK) return rc;
  if ((rc = check_shape3(geo->dilation, "dilation")) != TSC_OK) return rc;
  if (strided) {
    if ((rc = check_shape3(geo->out_shape, "output spatial_shape")) != TSC_OK) return rc;
    if ((rc = check_shape3(geo->stride, "stride")) != TSC_OK) return rc;
    for (int d = 0; d < 3; ++d)
      TSC_CHECK_ARG(geo->padding[d] >= 0, "padding[%d] = %d must be >= 0", d, geo->padding[d]);
  }
  const int64_t K = static_cast<int64_t>(geo->ksize[0]) * geo->ksize[1] * geo->ksize[2];
  TSC_CHECK_ARG(K <= 4096, "kernel volume %lld exceeds 4096", static_cast<long long>(K));
  return TSC_OK;
}

// batch*D*H*W, saturated to UINT64_MAX (every such grid is refused).
uint64_t cells_of(int32_t batch, const int32_t* s) {
  const uint64_t f[4] = {static_cast<uint64_t>(batch < 0 ? 0 : batch), static_cast<uint64_t>(s[0] < 0 ? 0 : s[0]),
                         static_cast<uint64_t>(s[1] < 0 ? 0 : s[1]), static_cast<uint64_t>(s[2] < 0 ? 0 : s[2])};
  uint64_t c = 1;
  for (uint64_t v : f) {
    if (v != 0 && c > UINT64_MAX / v) return UINT64_MAX;
    c *= v;
  }
  return c;
}

struct StridedWs {
  uint64_t nbits;
  int64_t nwords_pad;
  int64_t nblocks;
  size_t off_prefix, off_sums, bytes;
};

StridedWs strided_ws(const tsc_geometry& g) {
  StridedWs w;
  w.nbits = cells_of(g.batch, g.out_shape);
  const int64_t nwords = static_cast<int64_t>((w.nbits + 31) / 32);
  w.nblocks = ceil_div(nwords < 1 ? 1 : nwords, kTile);
  w.nwords_pad = w.nblocks * kTile;
  w.off_prefix = align_up(static_cast<size_t>(w.nwords_pad) * 4, 256);
  w.off_sums = w.off_prefix + align_up(static_cast<size_t>(w.nwords_pad) * 4, 256);
  w.bytes = w.off_sums + align_up(static_cast<size_t>(w.nblocks + 1) * 4, 256);
  return w;
}

size_t rows_scan_bytes(int64_t n) {
  const int64_t nblocks = ceil_div(n < 1 ? 1 : n, kTile);
  return align_up(static_cast<size_t>(nblocks + 1) * 8, 256);
}

}  // namespace
}  // namespace tsc

using namespace tsc;

extern "C" {

size_t tsc_subm_kmap_workspace(int64_t n) {
  // 8-byte key|row slots for grids of at most 2^32-2 cells; above, 8-byte
  // keys plus 4-byte rows per slot (the larger of the two)
  return static_cast<size_t>(12) << (subm_log2cap(n) + kSubmSpread);
}

int tsc_subm_kmap(const int32_t* indices, int64_t n, const tsc_geometry* geo, void* workspace,
                  size_t workspace_bytes, int32_t* gather_map, int64_t* meta, int64_t* status,
                  void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = check_geometry(geo, false);
  if (rc != TSC_OK) return rc;
  TSC_CHECK_ARG(n >= 0 && n <= 0x7fffffffLL, "number of voxels %lld out of range", (long long)n);
  TSC_CHECK_ARG(meta != nullptr && status != nullptr, "meta/status must not be NULL");
  const uint64_t cells = cells_of(geo->batch, geo->in_shape);
  if (cells > kMaxCells64) {
    set_error("grid batch*D*H*W = %llu exceeds the 64-bit key limit 2^62", (unsigned long long)cells);
    return TSC_ERR_GRID_TOO_LARGE;
  }
  const bool wide = cells > kMaxCells;  // 64-bit keys
  const int K = geo->ksize[0] * geo->ksize[1] * geo->ksize[2];
  const int64_t meta_words = 2 * static_cast<int64_t>(TSC_META_COUNTS + K);
  if (n == 0) return fill_words(meta, 0u, meta_words, nullptr, 0u, 0, stream);
  TSC_CHECK_ARG(indices != nullptr && aligned(indices, 16), "indices must be 16-byte aligned");
  TSC_CHECK_ARG(gather_map != nullptr && aligned(gather_map, 4), "gather_map must not be NULL");
  const size_t slot_bytes = wide ? 12 : 8;
  const size_t need = slot_bytes << subm_log2cap(n);
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16)) {
    set_error("subm workspace needs %zu bytes (16-byte aligned), got %zu", need, workspace_bytes);
    return TSC_ERR_WORKSPACE;
  }
  const int log2cap = subm_ws_log2cap(n, workspace_bytes, slot_bytes);
  if (wide) {
    // keys (all ones = empty) then rows (-1), one fill with meta = 0
    auto* keys = static_cast<unsigned long long*>(workspace);
    auto* rows = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + (static_cast<size_t>(8) << log2cap));
    rc = fill_words(meta, 0u, meta_words, keys, 0xFFFFFFFFu, static_cast<int64_t>(3) << log2cap, stream);
    if (rc != TSC_OK) return rc;
    const GeoDev g = to_dev(*geo);
    const int4* idx = reinterpret_cast<const int4*>(indices);
    const unsigned grid = static_cast<unsigned>(ceil_div(n, kThreads));
    TSC_LAUNCH_PDL("k_hash_build64", k_hash_build64, dim3(grid), dim3(kThreads), 0, stream, idx, n, g.B, g.D, g.H,
                   g.W, keys, rows, log2cap, status);
    return launch_subm_query(idx, n, g,
                             HashLookup64{keys, rows, log2cap, static_cast<unsigned>(g.D), static_cast<unsigned>(g.H),
                                          static_cast<unsigned>(g.W)},
                             gather_map, meta, stream);
  }
  auto* table = static_cast<unsigned long long*>(workspace);
  // meta = 0 and every table slot empty (all ones), one launch
  rc = fill_words(meta, 0u, meta_words, table, 0xFFFFFFFFu, static_cast<int64_t>(2) << log2cap, stream);
  if (rc != TSC_OK) return rc;
  const GeoDev g = to_dev(*geo);
  const int4* idx = reinterpret_cast<const int4*>(indices);
  const unsigned grid = static_cast<unsigned>(ceil_div(n, kThreads));
  TSC_LAUNCH_PDL("k_hash_build", k_hash_build, dim3(grid), dim3(kThreads), 0, stream, idx, n, g.B, g.D, g.H, g.W,
                 table, log2cap, status);
  return launch_subm_query(idx, n, g, table, log2cap, gather_map, meta, stream);
}

int tsc_subm_kmap_dense(const int32_t* indices, int64_t n, const tsc_geometry* geo, int32_t* table,
                        int64_t table_cells, int32_t* gather_map, int64_t* meta, int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = check_geometry(geo, false);
  if (rc != TSC_OK) return rc;
  TSC_CHECK_ARG(n >= 0 && n <= 0x7fffffffLL, "number of voxels %lld out of range", (long long)n);
  TSC_CHECK_ARG(meta != nullptr && status != nullptr, "meta/status must not be NULL");
  const uint64_t cells = cells_of(geo->batch, geo->in_shape);
  if (cells > kMaxCells) {
    set_error("grid batch*D*H*W = %llu exceeds the packed-key limit 2^32-2", (unsigned long long)cells);
    return TSC_ERR_GRID_TOO_LARGE;
  }
  TSC_CHECK_ARG(table != nullptr && table_cells >= 0 && static_cast<uint64_t>(table_cells) >= cells,
                "dense table holds %lld cells, the grid has %llu", (long long)table_cells,
                (unsigned long long)cells);
  const int K = geo->ksize[0] * geo->ksize[1] * geo->ksize[2];
  rc = fill_words(meta, 0u, 2 * static_cast<int64_t>(TSC_META_COUNTS + K), nullptr, 0u, 0, stream);
  if (rc != TSC_OK || n == 0) return rc;
  TSC_CHECK_ARG(indices != nullptr && aligned(indices, 16), "indices must be 16-byte aligned");
  TSC_CHECK_ARG(gather_map != nullptr && aligned(gather_map, 4), "gather_map must not be NULL");
  const GeoDev g = to_dev(*geo);
  const int4* idx = reinterpret_cast<const int4*>(indices);
  const unsigned grid = static_cast<unsigned>(ceil_div(n, kThreads));
  TSC_LAUNCH_PDL("k_dense_build", k_dense_build, dim3(grid), dim3(kThreads), 0, stream, idx, n, g.B, g.D, g.H, g.W,
                 table, status);
  rc = launch_subm_query(idx, n, g,
                         DenseLookup{table, static_cast<unsigned>(g.D), static_cast<unsigned>(g.H),
                                     static_cast<unsigned>(g.W)},
                         gather_map, meta, stream);
  if (rc != TSC_OK) return rc;
  TSC_LAUNCH_PDL("k_dense_clear", k_dense_clear, dim3(grid), dim3(kThreads), 0, stream, idx, n, g.B, g.D, g.H, g.W,
                 table);
  return TSC_OK;
}

int tsc_subm_kmap_ranked(const int32_t* indices, int64_t n, const tsc_geometry* geo, const void* strided_workspace,
                         size_t workspace_bytes, int32_t* gather_map, int64_t* meta, int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = check_geometry(geo, false);
  if (rc != TSC_OK) return rc;
  TSC_CHECK_ARG(n >= 0 && n <= 0x7fffffffLL, "number of voxels %lld out of range", (long long)n);
  TSC_CHECK_ARG(meta != nullptr && status != nullptr, "meta/status must not be NULL");
  const uint64_t cells = cells_of(geo->batch, geo->in_shape);
  if (cells > kMaxCells64) {
    set_error("grid batch*D*H*W = %llu exceeds the 64-bit key limit 2^62", (unsigned long long)cells);
    return TSC_ERR_GRID_TOO_LARGE;
  }
  // the strided map's workspace over its output grid == this grid
  tsc_geometry og = *geo;
  for (int d = 0; d < 3; ++d) og.out_shape[d] = geo->in_shape[d];
  const StridedWs w = strided_ws(og);
  if (strided_workspace == nullptr || workspace_bytes < w.bytes || !aligned(strided_workspace, 256)) {
    set_error("the strided workspace of this grid has %zu bytes (256-byte aligned), got %zu", w.bytes,
              workspace_bytes);
    return TSC_ERR_WORKSPACE;
  }
  const int K = geo->ksize[0] * geo->ksize[1] * geo->ksize[2];
  rc = fill_words(meta, 0u, 2 * static_cast<int64_t>(TSC_META_COUNTS + K), nullptr, 0u, 0, stream);
  if (rc != TSC_OK || n == 0) return rc;
  TSC_CHECK_ARG(indices != nullptr && aligned(indices, 16), "indices must be 16-byte aligned");
  TSC_CHECK_ARG(gather_map != nullptr && aligned(gather_map, 4), "gather_map must not be NULL");
  const char* ws = static_cast<const char*>(strided_workspace);
  const auto* bitmap = reinterpret_cast<const uint32_t*>(ws);
  const auto* prefix = reinterpret_cast<const uint32_t*>(ws + w.off_prefix);
  const GeoDev g = to_dev(*geo);
  const int4* idx = reinterpret_cast<const int4*>(indices);
  const unsigned D = static_cast<unsigned>(g.D), H = static_cast<unsigned>(g.H), W = static_cast<unsigned>(g.W);
  if (cells > kMaxCells)
    return launch_subm_query(idx, n, g, RankLookup<unsigned long long>{bitmap, prefix, D, H, W}, gather_map, meta,
                             stream);
  return launch_subm_query(idx, n, g, RankLookup<uint32_t>{bitmap, prefix, D, H, W}, gather_map, meta, stream);
}

size_t tsc_strided_kmap_workspace(const tsc_geometry* geo) {
  if (geo == nullptr) return 0;
  // grids the count step refuses need no workspace
  if (cells_of(geo->batch, geo->out_shape) > kMaxCells64) return 0;
  return strided_ws(*geo).bytes;
}

}  // extern "C"

namespace {

int strided_count(const int32_t* indices, int64_t n_in, const tsc_geometry* geo, void* workspace,
                  size_t workspace_bytes, int64_t* meta, int64_t* host_meta, int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = check_geometry(geo, true);
  if (rc != TSC_OK) return rc;
  TSC_CHECK_ARG(n_in >= 0 && n_in <= 0x7fffffffLL, "number of voxels %lld out of range", (long long)n_in);
  TSC_CHECK_ARG(meta != nullptr && status != nullptr, "meta/status must not be NULL");
  const uint64_t out_cells = cells_of(geo->batch, geo->out_shape);
  if (out_cells > kMaxCells64 || out_cells / 32 + kTile > static_cast<uint64_t>(INT64_MAX / 64)) {
    set_error("output grid batch*D*H*W = %llu exceeds the 64-bit key limit 2^62", (unsigned long long)out_cells);
    return TSC_ERR_GRID_TOO_LARGE;
  }
  const bool wide = out_cells > kMaxCells;  // 64-bit bitmap positions
  TSC_CHECK_ARG(n_in == 0 || (indices != nullptr && aligned(indices, 16)),
                "indices must be 16-byte aligned");
  const StridedWs w = strided_ws(*geo);
  if (workspace == nullptr || workspace_bytes < w.bytes || !aligned(workspace, 256)) {
    set_error("strided workspace needs %zu bytes (256-byte aligned), got %zu", w.bytes, workspace_bytes);
    return TSC_ERR_WORKSPACE;
  }
  const int K = geo->ksize[0] * geo->ksize[1] * geo->ksize[2];
  char* ws = static_cast<char*>(workspace);
  auto* bitmap = reinterpret_cast<uint32_t*>(ws);
  auto* sums = reinterpret_cast<uint32_t*>(ws + w.off_sums);
  auto* umeta = reinterpret_cast<unsigned long long*>(meta);
  // meta = 0 and an empty occupancy bitmap, one launch
  int rc2 = fill_words(meta, 0u, 2 * static_cast<int64_t>(TSC_META_COUNTS + K), bitmap, 0u,
                       static_cast<int64_t>(w.nwords_pad), stream);
  if (rc2 != TSC_OK) return rc2;
  const GeoDev g = to_dev(*geo);
  if (n_in > 0) {
    const unsigned grid = static_cast<unsigned>(ceil_div(n_in, kThreads));
    if (wide)
      TSC_LAUNCH_PDL("k_strided_mark", k_strided_mark<unsigned long long>, dim3(grid), dim3(kThreads),
                     sizeof(unsigned) * (K + 1), stream, reinterpret_cast<const int4*>(indices), n_in, g, bitmap, umeta,
                     status);
    else
      TSC_LAUNCH_PDL("k_strided_mark", k_strided_mark<uint32_t>, dim3(grid), dim3(kThreads),
                     sizeof(unsigned) * (K + 1), stream, reinterpret_cast<const int4*>(indices), n_in, g, bitmap, umeta,
                     status);
  }
  TSC_LAUNCH_PDL("k_bitmap_tile_count", k_bitmap_tile_count, dim3(static_cast<unsigned>(w.nblocks)), dim3(kThreads), 0,
                 stream, reinterpret_cast<const uint4*>(bitmap), sums);
  unsigned long long* dev_host_meta = nullptr;
  if (host_meta != nullptr) {
    // the device address of the caller's page-locked buffer (the same
    // address under unified addressing); memory the device cannot address
    // gets an ordinary copy instead
    void* p = nullptr;
    if (cudaHostGetDevicePointer(&p, host_meta, 0) == cudaSuccess && p != nullptr) {
      dev_host_meta = static_cast<unsigned long long*>(p);
    } else {
      (void)cudaGetLastError();
    }
  }
  TSC_LAUNCH_PDL("k_scan_tile_sums", k_scan_tile_sums<uint32_t>, dim3(1), dim3(kScanBlockThreads), 0, stream, sums,
                 w.nblocks, umeta, TSC_META_N_OUT, static_cast<const int64_t*>(status), dev_host_meta,
                 TSC_META_COUNTS + K);
  if (host_meta != nullptr && dev_host_meta == nullptr)
    TSC_CUDA(cudaMemcpyAsync(host_meta, meta, sizeof(int64_t) * (TSC_META_COUNTS + K), cudaMemcpyDeviceToHost,
                             stream));
  return TSC_OK;
}

}  // namespace

extern "C" {

int tsc_strided_kmap_count(const int32_t* indices, int64_t n_in, const tsc_geometry* geo,
                           void* workspace, size_t workspace_bytes, int64_t* meta, int64_t* status,
                           void* stream) {
  return strided_count(indices, n_in, geo, workspace, workspace_bytes, meta, nullptr, status, stream);
}

int tsc_strided_kmap_count_host(const int32_t* indices, int64_t n_in, const tsc_geometry* geo,
                                void* workspace, size_t workspace_bytes, int64_t* meta, int64_t* host_meta,
                                int64_t* status, void* stream) {
  TSC_CHECK_ARG(host_meta != nullptr, "host_meta must not be NULL");
  return strided_count(indices, n_in, geo, workspace, workspace_bytes, meta, host_meta, status, stream);
}

int tsc_strided_kmap_emit(const int32_t* indices, int64_t n_in, const tsc_geometry* geo,
                          void* workspace, size_t workspace_bytes, int64_t n_out,
                          int32_t* out_indices, int32_t* gather_map, int32_t* scatter_map,
                          int32_t* overflow, int64_t overflow_cap, int64_t* meta, int64_t* status,
                          void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = check_geometry(geo, true);
  if (rc != TSC_OK) return rc;
  TSC_CHECK_ARG(n_out >= 0 && n_out <= 0x7fffffffLL, "n_out %lld out of range", (long long)n_out);
  TSC_CHECK_ARG(meta != nullptr && status != nullptr, "meta/status must not be NULL");
  const StridedWs w = strided_ws(*geo);
  if (workspace == nullptr || workspace_bytes < w.bytes || !aligned(workspace, 256)) {
    set_error("strided workspace needs %zu bytes, got %zu", w.bytes, workspace_bytes);
    return TSC_ERR_WORKSPACE;
  }
  if (n_out == 0 || n_in == 0) return TSC_OK;
  TSC_CHECK_ARG(indices != nullptr && aligned(indices, 16), "indices must be 16-byte aligned");
  TSC_CHECK_ARG(out_indices != nullptr && aligned(out_indices, 16), "out_indices must be 16-byte aligned");
  TSC_CHECK_ARG(gather_map != nullptr && scatter_map != nullptr, "maps must not be NULL");
  TSC_CHECK_ARG(overflow_cap == 0 || overflow != nullptr, "overflow buffer is NULL");
  const int K = geo->ksize[0] * geo->ksize[1] * geo->ksize[2];
  char* ws = static_cast<char*>(workspace);
  auto* bitmap = reinterpret_cast<uint32_t*>(ws);
  auto* prefix = reinterpret_cast<uint32_t*>(ws + w.off_prefix);
  auto* sums = reinterpret_cast<uint32_t*>(ws + w.off_sums);
  const GeoDev g = to_dev(*geo);
  // gather map = -1 and the overflow count = 0, one launch
  rc = fill_words(gather_map, 0xFFFFFFFFu, static_cast<int64_t>(K) * n_out, meta + TSC_META_N_OVERFLOW, 0u, 2,
                  stream);
  if (rc != TSC_OK) return rc;
  TSC_LAUNCH_PDL("k_bitmap_prefix", k_bitmap_prefix, dim3(static_cast<unsigned>(w.nblocks)), dim3(kThreads), 0,
                 stream, reinterpret_cast<const uint4*>(bitmap), static_cast<const uint32_t*>(sums), prefix);
  const int64_t nwords = static_cast<int64_t>((w.nbits + 31) / 32);
  const bool wide = w.nbits > kMaxCells;  // 64-bit bitmap positions (the count step refused larger grids)
  const unsigned cgrid = static_cast<unsigned>(ceil_div(nwords, kThreads));
  if (wide)
    TSC_LAUNCH_PDL("k_bitmap_coords", k_bitmap_coords<unsigned long long>, dim3(cgrid), dim3(kThreads), 0, stream,
                   static_cast<const uint32_t*>(bitmap), static_cast<const uint32_t*>(prefix), nwords, g,
                   reinterpret_cast<int4*>(out_indices), n_out);
  else
    TSC_LAUNCH_PDL("k_bitmap_coords", k_bitmap_coords<uint32_t>, dim3(cgrid), dim3(kThreads), 0, stream,
                   static_cast<const uint32_t*>(bitmap), static_cast<const uint32_t*>(prefix), nwords, g,
                   reinterpret_cast<int4*>(out_indices), n_out);
  const unsigned grid = static_cast<unsigned>(ceil_div(n_in, kThreads));
  if (wide)
    TSC_LAUNCH_PDL("k_strided_pairs", k_strided_pairs<unsigned long long>, dim3(grid), dim3(kThreads), 0, stream,
                   reinterpret_cast<const int4*>(indices), n_in, g, static_cast<const uint32_t*>(bitmap),
                   static_cast<const uint32_t*>(prefix), n_out, gather_map, scatter_map, overflow, overflow_cap,
                   reinterpret_cast<unsigned long long*>(meta), status);
  else
    TSC_LAUNCH_PDL("k_strided_pairs", k_strided_pairs<uint32_t>, dim3(grid), dim3(kThreads), 0, stream,
                   reinterpret_cast<const int4*>(indices), n_in, g, static_cast<const uint32_t*>(bitmap),
                   static_cast<const uint32_t*>(prefix), n_out, gather_map, scatter_map, overflow, overflow_cap,
                   reinterpret_cast<unsigned long long*>(meta), status);
  return TSC_OK;
}

size_t tsc_inverse_kmap_workspace(int64_t n_in) { return rows_scan_bytes(n_in); }

int tsc_inverse_kmap_strided(const int32_t* in_indices, int64_t n_in, const int32_t* scatter_map,
                             int32_t k_vol, int64_t n_part, void* workspace, size_t workspace_bytes,
                             int32_t* out_indices, int32_t* inv_gather, int32_t* compact,
                             int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  TSC_CHECK_ARG(k_vol > 0 && k_vol <= 4096, "kernel volume %d out of range", k_vol);
  TSC_CHECK_ARG(n_in >= 0 && n_in <= 0x7fffffffLL && n_part >= 0 && n_part <= n_in,
                "row counts out of range (n_in=%lld, n_part=%lld)", (long long)n_in, (long long)n_part);
  if (n_in == 0) return TSC_OK;
  TSC_CHECK_ARG(in_indices != nullptr && aligned(in_indices, 16), "in_indices must be 16-byte aligned");
  TSC_CHECK_ARG(n_part == 0 || (out_indices != nullptr && aligned(out_indices, 16)),
                "out_indices must be 16-byte aligned");
  TSC_CHECK_ARG(scatter_map != nullptr, "scatter_map is NULL");
  if (n_part == n_in) {
    // Every forward-input row participates: identity compaction.
    TSC_CUDA(cudaMemcpyAsync(out_indices, in_indices, sizeof(int32_t) * 4 * static_cast<size_t>(n_in),
                             cudaMemcpyDeviceToDevice, stream));
    if (inv_gather != nullptr && inv_gather != scatter_map) {
      TSC_CUDA(cudaMemcpyAsync(inv_gather, scatter_map, sizeof(int32_t) * static_cast<size_t>(k_vol) * n_in,
                               cudaMemcpyDeviceToDevice, stream));
    }
    if (compact != nullptr) {
      k_iota<<<static_cast<unsigned>(ceil_div(n_in, kThreads)), kThreads, 0, stream>>>(compact, n_in);
      TSC_LAUNCH_CHECK("k_iota");
    }
    return TSC_OK;
  }
  const size_t need = rows_scan_bytes(n_in);
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16)) {
    set_error("inverse workspace needs %zu bytes, got %zu", need, workspace_bytes);
    return TSC_ERR_WORKSPACE;
  }
  TSC_CHECK_ARG(n_part == 0 || (inv_gather != nullptr && inv_gather != scatter_map),
                "inv_gather must be a separate buffer");
  auto* sums = static_cast<uint32_t*>(workspace);
  const int64_t nblocks = ceil_div(n_in, kTile);
  k_part_tile_count<<<static_cast<unsigned>(nblocks), kThreads, 0, stream>>>(scatter_map, k_vol, n_in, sums);
  TSC_LAUNCH_CHECK("k_part_tile_count");
  k_scan_tile_sums<uint32_t><<<1, kScanBlockThreads, 0, stream>>>(sums, nblocks, nullptr, 0, nullptr);
  TSC_LAUNCH_CHECK("k_scan_tile_sums");
  k_inverse_strided_emit<<<static_cast<unsigned>(nblocks), kThreads, 0, stream>>>(
      reinterpret_cast<const int4*>(in_indices), scatter_map, k_vol, n_in, sums, n_part,
      reinterpret_cast<int4*>(out_indices), inv_gather, compact);
  TSC_LAUNCH_CHECK("k_inverse_strided_emit");
  return TSC_OK;
}

int tsc_inverse_kmap_subm_count(const int32_t* gather_map, int32_t k_vol, int64_t n, void* workspace,
                                size_t workspace_bytes, int32_t* compact, int64_t* meta,
                                int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  TSC_CHECK_ARG(k_vol > 0 && k_vol <= 4096, "kernel volume %d out of range", k_vol);
  TSC_CHECK_ARG(n >= 0 && n <= 0x7fffffffLL, "row count out of range");
  TSC_CHECK_ARG(meta != nullptr, "meta is NULL");
  TSC_CUDA(cudaMemsetAsync(meta + TSC_META_N_PART, 0, sizeof(int64_t), stream));
  if (n == 0) return TSC_OK;
  TSC_CHECK_ARG(gather_map != nullptr && compact != nullptr, "maps must not be NULL");
  const size_t need = rows_scan_bytes(n);
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16)) {
    set_error("inverse workspace needs %zu bytes, got %zu", need, workspace_bytes);
    return TSC_ERR_WORKSPACE;
  }
  auto* sums = static_cast<uint32_t*>(workspace);
  const int64_t total = static_cast<int64_t>(k_vol) * n;
  TSC_CUDA(cudaMemsetAsync(compact, 0, sizeof(int32_t) * static_cast<size_t>(n), stream));
  k_flag_targets<<<static_cast<unsigned>(ceil_div(total, kThreads)), kThreads, 0, stream>>>(
      gather_map, total, n, compact);
  TSC_LAUNCH_CHECK("k_flag_targets");
  const int64_t nblocks = ceil_div(n, kTile);
  k_flag_tile_count<<<static_cast<unsigned>(nblocks), kThreads, 0, stream>>>(compact, n, sums);
  TSC_LAUNCH_CHECK("k_flag_tile_count");
  k_scan_tile_sums<uint32_t><<<1, kScanBlockThreads, 0, stream>>>(
      sums, nblocks, reinterpret_cast<unsigned long long*>(meta), TSC_META_N_PART, status);
  TSC_LAUNCH_CHECK("k_scan_tile_sums");
  k_flag_compact<<<static_cast<unsigned>(nblocks), kThreads, 0, stream>>>(compact, n, sums);
  TSC_LAUNCH_CHECK("k_flag_compact");
  return TSC_OK;
}

int tsc_inverse_kmap_subm_emit(const int32_t* in_indices, const int32_t* gather_map, int32_t k_vol,
                               int64_t n, const int32_t* compact, int64_t n_part, int32_t* out_indices,
                               int32_t* inv_gather, int32_t* overflow, int64_t overflow_cap,
                               int64_t* meta, int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  TSC_CHECK_ARG(k_vol > 0 && k_vol <= 4096, "kernel volume %d out of range", k_vol);
  TSC_CHECK_ARG(n >= 0 && n <= 0x7fffffffLL && n_part >= 0 && n_part <= n, "row counts out of range");
  TSC_CHECK_ARG(meta != nullptr && status != nullptr, "meta/status must not be NULL");
  TSC_CUDA(cudaMemsetAsync(meta + TSC_META_N_OVERFLOW, 0, sizeof(int64_t), stream));
  if (n == 0 || n_part == 0) return TSC_OK;
  TSC_CHECK_ARG(in_indices != nullptr && aligned(in_indices, 16), "in_indices must be 16-byte aligned");
  TSC_CHECK_ARG(out_indices != nullptr && aligned(out_indices, 16), "out_indices must be 16-byte aligned");
  TSC_CHECK_ARG(gather_map != nullptr && compact != nullptr && inv_gather != nullptr, "NULL map");
  TSC_CHECK_ARG(overflow_cap == 0 || overflow != nullptr, "overflow buffer is NULL");
  k_gather_rows<<<static_cast<unsigned>(ceil_div(n, kThreads)), kThreads, 0, stream>>>(
      reinterpret_cast<const int4*>(in_indices), compact, n, n_part, reinterpret_cast<int4*>(out_indices));
  TSC_LAUNCH_CHECK("k_gather_rows");
  TSC_CUDA(cudaMemsetAsync(inv_gather, 0xFF, sizeof(int32_t) * static_cast<size_t>(k_vol) * n_part, stream));
  const int64_t total = static_cast<int64_t>(k_vol) * n;
  k_transpose_map<<<static_cast<unsigned>(ceil_div(total, kThreads)), kThreads, 0, stream>>>(
      gather_map, k_vol, n, compact, n_part, inv_gather, overflow, overflow_cap,
      reinterpret_cast<unsigned long long*>(meta), status);
  TSC_LAUNCH_CHECK("k_transpose_map");
  return TSC_OK;
}

size_t tsc_pairs_workspace(int32_t k_vol, int64_t n) {
  return rows_scan_bytes(static_cast<int64_t>(k_vol) * n);
}

int tsc_pairs_materialize(const int32_t* map, int32_t k_vol, int64_t n, int32_t mode,
                          const int32_t* remap, int64_t* pairs_in, int64_t* pairs_out, int64_t capacity,
                          void* workspace, size_t workspace_bytes, int64_t* status, void* stream_) {
  (void)status;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  TSC_CHECK_ARG(k_vol > 0 && k_vol <= 4096, "kernel volume %d out of range", k_vol);
  TSC_CHECK_ARG(mode == 0 || mode == 1, "mode must be 0 or 1");
  TSC_CHECK_ARG(n >= 0, "row count out of range");
  const int64_t total = static_cast<int64_t>(k_vol) * n;
  if (total == 0 || capacity <= 0) return TSC_OK;
  TSC_CHECK_ARG(map != nullptr && pairs_in != nullptr && pairs_out != nullptr, "NULL buffer");
  const size_t need = rows_scan_bytes(total);
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16)) {
    set_error("pairs workspace needs %zu bytes, got %zu", need, workspace_bytes);
    return TSC_ERR_WORKSPACE;
  }
  const int64_t nblocks = ceil_div(total, kTile);
  TSC_CHECK_ARG(nblocks <= 0x7fffffffLL, "pair map too large");
  auto* sums = static_cast<unsigned long long*>(workspace);
  k_map_tile_count<<<static_cast<unsigned>(nblocks), kThreads, 0, stream>>>(map, total, sums);
  TSC_LAUNCH_CHECK("k_map_tile_count");
  k_scan_tile_sums<unsigned long long><<<1, kScanBlockThreads, 0, stream>>>(sums, nblocks, nullptr, 0, nullptr);
  TSC_LAUNCH_CHECK("k_scan_tile_sums");
  k_map_emit_pairs<<<static_cast<unsigned>(nblocks), kThreads, 0, stream>>>(
      map, total, n, mode, remap, sums, pairs_in, pairs_out, capacity);
  TSC_LAUNCH_CHECK("k_map_emit_pairs");
  return TSC_OK;
}

int tsc_gather_from_pairs(const int64_t* pairs_in, const int64_t* pairs_out, const int64_t* offsets_host,
                          int32_t k_vol, int64_t n_out, int32_t* gather_map, int32_t* overflow,
                          int64_t overflow_cap, int64_t* meta, int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  TSC_CHECK_ARG(k_vol > 0 && k_vol <= 4096, "kernel volume %d out of range", k_vol);
  TSC_CHECK_ARG(n_out >= 0 && n_out <= 0x7fffffffLL, "n_out out of range");
  TSC_CHECK_ARG(offsets_host != nullptr && meta != nullptr && status != nullptr, "NULL argument");
  TSC_CUDA(cudaMemsetAsync(meta + TSC_META_N_OVERFLOW, 0, sizeof(int64_t), stream));
  if (n_out == 0) return TSC_OK;
  TSC_CHECK_ARG(gather_map != nullptr, "gather_map is NULL");
  TSC_CHECK_ARG(overflow_cap == 0 || overflow != nullptr, "overflow buffer is NULL");
  TSC_CUDA(cudaMemsetAsync(gather_map, 0xFF, sizeof(int32_t) * static_cast<size_t>(k_vol) * n_out, stream));
  for (int k = 0; k < k_vol; ++k) {
    const int64_t b = offsets_host[k], e = offsets_host[k + 1];
    TSC_CHECK_ARG(b >= 0 && e >= b, "pair offsets are not monotone at k=%d", k);
    if (e == b) continue;
    k_pairs_to_gather<<<static_cast<unsigned>(ceil_div(e - b, kThreads)), kThreads, 0, stream>>>(
        pairs_in + b, pairs_out + b, e - b, k, n_out, gather_map, overflow, overflow_cap,
        reinterpret_cast<unsigned long long*>(meta), status);
    TSC_LAUNCH_CHECK("k_pairs_to_gather");
  }
  return TSC_OK;
}

}  // extern "C"

// ---- allocation-free submanifold kernel map ---------------------------------
// Some callers cannot allocate device memory at the moment they build a map:
// code running under a caller-owned memory pool or budget that forbids
// cudaMalloc, host code that must not synchronise the device (cudaMalloc and
// cudaFree can), and language bindings that have no allocator of their own.
// tsc_subm_kmap_noalloc serves them with a hash table that lives in a fixed
// file-scope device array instead of a caller-provided workspace.

namespace tsc {
namespace {

constexpr int kNoAllocLog2Cap = 21;  // 2^21 hash entries of 8 bytes = 16 MiB per device
constexpr int64_t kNoAllocMaxVoxels = int64_t{1} << (kNoAllocLog2Cap - 1);
constexpr int kNoAllocMaxDevices = 64;

// Held by every GPU that loads this library until the process exits.  In host
// code this name denotes a host-side stand-in, not a device address: the
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned long long g_subm_scratch[size_t{1} << kNoAllocLog2Cap];

std::mutex g_scratch_mu;
void* g_scratch_addr[kNoAllocMaxDevices] = {};

// Device address of g_subm_scratch on the device that owns `stream`, looked
// up once per device (the first call on each device does it).  That device
// must be the current one: the kernels are launched on the current device.
int scratch_address(cudaStream_t stream, void** out) {
  int dev = 0;
  TSC_CUDA(cudaGetDevice(&dev));
  int sdev = dev;
  TSC_CUDA(cudaStreamGetDevice(stream, &sdev));
  if (sdev != dev) {
    set_error("the stream belongs to device %d but device %d is current; make the stream's device current",
              sdev, dev);
    return TSC_ERR_UNSUPPORTED;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    set_error("device ordinal %d exceeds the %d devices the allocation-free path supports", dev,
              kNoAllocMaxDevices);
    return TSC_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    TSC_CUDA(cudaGetSymbolAddress(&p, g_subm_scratch));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return TSC_OK;
}

}  // namespace
}  // namespace tsc

extern "C" {

int64_t tsc_subm_kmap_noalloc_max_voxels(void) { return tsc::kNoAllocMaxVoxels; }

int tsc_subm_kmap_noalloc(const int32_t* indices, int64_t n, const tsc_geometry* geo, int32_t* gather_map,
                          int64_t* meta, int64_t* status, void* stream_) {
  using namespace tsc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = check_geometry(geo, false);
  if (rc != TSC_OK) return rc;
  TSC_CHECK_ARG(n >= 0, "number of voxels %lld is negative", (long long)n);
  if (n > kNoAllocMaxVoxels) {
    set_error("tsc_subm_kmap_noalloc takes at most %lld voxels (fixed 16 MiB device table), got %lld; "
              "use tsc_subm_kmap with a caller-provided workspace",
              (long long)kNoAllocMaxVoxels, (long long)n);
    return TSC_ERR_WORKSPACE;
  }
  TSC_CHECK_ARG(meta != nullptr && status != nullptr, "meta/status must not be NULL");
  const uint64_t cells = cells_of(geo->batch, geo->in_shape);
  if (cells > kMaxCells) {
    set_error("grid batch*D*H*W = %llu exceeds the packed-key limit 2^32-2", (unsigned long long)cells);
    return TSC_ERR_GRID_TOO_LARGE;
  }
  void* scratch = nullptr;
  rc = scratch_address(stream, &scratch);
  if (rc != TSC_OK) return rc;
  const int K = geo->ksize[0] * geo->ksize[1] * geo->ksize[2];
  const int64_t meta_words = 2 * static_cast<int64_t>(TSC_META_COUNTS + K);
  if (n == 0) return fill_words(meta, 0u, meta_words, nullptr, 0u, 0, stream);
  TSC_CHECK_ARG(indices != nullptr && aligned(indices, 16), "indices must be 16-byte aligned");
  TSC_CHECK_ARG(gather_map != nullptr && aligned(gather_map, 4), "gather_map must not be NULL");
  // same table capacity as tsc_subm_kmap; the part in use is reset on every
  // call because the array keeps the previous call's entries.  From here on
  // the launches are those of tsc_subm_kmap: meta and table cleared by one
  // fill kernel, then the build and the query as dependent launches.
  const int log2cap = subm_log2cap(n);
  auto* table = static_cast<unsigned long long*>(scratch);
  rc = fill_words(meta, 0u, meta_words, table, 0xFFFFFFFFu, static_cast<int64_t>(2) << log2cap, stream);
  if (rc != TSC_OK) return rc;
  const GeoDev g = to_dev(*geo);
  const int4* idx = reinterpret_cast<const int4*>(indices);
  const unsigned grid = static_cast<unsigned>(ceil_div(n, kThreads));
  TSC_LAUNCH_PDL("k_hash_build", k_hash_build, dim3(grid), dim3(kThreads), 0, stream, idx, n, g.B, g.D, g.H, g.W,
                 table, log2cap, status);
  return launch_subm_query(idx, n, g, table, log2cap, gather_map, meta, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Voxelisation: points -> unique voxels in (b, z, y, x) key order
// ---------------------------------------------------------------------------

namespace tsc {
namespace {

struct VoxDev {
  int B, D, H, W;
  float lo[3];
  float size[3];
};

VoxDev to_vox(const tsc_voxel_params& p) {
  VoxDev v;
  v.B = p.batch;
  v.D = p.grid[0];
  v.H = p.grid[1];
  v.W = p.grid[2];
  for (int d = 0; d < 3; ++d) {
    v.lo[d] = p.range_lo[d];
    v.size[d] = p.voxel_size[d];
  }
  return v;
}

// Voxel (b, z, y, x) of point i; false when it lies outside the grid (NaN
// coordinates included) or its batch id is outside [0, B) (then *bad).
__device__ __forceinline__ bool point_voxel(const float* __restrict__ pts, int dim, const int32_t* __restrict__ bid,
                                            int64_t i, const VoxDev& v, int& b, int& z, int& y, int& x, bool& bad) {
  b = bid != nullptr ? __ldg(&bid[i]) : 0;
  bad = b < 0 || b >= v.B;
  if (bad) return false;
  const float* p = pts + i * dim;
  const float fx = floorf((__ldg(&p[0]) - v.lo[0]) / v.size[0]);
  const float fy = floorf((__ldg(&p[1]) - v.lo[1]) / v.size[1]);
  const float fz = floorf((__ldg(&p[2]) - v.lo[2]) / v.size[2]);
  if (!(fx >= 0.f && fx < static_cast<float>(v.W) && fy >= 0.f && fy < static_cast<float>(v.H) && fz >= 0.f &&
        fz < static_cast<float>(v.D)))
    return false;
  x = static_cast<int>(fx);
  y = static_cast<int>(fy);
  z = static_cast<int>(fz);
  return x < v.W && y < v.H && z < v.D;
}

template <typename KeyT>
__global__ void __launch_bounds__(kThreads)
k_vox_mark(const float* __restrict__ pts, int64_t n, int dim, const int32_t* __restrict__ bid, VoxDev v,
           uint32_t* __restrict__ bitmap, unsigned long long* __restrict__ meta, int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int b = 0, z = 0, y = 0, x = 0;
  bool bad = false;
  const bool ok = i < n && point_voxel(pts, dim, bid, i, v, b, z, y, x, bad);
  if (i < n && bad) raise_status(status, TSC_STATUS_KEY_RANGE);
  const unsigned kept = __ballot_sync(kFullMask, ok);
  if (ok) {
    // lanes that hit the same bitmap word combine their bits; one atomic per word
    const KeyT lin = cell_key_t<KeyT>(b, z, y, x, v.D, v.H, v.W);
    const KeyT word = lin >> 5;
    const unsigned same = __match_any_sync(kept, word);
    const unsigned bits = __reduce_or_sync(same, 1u << static_cast<unsigned>(lin & 31u));
    if ((threadIdx.x & 31) == static_cast<unsigned>(__ffs(same) - 1)) atomicOr(&bitmap[word], bits);
  }
  if ((threadIdx.x & 31) == 0 && kept) atomicAdd(&meta[TSC_META_N_PART], static_cast<unsigned long long>(__popc(kept)));
}

// Voxel rank of every kept point (-1 for dropped ones) and the points per voxel.
template <typename KeyT>
__global__ void __launch_bounds__(kThreads)
k_vox_rank(const float* __restrict__ pts, int64_t n, int dim, const int32_t* __restrict__ bid, VoxDev v,
           const uint32_t* __restrict__ bitmap, const uint32_t* __restrict__ word_prefix, int64_t n_vox,
           int32_t* __restrict__ rank, int32_t* __restrict__ counts, int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int b = 0, z = 0, y = 0, x = 0;
  bool bad = false;
  int r = -1;
  if (point_voxel(pts, dim, bid, i, v, b, z, y, x, bad)) {
    const KeyT lin = cell_key_t<KeyT>(b, z, y, x, v.D, v.H, v.W);
    const KeyT w = lin >> 5;
    r = static_cast<int>(__ldg(&word_prefix[w]) +
                         __popc(__ldg(&bitmap[w]) & ((1u << static_cast<unsigned>(lin & 31u)) - 1u)));
    if (r >= n_vox) {
      raise_status(status, TSC_STATUS_INTERNAL);
      r = -1;
    } else {
      atomicAdd(&counts[r], 1);
    }
  }
  rank[i] = r;
}

// Exclusive prefix of per-voxel counts: tile sums, then per element.
__global__ void __launch_bounds__(kThreads)
k_vox_tile_sums(const int32_t* __restrict__ counts, int64_t n, uint32_t* __restrict__ tile_sums) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t ws[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile + threadIdx.x * kItems;
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j)
    if (base + j < n) s += static_cast<uint32_t>(counts[base + j]);
  uint32_t total;
  block_exclusive_scan(s, ws, &total);
  if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kThreads)
k_vox_offsets(const int32_t* __restrict__ counts, int64_t n, const uint32_t* __restrict__ tile_off,
              int32_t* __restrict__ offsets) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t ws[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile + threadIdx.x * kItems;
  uint32_t c[kItems];
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    c[j] = base + j < n ? static_cast<uint32_t>(counts[base + j]) : 0u;
    s += c[j];
  }
  uint32_t total;
  uint32_t run = block_exclusive_scan(s, ws, &total) + tile_off[blockIdx.x];
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    if (base + j < n) offsets[base + j] = static_cast<int32_t>(run);
    run += c[j];
  }
}

// Every kept point into its voxel's segment of `list` (order within the
// segment depends on the atomics; k_vox_reduce sorts it).
__global__ void __launch_bounds__(kThreads)
k_vox_fill(const int32_t* __restrict__ rank, int64_t n, const int32_t* __restrict__ offsets,
           int32_t* __restrict__ fill, int32_t* __restrict__ list) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = rank[i];
  if (r < 0) return;
  const int slot = atomicAdd(&fill[r], 1);
  list[offsets[r] + slot] = static_cast<int32_t>(i);
}

// One thread per voxel: sort its point indices ascending (insertion sort:
// voxels hold few points), keep the first max_points, and average every
// column over them, summing in index order.
__global__ void __launch_bounds__(kThreads)
k_vox_reduce(const float* __restrict__ pts, int dim, int32_t* __restrict__ list, const int32_t* __restrict__ offsets,
             const int32_t* __restrict__ counts, int64_t n_vox, int max_points, float* __restrict__ features,
             int32_t* __restrict__ num_points) {
  pdl_wait();
  pdl_trigger();
  const int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (v >= n_vox) return;
  const int c = counts[v];
  int32_t* seg = list + offsets[v];
  for (int a = 1; a < c; ++a) {
    const int32_t key = seg[a];
    int j = a - 1;
    while (j >= 0 && seg[j] > key) {
      seg[j + 1] = seg[j];
      --j;
    }
    seg[j + 1] = key;
  }
  const int m = (max_points > 0 && c > max_points) ? max_points : c;
  num_points[v] = m;
  for (int d = 0; d < dim; ++d) {
    float s = 0.f;
    for (int a = 0; a < m; ++a) s += __ldg(&pts[static_cast<int64_t>(seg[a]) * dim + d]);
    features[v * dim + d] = m > 0 ? s / static_cast<float>(m) : 0.f;
  }
}

struct VoxWs {
  StridedWs bm;  // occupancy bitmap, word prefix, tile sums over batch*D*H*W
  size_t off_rank, off_counts, off_offsets, off_fill, off_list, off_vsums, bytes;
  int64_t vtiles;
};

VoxWs vox_ws(const tsc_voxel_params& p, int64_t n) {
  tsc_geometry g{};
  g.batch = p.batch;
  for (int d = 0; d < 3; ++d) g.out_shape[d] = p.grid[d];
  VoxWs w;
  w.bm = strided_ws(g);
  const size_t nn = static_cast<size_t>(n < 1 ? 1 : n);
  w.vtiles = ceil_div(static_cast<int64_t>(nn), kTile);
  w.off_rank = align_up(w.bm.bytes, 256);
  w.off_counts = w.off_rank + align_up(nn * 4, 256);
  w.off_offsets = w.off_counts + align_up(nn * 4, 256);
  w.off_fill = w.off_offsets + align_up(nn * 4, 256);
  w.off_list = w.off_fill + align_up(nn * 4, 256);
  w.off_vsums = w.off_list + align_up(nn * 4, 256);
  w.bytes = w.off_vsums + align_up(static_cast<size_t>(w.vtiles + 1) * 4, 256);
  return w;
}

int check_vox(const float* points, int64_t n, int32_t dim, const tsc_voxel_params* vp, int64_t* meta,
              int64_t* status) {
  TSC_CHECK_ARG(vp != nullptr, "voxel parameters are NULL");
  TSC_CHECK_ARG(vp->batch > 0 && vp->grid[0] > 0 && vp->grid[1] > 0 && vp->grid[2] > 0,
                "batch and grid extents must be positive");
  for (int d = 0; d < 3; ++d)
    TSC_CHECK_ARG(vp->voxel_size[d] > 0.f, "voxel_size[%d] must be positive", d);
  TSC_CHECK_ARG(dim >= 3 && dim <= 64, "point_dim %d must be in [3, 64]", dim);
  TSC_CHECK_ARG(n >= 0 && n <= 0x7fffffffLL, "number of points %lld out of range", (long long)n);
  TSC_CHECK_ARG(n == 0 || (points != nullptr && aligned(points, 4)), "points must not be NULL");
  TSC_CHECK_ARG(meta != nullptr && status != nullptr, "meta/status must not be NULL");
  tsc_geometry g{};
  g.batch = vp->batch;
  for (int d = 0; d < 3; ++d) g.out_shape[d] = vp->grid[d];
  if (cells_of(g.batch, g.out_shape) > kMaxCells64) {
    set_error("voxel grid batch*D*H*W exceeds 2^62 cells");
    return TSC_ERR_GRID_TOO_LARGE;
  }
  return TSC_OK;
}

}  // namespace
}  // namespace tsc

extern "C" {

size_t tsc_voxelize_workspace(const tsc_voxel_params* vp, int64_t n_points) {
  if (vp == nullptr || vp->batch <= 0 || vp->grid[0] <= 0 || vp->grid[1] <= 0 || vp->grid[2] <= 0) return 0;
  tsc_geometry g{};
  g.batch = vp->batch;
  for (int d = 0; d < 3; ++d) g.out_shape[d] = vp->grid[d];
  if (cells_of(g.batch, g.out_shape) > kMaxCells64) return 0;
  return vox_ws(*vp, n_points).bytes;
}

int tsc_voxelize_count(const float* points, int64_t n, int32_t point_dim, const int32_t* batch_ids,
                       const tsc_voxel_params* vp, void* workspace, size_t workspace_bytes, int64_t* meta,
                       int64_t* status, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = check_vox(points, n, point_dim, vp, meta, status);
  if (rc != TSC_OK) return rc;
  const VoxWs w = vox_ws(*vp, n);
  if (workspace == nullptr || workspace_bytes < w.bytes || !aligned(workspace, 256)) {
    set_error("voxelize workspace needs %zu bytes (256-byte aligned), got %zu", w.bytes, workspace_bytes);
    return TSC_ERR_WORKSPACE;
  }
  char* ws = static_cast<char*>(workspace);
  auto* bitmap = reinterpret_cast<uint32_t*>(ws);
  auto* sums = reinterpret_cast<uint32_t*>(ws + w.bm.off_sums);
  auto* umeta = reinterpret_cast<unsigned long long*>(meta);
  rc = fill_words(meta, 0u, 2 * static_cast<int64_t>(TSC_META_COUNTS), bitmap, 0u, w.bm.nwords_pad, stream);
  if (rc != TSC_OK) return rc;
  const VoxDev v = to_vox(*vp);
  const bool wide = w.bm.nbits > kMaxCells;
  if (n > 0) {
    const unsigned grid = static_cast<unsigned>(ceil_div(n, kThreads));
    if (wide)
      TSC_LAUNCH_PDL("k_vox_mark", k_vox_mark<unsigned long long>, dim3(grid), dim3(kThreads), 0, stream, points, n,
                     point_dim, batch_ids, v, bitmap, umeta, status);
    else
      TSC_LAUNCH_PDL("k_vox_mark", k_vox_mark<uint32_t>, dim3(grid), dim3(kThreads), 0, stream, points, n,
                     point_dim, batch_ids, v, bitmap, umeta, status);
  }
  TSC_LAUNCH_PDL("k_bitmap_tile_count", k_bitmap_tile_count, dim3(static_cast<unsigned>(w.bm.nblocks)), dim3(kThreads),
                 0, stream, reinterpret_cast<const uint4*>(bitmap), sums);
  TSC_LAUNCH_PDL("k_scan_tile_sums", k_scan_tile_sums<uint32_t>, dim3(1), dim3(kScanBlockThreads), 0, stream, sums,
                 w.bm.nblocks, umeta, TSC_META_N_OUT, static_cast<const int64_t*>(status),
                 static_cast<unsigned long long*>(nullptr), 0);
  return TSC_OK;
}

int tsc_voxelize_emit(const float* points, int64_t n, int32_t point_dim, const int32_t* batch_ids,
                      const tsc_voxel_params* vp, void* workspace, size_t workspace_bytes, int64_t n_vox,
                      int32_t* coords, float* features, int32_t* num_points, int64_t* meta, int64_t* status,
                      void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = check_vox(points, n, point_dim, vp, meta, status);
  if (rc != TSC_OK) return rc;
  TSC_CHECK_ARG(n_vox >= 0 && n_vox <= n, "n_vox %lld must lie in [0, n]", (long long)n_vox);
  const VoxWs w = vox_ws(*vp, n);
  if (workspace == nullptr || workspace_bytes < w.bytes || !aligned(workspace, 256)) {
    set_error("voxelize workspace needs %zu bytes (256-byte aligned), got %zu", w.bytes, workspace_bytes);
    return TSC_ERR_WORKSPACE;
  }
  if (n_vox == 0) return TSC_OK;
  TSC_CHECK_ARG(coords != nullptr && aligned(coords, 16) && features != nullptr && num_points != nullptr,
                "coords (16-byte aligned), features and num_points must not be NULL");
  char* ws = static_cast<char*>(workspace);
  auto* bitmap = reinterpret_cast<uint32_t*>(ws);
  auto* prefix = reinterpret_cast<uint32_t*>(ws + w.bm.off_prefix);
  auto* sums = reinterpret_cast<uint32_t*>(ws + w.bm.off_sums);
  auto* rank = reinterpret_cast<int32_t*>(ws + w.off_rank);
  auto* counts = reinterpret_cast<int32_t*>(ws + w.off_counts);
  auto* offsets = reinterpret_cast<int32_t*>(ws + w.off_offsets);
  auto* fill = reinterpret_cast<int32_t*>(ws + w.off_fill);
  auto* list = reinterpret_cast<int32_t*>(ws + w.off_list);
  auto* vsums = reinterpret_cast<uint32_t*>(ws + w.off_vsums);
  const VoxDev v = to_vox(*vp);
  const bool wide = w.bm.nbits > kMaxCells;
  rc = fill_words(counts, 0u, n_vox, fill, 0u, n_vox, stream);
  if (rc != TSC_OK) return rc;
  TSC_LAUNCH_PDL("k_bitmap_prefix", k_bitmap_prefix, dim3(static_cast<unsigned>(w.bm.nblocks)), dim3(kThreads), 0,
                 stream, reinterpret_cast<const uint4*>(bitmap), static_cast<const uint32_t*>(sums), prefix);
  // voxel coordinates in key order: the bitmap decoded like a strided map's
  // output set (B = batch, out grid = the voxel grid)
  GeoDev g{};
  g.B = v.B;
  g.oD = v.D;
  g.oH = v.H;
  g.oW = v.W;
  const int64_t nwords = static_cast<int64_t>((w.bm.nbits + 31) / 32);
  const unsigned cgrid = static_cast<unsigned>(ceil_div(nwords, kThreads));
  if (wide)
    TSC_LAUNCH_PDL("k_bitmap_coords", k_bitmap_coords<unsigned long long>, dim3(cgrid), dim3(kThreads), 0, stream,
                   static_cast<const uint32_t*>(bitmap), static_cast<const uint32_t*>(prefix), nwords, g,
                   reinterpret_cast<int4*>(coords), n_vox);
  else
    TSC_LAUNCH_PDL("k_bitmap_coords", k_bitmap_coords<uint32_t>, dim3(cgrid), dim3(kThreads), 0, stream,
                   static_cast<const uint32_t*>(bitmap), static_cast<const uint32_t*>(prefix), nwords, g,
                   reinterpret_cast<int4*>(coords), n_vox);
  const unsigned pgrid = static_cast<unsigned>(ceil_div(n, kThreads));
  if (wide)
    TSC_LAUNCH_PDL("k_vox_rank", k_vox_rank<unsigned long long>, dim3(pgrid), dim3(kThreads), 0, stream, points, n,
                   point_dim, batch_ids, v, static_cast<const uint32_t*>(bitmap), static_cast<const uint32_t*>(prefix),
                   n_vox, rank, counts, status);
  else
    TSC_LAUNCH_PDL("k_vox_rank", k_vox_rank<uint32_t>, dim3(pgrid), dim3(kThreads), 0, stream, points, n, point_dim,
                   batch_ids, v, static_cast<const uint32_t*>(bitmap), static_cast<const uint32_t*>(prefix), n_vox,
                   rank, counts, status);
  const int64_t vt = ceil_div(n_vox, kTile);
  TSC_LAUNCH_PDL("k_vox_tile_sums", k_vox_tile_sums, dim3(static_cast<unsigned>(vt)), dim3(kThreads), 0, stream,
                 static_cast<const int32_t*>(counts), n_vox, vsums);
  TSC_LAUNCH_PDL("k_scan_tile_sums", k_scan_tile_sums<uint32_t>, dim3(1), dim3(kScanBlockThreads), 0, stream, vsums,
                 vt, static_cast<unsigned long long*>(nullptr), 0, static_cast<const int64_t*>(nullptr),
                 static_cast<unsigned long long*>(nullptr), 0);
  TSC_LAUNCH_PDL("k_vox_offsets", k_vox_offsets, dim3(static_cast<unsigned>(vt)), dim3(kThreads), 0, stream,
                 static_cast<const int32_t*>(counts), n_vox, static_cast<const uint32_t*>(vsums), offsets);
  TSC_LAUNCH_PDL("k_vox_fill", k_vox_fill, dim3(pgrid), dim3(kThreads), 0, stream, static_cast<const int32_t*>(rank),
                 n, static_cast<const int32_t*>(offsets), fill, list);
  TSC_LAUNCH_PDL("k_vox_reduce", k_vox_reduce, dim3(static_cast<unsigned>(ceil_div(n_vox, kThreads))), dim3(kThreads),
                 0, stream, points, point_dim, list, static_cast<const int32_t*>(offsets),
                 static_cast<const int32_t*>(counts), n_vox, vp->max_points, features, num_points);
  return TSC_OK;
}

}  // extern "C"
