// Persistent tcgen05 implicit GEMM with a per-tile input halo in shared
// memory (sm_100a), for 64-channel input rows.
//
// The TMA-gather kernel (conv_tcp.cuh) fetches one feature row from L2 for
// every (output row, offset) pair of a tile, so an input row that feeds n
// outputs of the tile crosses the L2 -> SM path n times.  On LiDAR-like maps
// the 256 output rows of a tile touch only 25-40 % as many distinct input
// rows as they have pairs.  This kernel fetches each distinct input row of a
// tile once (the tile's "halo", listed by tsc_tile_halo) into shared memory
// with TMA gather4 and builds every A operand tile from there with
// shared-memory copies.  Rows that do not fit the halo buffer are read from
// global memory by the same copy loop.
//
// Same tile shape, accumulators, masks, MMA sequence and epilogue as the
// TMA-gather kernel, so both produce bit-identical outputs.  Warp roles
// (288 threads):
//   warps 0-3  producers.  Warp 0 loads the tile's halo (TMA gather4 of the
//              halo list, one 128-byte row per input voxel) once the previous
//              tile's copies are done, and the weight slice of every step
//              (TMA tile load).  For every active offset k, warp w copies
//              the rows 64w..64w+63 that have a pair at k from the halo (or
//              global memory) into the swizzled A stage, 8 lanes per row, and
//              arrives on the stage's full barrier after a proxy fence.
//   warp 4     one thread issues tcgen05.mma with the per-row
//              disable-output-lane masks (as in the TMA-gather kernel).
//   warps 5-8  epilogue and set-up of the tile two ahead: output rows and
//              per-offset lane masks from the halo map.
// All mbarrier waits are bounded; no named barrier is used after the start.
#pragma once

#include <cuda.h>

#include "conv_tc.cuh"
#include "conv_tcp.cuh"

namespace tsc {
namespace tch {

using tcp::BMT;
using tcp::HALF;
using tcp::KMAX;
constexpr int NPROD = 128;
constexpr int NEPI = 128;
constexpr int EPI0 = NPROD + 32;
constexpr int NT = NPROD + 32 + NEPI;
constexpr int KC = 64;              // input channels (one 128-byte row per voxel)
constexpr int ROW_BYTES = KC * 2;   // 16-bit elements
constexpr int NS = 2;               // A/B stages
constexpr int SMEM_MAX = 227 * 1024;

// halo map entries: local row (>= 0), no pair, or "read from the gather map"
constexpr int kNoPair = -1;
constexpr int kOutsideHalo = -2;

struct Info {
  static constexpr int OROW = BMT * 4;            // int32 output row, -1 past the end
  static constexpr int LMASK = KMAX * 2 * 4 * 4;  // uint32 [k][half][word]: rows WITHOUT a pair
  static constexpr int KMASK = 4 * 4;             // uint32 [epilogue warp]: active offsets, OR them
  static constexpr int OFF_OROW = 0;
  static constexpr int OFF_LMASK = OFF_OROW + OROW;
  static constexpr int OFF_KMASK = OFF_LMASK + LMASK;
  static constexpr int OFF_TILE = OFF_KMASK + KMASK;  // int32 tile index, -1 = no more tiles
  static constexpr int BYTES = (OFF_TILE + 4 + 127) / 128 * 128;
};

template <int TN>
struct Cfg {
  static_assert(TN == 32 || TN == 64 || TN == 128 || TN == 256, "halo kernel tile width");
  static constexpr int NACC = (4 * TN <= 512) ? 2 : 1;
  static constexpr int TMEM_COLS = NACC * 2 * TN;
  static constexpr int A_BYTES = BMT * ROW_BYTES;
  static constexpr int B_BYTES = TN * ROW_BYTES;
  static constexpr int STAGE = (A_BYTES + B_BYTES + 1023) / 1024 * 1024;
  static constexpr int CTRL = 256;
  static constexpr int BIAS = 256 * 4;
  static constexpr int FIXED = 1024 /*alignment slack*/ + CTRL + 2 * Info::BYTES + BIAS;
  // halo rows: what is left after two stages, a multiple of 32 rows
  static constexpr int HALO = (SMEM_MAX - FIXED - NS * STAGE) / ROW_BYTES / 32 * 32;
  static_assert(HALO >= 256, "halo buffer");
  static constexpr int OFF_HALO = NS * STAGE;  // 1024-aligned: swizzle atoms are address based
  static constexpr int OFF_CTRL = OFF_HALO + HALO * ROW_BYTES;
  static constexpr int OFF_FULL = 0;
  static constexpr int OFF_EMPTY = 8 * NS;
  static constexpr int OFF_HFULL = 16 * NS;
  static constexpr int OFF_HFREE = OFF_HFULL + 8;
  static constexpr int OFF_IFULL = OFF_HFREE + 8;
  static constexpr int OFF_IEMPTY = OFF_IFULL + 16;
  static constexpr int OFF_AFULL = OFF_IEMPTY + 16;
  static constexpr int OFF_AEMPTY = OFF_AFULL + 16;
  static constexpr int OFF_TIDXB = OFF_AEMPTY + 16;
  static constexpr int OFF_TMEM = OFF_TIDXB + 16;
  static constexpr int OFF_ABORT = OFF_TMEM + 4;
  static constexpr int OFF_TIDX = OFF_ABORT + 4;  // int32[2]
  static_assert(OFF_TIDX + 8 <= CTRL, "control block");
  static constexpr int OFF_INFO = OFF_CTRL + CTRL;
  static constexpr int OFF_BIAS = OFF_INFO + 2 * Info::BYTES;
  static constexpr int TOTAL = 1024 + OFF_BIAS + BIAS;
  static_assert(TOTAL <= SMEM_MAX, "shared memory");
  static constexpr int SWZ_MODE = 2;  // 128-byte swizzle, K-major
  static constexpr int SBO = 8 * ROW_BYTES;
};

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// byte offset of 16-byte chunk `c` of row `r` in a 128-byte-swizzled tile
// whose base is 1024-byte aligned (the layout TMA writes and UMMA reads)
__device__ __forceinline__ uint32_t swz128(int r, int c) {
  return static_cast<uint32_t>(r) * ROW_BYTES + (static_cast<uint32_t>(c ^ (r & 7)) << 4);
}

template <typename T, int TN>
__global__ void __launch_bounds__(NT, 1)
k_conv_tch(const __grid_constant__ CUtensorMap tmap_f, const __grid_constant__ CUtensorMap tmap_w,
           const T* __restrict__ F, int64_t n_in, const T* __restrict__ W, const T* __restrict__ bias,
           const int32_t* __restrict__ gmap, int K, int64_t n_out, int c_out, const int32_t* __restrict__ ovf,
           int64_t ovf_cap, const int64_t* __restrict__ meta, T* __restrict__ out, int flags,
           int64_t* __restrict__ status, unsigned* __restrict__ tile_counter,
           const int32_t* __restrict__ halo_rows, const int32_t* __restrict__ halo_count,
           const int16_t* __restrict__ hmap) {
  pdl_wait();
  pdl_trigger();
  using C = Cfg<TN>;
  constexpr int NACC = C::NACC;
  constexpr int HALO = C::HALO;
  constexpr int QPL = (HALO / 4 + 31) / 32;  // halo quads per lane of warp 0
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u32 = mma::smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_u32 & 1023u)) & 1023u;
  unsigned char* ring = smem_raw + pad;
  const uint32_t ring_u32 = raw_u32 + pad;
  const uint32_t halo_u32 = ring_u32 + C::OFF_HALO;
  unsigned char* ctrl = ring + C::OFF_CTRL;
  const uint32_t ctrl_u32 = ring_u32 + C::OFF_CTRL;
  const uint32_t bar_full = ctrl_u32 + C::OFF_FULL;
  const uint32_t bar_empty = ctrl_u32 + C::OFF_EMPTY;
  const uint32_t bar_hfull = ctrl_u32 + C::OFF_HFULL;
  const uint32_t bar_hfree = ctrl_u32 + C::OFF_HFREE;
  const uint32_t bar_ifull = ctrl_u32 + C::OFF_IFULL;
  const uint32_t bar_iempty = ctrl_u32 + C::OFF_IEMPTY;
  const uint32_t bar_afull = ctrl_u32 + C::OFF_AFULL;
  const uint32_t bar_aempty = ctrl_u32 + C::OFF_AEMPTY;
  const uint32_t bar_tidx = ctrl_u32 + C::OFF_TIDXB;
  volatile int32_t* s_tidx = reinterpret_cast<volatile int32_t*>(ctrl + C::OFF_TIDX);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(ctrl + C::OFF_TMEM);
  volatile int* s_abort = reinterpret_cast<volatile int*>(ctrl + C::OFF_ABORT);
  unsigned char* info0 = ring + C::OFF_INFO;
  float* s_bias = reinterpret_cast<float*>(ring + C::OFF_BIAS);
  auto orow_of = [&](int ib) { return reinterpret_cast<int32_t*>(info0 + ib * Info::BYTES + Info::OFF_OROW); };
  auto lmask_of = [&](int ib) { return reinterpret_cast<uint32_t*>(info0 + ib * Info::BYTES + Info::OFF_LMASK); };
  auto kmask_of = [&](int ib) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(info0 + ib * Info::BYTES + Info::OFF_KMASK);
    return p[0] | p[1] | p[2] | p[3];
  };
  auto tile_of = [&](int ib) { return *reinterpret_cast<const int32_t*>(info0 + ib * Info::BYTES + Info::OFF_TILE); };

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const unsigned long long deadline = 0;  // waits are bounded by a cycle count
  const int64_t n_row_tiles = (n_out + BMT - 1) / BMT;
  const int n_col_tiles = (c_out + TN - 1) / TN;
  const int64_t n_tiles = n_row_tiles * n_col_tiles;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(bar_full + 8 * s, NPROD / 32);  // one arrive per producer warp (+ weight bytes)
      tc::mbar_init(bar_empty + 8 * s, 1);
    }
    tc::mbar_init(bar_hfull, 1);           // warp 0 after issuing the halo gathers (+ halo bytes)
    tc::mbar_init(bar_hfree, NPROD / 32);  // every producer warp after its last copy of a tile
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar_ifull + 8 * b, NEPI);
      tc::mbar_init(bar_iempty + 8 * b, NPROD / 32 + 1);  // producer warps + MMA issuer
      tc::mbar_init(bar_afull + 8 * b, 1);
      tc::mbar_init(bar_aempty + 8 * b, NEPI);
      tc::mbar_init(bar_tidx + 8 * b, 1);
    }
    *s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 4) {
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ctrl_u32 + C::OFF_TMEM),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp < 4) {
    // =============================== producers ===============================
    int64_t gstep = 0;  // ring position (same sequence in every producer warp)
    const int sub = lane & 7;       // 16-byte chunk of a row this lane copies
    const int rsub = lane >> 3;     // row of a 4-row group this lane copies
    for (int it = 0;; ++it) {
      const int ib = it & 1;
      if (!__all_sync(kFullMask, tc::mbar_wait(bar_ifull + 8 * ib, (it >> 1) & 1, deadline, s_abort, status)))
        break;
      const int64_t t = tile_of(ib);
      if (t < 0) break;  // no more tiles for this CTA
      const int64_t row_tile = t / n_col_tiles;
      const int n0 = static_cast<int>(t - row_tile * n_col_tiles) * TN;
      const int64_t row0 = row_tile * BMT;
      unsigned rem = kmask_of(ib);
      const int steps = __popc(rem);
      int hc = 0;  // rows in this tile's halo
      if (steps > 0) {
        hc = __ldg(&halo_count[row_tile]);
        if (hc < 0 || hc > HALO) {
          if (lane == 0) raise_status(status, TSC_STATUS_INTERNAL);
          hc = 0;
        }
      }
      // ---- warp 0: the tile's halo, once every warp is done with the previous one
      if (warp == 0) {
        if (it > 0 && !__all_sync(kFullMask, tc::mbar_wait(bar_hfree, (it - 1) & 1, deadline, s_abort, status)))
          break;
        // all of the list's quads are loaded first (one memory latency), then
        // gathered: lane l takes quads l, l + 32, ...
        const int nq = (hc + 3) >> 2;
        const int4* hr = reinterpret_cast<const int4*>(halo_rows + row_tile * static_cast<int64_t>(HALO));
        int4 e[QPL];
#pragma unroll
        for (int r = 0; r < QPL; ++r) {
          const int q = r * 32 + lane;
          e[r] = q < nq ? __ldg(hr + q) : make_int4(-1, -1, -1, -1);
        }
        unsigned fetch = 0, bytes = 0;
        bool bad = false;
#pragma unroll
        for (int r = 0; r < QPL; ++r) {
          const int q = r * 32 + lane;
          const bool ok = e[r].x >= 0 && e[r].x < n_in && e[r].y >= 0 && e[r].y < n_in && e[r].z >= 0 &&
                          e[r].z < n_in && e[r].w >= 0 && e[r].w < n_in;
          bad |= q < nq && !ok;
          fetch |= (q < nq && ok ? 1u : 0u) << r;
          bytes += __popc(__ballot_sync(kFullMask, q < nq && ok)) * 4 * ROW_BYTES;
        }
        if (bad) raise_status(status, TSC_STATUS_INTERNAL);
        if (lane == 0) mbar_expect_tx(bar_hfull, bytes);
        __syncwarp();
#pragma unroll
        for (int r = 0; r < QPL; ++r)
          if (fetch >> r & 1)
            tcp::tma_gather4(halo_u32 + (r * 32 + lane) * 4 * ROW_BYTES, &tmap_f, 0, e[r].x, e[r].y, e[r].z,
                             e[r].w, bar_hfull);
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_hfull);
      }
      if (!__all_sync(kFullMask, tc::mbar_wait(bar_hfull, it & 1, deadline, s_abort, status))) break;

      // halo-map entries of this warp's 64 rows at offset k: lane l holds rows
      // 64w+l (a) and 64w+32+l (b)
      const int64_t ra = row0 + warp * 64 + lane;
      auto load_ids = [&](int k, int& a, int& b) {
        const int64_t base = static_cast<int64_t>(k) * n_out;
        a = ra < n_out ? static_cast<int>(__ldg(&hmap[base + ra])) : kNoPair;
        b = ra + 32 < n_out ? static_cast<int>(__ldg(&hmap[base + ra + 32])) : kNoPair;
      };
      int k = 0, ida = kNoPair, idb = kNoPair;
      if (steps > 0) {
        k = __ffs(rem) - 1;
        rem &= rem - 1;
        load_ids(k, ida, idb);
      }
      bool alive = true;
      for (int s = 0; s < steps; ++s, ++gstep) {
        // next offset's entries, loaded under this step's copies
        int kn = k, na = kNoPair, nb = kNoPair;
        if (s + 1 < steps) {
          kn = __ffs(rem) - 1;
          rem &= rem - 1;
          load_ids(kn, na, nb);
        }
        const int stage = static_cast<int>(gstep % NS);
        const int64_t fill = gstep / NS;
        if (fill > 0 && !__all_sync(kFullMask, tc::mbar_wait(bar_empty + 8 * stage,
                                                              static_cast<uint32_t>((fill - 1) & 1), deadline,
                                                              s_abort, status))) {
          alive = false;
          break;
        }
        const uint32_t sa = ring_u32 + stage * C::STAGE;
        const uint32_t full = bar_full + 8 * stage;
        if (warp == 0 && lane == 0) {
          if (k < K && n0 + TN <= c_out) {
            mbar_expect_tx(full, C::B_BYTES);
            tcp::tma_load_3d(sa + C::A_BYTES, &tmap_w, 0, k, n0, full);
          } else {
            raise_status(status, TSC_STATUS_INTERNAL);
          }
        }
        // copy this warp's 64 rows at k: 4 rows per pass, 8 lanes per row,
        // all loads first, then all stores.  Every lane copies (a row
        // without a pair copies halo row 0; the MMA masks it off), so the
        // loop has no branches.  Rows outside the halo are then overwritten
        // from global memory.
        uint4 v[16];
        unsigned outside = 0;
        bool bad = false;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int id = __shfl_sync(kFullMask, i < 8 ? ida : idb, (4 * i + rsub) & 31);
          const bool in = id >= 0 && id < hc;
          outside |= (id == kOutsideHalo ? 1u : 0u) << i;
          bad |= id >= hc || id < kOutsideHalo;
          v[i] = lds128(halo_u32 + swz128(in ? id : 0, sub));
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) sts128(sa + swz128(warp * 64 + 4 * i + rsub, sub), v[i]);
        if (__any_sync(kFullMask, outside != 0)) {
#pragma unroll 1
          for (int i = 0; i < 16; ++i) {
            if (!(outside >> i & 1)) continue;
            const int j = 4 * i + rsub;
            const int g = __ldg(&gmap[static_cast<int64_t>(k) * n_out + row0 + warp * 64 + j]);
            if (g >= 0 && g < n_in)
              sts128(sa + swz128(warp * 64 + j, sub),
                     __ldg(reinterpret_cast<const uint4*>(F + static_cast<int64_t>(g) * KC) + sub));
            else
              bad = true;
          }
        }
        if (bad) raise_status(status, TSC_STATUS_INTERNAL);
        // generic-proxy stores -> visible to the tensor core's async proxy
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(full);
        k = kn;
        ida = na;
        idb = nb;
      }
      if (!alive) break;
      // this warp is done with the tile's halo and info block
      tc::fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(bar_hfree);
        tc::mbar_arrive(bar_iempty + 8 * ib);
      }
    }
    // the MMA issuer releases the last fill of each stage asynchronously:
    // collect those arrivals before the CTA may exit
    if (tid == 0 && !*s_abort) tc::drain_ring(bar_empty, NS, gstep, deadline, s_abort, status);
  } else if (warp == 4) {
    // ================================ MMA issuer ================================
    if (lane == 0) {
      constexpr uint32_t idesc = tc::instr_desc<T, TN>();
      int64_t gstep = 0;
      for (int it = 0;; ++it) {
        const int ib = it & 1;
        const int b = it % NACC;
        const int use = it / NACC;
        if (!tc::mbar_wait(bar_ifull + 8 * ib, (it >> 1) & 1, deadline, s_abort, status)) break;
        if (tile_of(ib) < 0) break;  // no more tiles for this CTA
        unsigned rem = kmask_of(ib);
        const int steps = __popc(rem);
        const uint32_t* lmask = lmask_of(ib);
        // accumulator buffer b is zeroed and drained (epilogue arrival #use)
        if (!tc::mbar_wait(bar_aempty + 8 * b, use & 1, deadline, s_abort, status)) break;
        tc::tc_fence_after();
        const uint32_t acc0 = tmem + static_cast<uint32_t>(b * 2 * TN);
        bool ok = true;
        for (int s = 0; s < steps; ++s, ++gstep) {
          const int k = __ffs(rem) - 1;
          rem &= rem - 1;
          const uint4 m0 = *reinterpret_cast<const uint4*>(lmask + (k * 2 + 0) * 4);
          const uint4 m1 = *reinterpret_cast<const uint4*>(lmask + (k * 2 + 1) * 4);
          const int stage = static_cast<int>(gstep % NS);
          if (!tc::mbar_wait(bar_full + 8 * stage, static_cast<uint32_t>((gstep / NS) & 1), deadline, s_abort,
                             status)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a_addr = ring_u32 + stage * C::STAGE;
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint4 m = h ? m1 : m0;
            if ((m.x & m.y & m.z & m.w) == kFullMask) continue;  // no pair in this half
#pragma unroll
            for (int kk = 0; kk < KC / 16; ++kk)
              tc::umma_f16_masked(acc0 + h * TN,
                                  tc::smem_desc<C::SWZ_MODE, C::SBO>(a_addr + h * (HALF * ROW_BYTES) + kk * 32),
                                  tc::smem_desc<C::SWZ_MODE, C::SBO>(b_addr + kk * 32), idesc, m.x, m.y, m.z, m.w);
          }
          tc::umma_commit(bar_empty + 8 * stage);
        }
        if (!ok) break;
        tc::umma_commit(bar_afull + 8 * b);
        tc::mbar_arrive(bar_iempty + 8 * ib);  // masks are read at issue
      }
    }
  } else {
    // ========================== epilogue and tile set-up ==========================
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int lrow = q * 32 + lane;
    const bool relu = (flags & TSC_CONV_RELU) != 0;
    int64_t n_ovf = 0;
    if (ovf != nullptr && meta != nullptr) {
      n_ovf = static_cast<int64_t>(__ldg(&meta[TSC_META_N_OVERFLOW]));
      if (n_ovf > ovf_cap) n_ovf = ovf_cap;
    }
    const bool bias_smem = n_col_tiles == 1;
    if (bias_smem) {
      for (int i = tid - EPI0; i < TN; i += NEPI)
        s_bias[i] = (bias != nullptr && i < c_out) ? to_f32(__ldg(&bias[i])) : 0.f;
      asm volatile("bar.sync 2, %0;" ::"r"(NEPI) : "memory");
    }

    // tile of this CTA's jt-th slot (dynamic through the tile counter, else
    // round robin); -1 = no more tiles
    auto grab = [&](int jt) -> int64_t {
      if (tile_counter == nullptr) {
        const int64_t t = blockIdx.x + static_cast<int64_t>(jt) * gridDim.x;
        return t < n_tiles ? t : -1;
      }
      if (warp == EPI0 / 32) {
        int64_t t = -1;
        if (lane == 0) {
          const unsigned v = atomicAdd(tile_counter, 1u);
          t = v < static_cast<uint64_t>(n_tiles) ? static_cast<int64_t>(v) : -1;
          s_tidx[jt & 1] = static_cast<int32_t>(t);
          tc::mbar_arrive(bar_tidx + 8 * (jt & 1));
        }
        return __shfl_sync(kFullMask, t, 0);
      }
      if (!__all_sync(kFullMask, tc::mbar_wait(bar_tidx + 8 * (jt & 1), (jt >> 1) & 1, deadline, s_abort, status)))
        return -1;
      return s_tidx[jt & 1];
    };

    // set-up of slot jt (tile t, or the end marker t = -1) into info block
    // jt & 1: output rows and per-offset masks of this warp's 2 x 32 rows
    auto setup = [&](int jt, int64_t t) {
      const int ib = jt & 1;
      if (t < 0) {
        if (lane == 0) {
          *reinterpret_cast<int32_t*>(info0 + ib * Info::BYTES + Info::OFF_TILE) = -1;
          reinterpret_cast<uint32_t*>(info0 + ib * Info::BYTES + Info::OFF_KMASK)[q] = 0u;
        }
        tc::mbar_arrive(bar_ifull + 8 * ib);
        return;
      }
      int32_t* orow = orow_of(ib);
      uint32_t* lmask = lmask_of(ib);
      const int64_t row_tile = t / n_col_tiles;
      unsigned act = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = lrow + h * HALF;
        const int64_t tr = row_tile * BMT + r;
        const bool row_ok = tr < n_out;
        orow[r] = row_ok ? static_cast<int>(tr) : -1;
        int hv[KMAX];
#pragma unroll
        for (int kk = 0; kk < KMAX; ++kk)
          hv[kk] = (kk < K && row_ok) ? static_cast<int>(__ldg(&hmap[static_cast<int64_t>(kk) * n_out + tr]))
                                      : kNoPair;
#pragma unroll
        for (int kk = 0; kk < KMAX; ++kk) {
          if (kk >= K) break;
          const int v = hv[kk];
          bool none = v == kNoPair;
          if (v < kOutsideHalo || v >= HALO) {
            raise_status(status, TSC_STATUS_INTERNAL);
            none = true;
          }
          const unsigned nm = __ballot_sync(kFullMask, none);
          if (lane == 0) lmask[(kk * 2 + h) * 4 + q] = nm;
          act |= (nm != kFullMask ? 1u : 0u) << kk;
        }
      }
      if (lane == 0) {
        reinterpret_cast<uint32_t*>(info0 + ib * Info::BYTES + Info::OFF_KMASK)[q] = act;
        *reinterpret_cast<int32_t*>(info0 + ib * Info::BYTES + Info::OFF_TILE) = static_cast<int32_t>(t);
      }
      tc::mbar_arrive(bar_ifull + 8 * ib);
    };

    for (int b = 0; b < NACC; ++b) {
      __syncwarp();
#pragma unroll 1
      for (int h = 0; h < 2; ++h)
#pragma unroll 1
        for (int c0 = 0; c0 < TN; c0 += 32)
          tc::tmem_st32_zero(tmem + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(b * 2 * TN + h * TN + c0));
    }
    tc::tmem_wait_st();
    int64_t tq0 = grab(0);
    setup(0, tq0);
    tc::tc_fence_before();
    for (int b = 0; b < NACC; ++b) tc::mbar_arrive(bar_aempty + 8 * b);
    int64_t tq1 = tq0 >= 0 ? grab(1) : -1;
    if (tq0 >= 0) setup(1, tq1);
    for (int it = 0;; ++it) {
      const int ib = it & 1;
      const int b = it % NACC;
      const int use = it / NACC;
      const int64_t t = ib ? tq1 : tq0;
      if (t < 0) break;
      const int64_t row_tile = t / n_col_tiles;
      const int n0 = static_cast<int>(t - row_tile * n_col_tiles) * TN;
      if (!__all_sync(kFullMask, tc::mbar_wait(bar_afull + 8 * b, use & 1, deadline, s_abort, status))) break;
      tc::tc_fence_after();
      const int32_t* orow = orow_of(ib);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int o = orow[h * HALF + lrow];
#pragma unroll 1
        for (int c0 = 0; c0 < TN; c0 += 32) {
          float v[32];
          __syncwarp();
          const uint32_t taddr =
              tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * 2 * TN + h * TN + c0);
          tc::tmem_ld32(taddr, v);
          tc::tmem_st32_zero(taddr);  // ready for the buffer's next tile
          if (o < 0 || n0 + c0 >= c_out) continue;
          for (int64_t e = 0; e < n_ovf; ++e) {
            if (__ldg(&ovf[3 * e + 1]) != o) continue;
            const int k = __ldg(&ovf[3 * e + 0]);
            const int j = __ldg(&ovf[3 * e + 2]);
            if (k < 0 || k >= K || j < 0 || j >= n_in) continue;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int n = n0 + c0 + i;
              if (n >= c_out) continue;
              const T* wrow = W + (static_cast<int64_t>(n) * K + k) * KC;
              const T* frow = F + static_cast<int64_t>(j) * KC;
              float s = 0.f;
              for (int c = 0; c < KC; ++c) s = fmaf(to_f32(frow[c]), to_f32(wrow[c]), s);
              v[i] += s;
            }
          }
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const int n = n0 + c0 + qq * 8;
            if (n >= c_out) break;
            union {
              uint4 u;
              T hv[8];
            } pk;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float x = v[qq * 8 + i];
              if (bias_smem)
                x += s_bias[n + i];
              else if (bias != nullptr)
                x += to_f32(__ldg(&bias[n + i]));
              if (relu) x = fmaxf(x, 0.f);
              pk.hv[i] = from_f32<T>(x);
            }
            *reinterpret_cast<uint4*>(out + static_cast<int64_t>(o) * c_out + n) = pk.u;
          }
        }
      }
      __syncwarp();
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_aempty + 8 * b);
      if (!__all_sync(kFullMask, tc::mbar_wait(bar_iempty + 8 * ib, (it >> 1) & 1, deadline, s_abort, status)))
        break;
      const int64_t tn = grab(it + 2);
      setup(it + 2, tn);
      if (ib)
        tq1 = tn;
      else
        tq0 = tn;
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

}  // namespace tch
}  // namespace tsc
