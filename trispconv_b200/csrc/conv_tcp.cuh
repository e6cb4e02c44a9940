// Persistent tcgen05 implicit GEMM for sparse convolution (sm_100a).
//
// One CTA per SM walks a strided list of tiles.  A tile is 256 output rows
// x TN output channels, computed as two UMMA M=128 halves that share every
// weight stage.  Warp roles (288 threads):
//   warps 0-3  producers, TMA only.  For every (active offset k, channel
//              chunk) step of a tile, lanes 0-15 of warp w each cover one
//              quad of tile rows 64w+4l..+3: a quad with at least one pair is
//              fetched with one TMA gather4 (rows without a pair inside it
//              repeat a valid row of the quad and are masked off in the MMA);
//              a quad without pairs is not fetched at all.  Warp 0 also loads
//              the weight slice W[n0:n0+TN, k, chunk] with a TMA tile load.
//              No TMA coordinate ever lies outside its tensor.
//   warp 4     one thread issues tcgen05.mma (M=128, N=TN, K=16) for both
//              halves into a TMEM accumulator, with the per-row
//              disable-output-lane mask of the offset; halves without any
//              pair are skipped.  tcgen05.commit frees the stage and, after
//              the tile, signals acc_full[b].
//   warps 5-8  epilogue and tile set-up.  Warp w owns TMEM lanes
//              32*(w%4)..+31 of both halves (tile rows q*32+lane and
//              128+q*32+lane, q = w%4).  For each finished tile it reads the
//              accumulator (tcgen05.ld), clears it for reuse, adds overflow
//              pairs and bias, applies ReLU and stores 16-byte vectors.  It
//              then prepares the tile two ahead: output rows, validated
//              gather entries, per-offset lane masks and active offsets, in a
//              double-buffered "tile info" block.  Set-up thus runs under the
//              MMAs of the current tile instead of stalling the producers.
// Two accumulator buffers (when 4*TN <= 512 TMEM columns) let the epilogue of
// one tile run under the MMAs of the next.  All mbarrier waits are bounded;
// no role uses a named barrier after the start, so a role that gives up
// cannot strand the others.
#pragma once

#include <cuda.h>

#include "conv_tc.cuh"

namespace tsc {
namespace tcp {

constexpr int BMT = 256;       // rows per tile
constexpr int HALF = 128;      // rows per UMMA
constexpr int NPROD = 128;     // producer threads (warps 0-3)
constexpr int NEPI = 128;      // epilogue threads (warps 5-8)
constexpr int EPI0 = NPROD + 32;
constexpr int NT = NPROD + 32 + NEPI;
constexpr int KMAX = 27;       // offsets per map (3x3x3 and smaller; 32-bit active mask)
constexpr int SMEM_MAX = 227 * 1024;

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// TMA gather of 4 feature rows y0..y3 (all inside the tensor) x box-width
// channels starting at channel x, into 4 consecutive swizzled rows at dst.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* tmap, int x, int y0, int y1, int y2,
                                            int y3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(bar)
      : "memory");
}

// TMA tile load of the weight slice W[z:z+TN, y, x:x+KC] (KRSC viewed as a
// 3-D tensor {C_in, K, C_out}); the launcher guarantees the box lies inside.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* tmap, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// Per-tile information block, double-buffered (tile parity).
struct Info {
  static constexpr int ROWS = KMAX * BMT * 4;      // int32 gather entry [k][row], -1 = no pair
  static constexpr int OROW = BMT * 4;             // int32 output row, -1 past the end
  static constexpr int LMASK = KMAX * 2 * 4 * 4;   // uint32 [k][half][word]: rows WITHOUT a pair
  static constexpr int KMASK = 4 * 4;              // uint32 [epilogue warp]: active offsets, OR them
  static constexpr int OFF_ROWS = 0;
  static constexpr int OFF_OROW = OFF_ROWS + ROWS;
  static constexpr int OFF_LMASK = OFF_OROW + OROW;
  static constexpr int OFF_KMASK = OFF_LMASK + LMASK;
  static constexpr int OFF_TILE = OFF_KMASK + KMASK;  // int32 tile index, -1 = no more tiles
  static constexpr int BYTES = (OFF_TILE + 4 + 127) / 128 * 128;
};

template <int TN, int KC>
struct Cfg {
  static_assert(TN >= 32 && (KC == 32 || KC == 64), "persistent kernel tile shape");
  static constexpr int NACC = (4 * TN <= 512) ? 2 : 1;
  static constexpr int TMEM_COLS = NACC * 2 * TN;  // 128, 256 or 512
  static constexpr int A_BYTES = BMT * KC * 2;
  static constexpr int B_BYTES = TN * KC * 2;
  // stages start on 1024-byte boundaries (swizzle atoms are address based)
  static constexpr int STAGE = (A_BYTES + B_BYTES + 1023) / 1024 * 1024;
  // control block: full[NS], empty[NS], ifull[2], iempty[2], afull[2],
  // aempty[2], tidx[2], tmem addr, abort, tile index hand-off[2]
  static constexpr int CTRL_MAX = 16 * 16 + 80 + 16;
  static constexpr int BIAS = 256 * 4;
  static constexpr int FIXED = 1024 /*alignment slack*/ + 2 * Info::BYTES + BIAS + (CTRL_MAX + 127) / 128 * 128;
  static constexpr int NS_FIT = (SMEM_MAX - FIXED) / STAGE;
  static constexpr int NS = NS_FIT > 16 ? 16 : NS_FIT;
  static_assert(NS >= 2, "tile configuration does not fit shared memory");
  static constexpr int PIPE = NS * STAGE;
  static constexpr int OFF_EMPTY = 8 * NS;
  static constexpr int OFF_IFULL = 16 * NS;
  static constexpr int OFF_IEMPTY = OFF_IFULL + 16;
  static constexpr int OFF_AFULL = OFF_IEMPTY + 16;
  static constexpr int OFF_AEMPTY = OFF_AFULL + 16;
  static constexpr int OFF_TIDXB = OFF_AEMPTY + 16;
  static constexpr int OFF_TMEM = OFF_TIDXB + 16;
  static constexpr int OFF_ABORT = OFF_TMEM + 4;
  static constexpr int OFF_TIDX = OFF_ABORT + 4;    // int32[2]
  static constexpr int CTRL = (OFF_TIDX + 8 + 127) / 128 * 128;
  static_assert(CTRL <= (CTRL_MAX + 127) / 128 * 128, "control block");
  static constexpr int OFF_INFO = PIPE + CTRL;         // from the ring base
  static constexpr int OFF_BIAS = OFF_INFO + 2 * Info::BYTES;
  static constexpr int TOTAL = 1024 + OFF_BIAS + BIAS;
  static_assert(TOTAL <= SMEM_MAX, "shared memory");
  static constexpr int SWZ_MODE = KC == 64 ? 2 : (KC == 32 ? 4 : 6);
  static constexpr int SBO = 8 * KC * 2;
};

// GEN: the general store epilogue (folded BatchNorm scale/shift, any
// activation); without it the store adds the bias and applies an optional
// ReLU, the common case, in the shortest code.
template <typename T, int TN, int KC, bool GEN>
__global__ void __launch_bounds__(NT, 1)
k_conv_tcp(const __grid_constant__ CUtensorMap tmap_f, const __grid_constant__ CUtensorMap tmap_w,
           const T* __restrict__ F, int64_t n_in, int c_in, const T* __restrict__ W,
           const T* __restrict__ bias, const int32_t* __restrict__ gmap, const int32_t* __restrict__ perm, int K,
           int64_t n_out, int c_out, const int32_t* __restrict__ ovf, int64_t ovf_cap,
           const int64_t* __restrict__ meta, T* __restrict__ out, int flags, EpiParams epi, int64_t* __restrict__ status,
           unsigned* __restrict__ tile_counter) {
  pdl_wait();
  pdl_trigger();
  using C = Cfg<TN, KC>;
  constexpr int NS = C::NS;
  constexpr int NACC = C::NACC;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u32 = mma::smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_u32 & 1023u)) & 1023u;
  unsigned char* ring = smem_raw + pad;
  const uint32_t ring_u32 = raw_u32 + pad;
  unsigned char* ctrl = ring + C::PIPE;
  const uint32_t ctrl_u32 = ring_u32 + C::PIPE;
  const uint32_t bar_full = ctrl_u32;
  const uint32_t bar_empty = ctrl_u32 + C::OFF_EMPTY;
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
  auto rows_of = [&](int ib) { return reinterpret_cast<int32_t*>(info0 + ib * Info::BYTES + Info::OFF_ROWS); };
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
  const int n_chunks = c_in / KC;  // the launcher guarantees c_in % KC == 0

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(bar_full + 8 * s, NPROD / 32);  // one arrive.expect_tx per producer warp
      tc::mbar_init(bar_empty + 8 * s, 1);
    }
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

  if (flags & TSC_CONV_TEST_WAIT_TIMEOUT) {
    // Testing the bounded waits: with TMEM held and nothing issued, one
    // thread waits with a short limit on the accumulator-full barrier of
    // buffer 0, which no role arrives at (no MMA was issued).  The wait runs
    // out, sets TSC_STATUS_WAIT_TIMEOUT and the abort flag, and every thread
    // goes to the teardown below, which frees TMEM.  No copy or MMA is in
    // flight at any point.
    if (tid == EPI0) tc::mbar_wait(bar_afull, 0u, deadline, s_abort, status, tc::kTestWaitCycles);
  } else if (warp < 4) {
    // =============================== producers ===============================
    int64_t gstep = 0;  // ring position (same sequence in every producer warp)
    for (int it = 0;; ++it) {
      const int ib = it & 1;
      const bool ok = __all_sync(kFullMask, tc::mbar_wait(bar_ifull + 8 * ib, (it >> 1) & 1, deadline, s_abort,
                                                          status));
      if (!ok) break;
      const int64_t t = tile_of(ib);
      if (t < 0) break;  // no more tiles for this CTA
      const int64_t row_tile = t / n_col_tiles;
      const int n0 = static_cast<int>(t - row_tile * n_col_tiles) * TN;
      const int32_t* rows = rows_of(ib);
      unsigned rem = kmask_of(ib);
      const int steps = __popc(rem) * n_chunks;
      int k = 0;
      bool alive = true;
      for (int s = 0; s < steps; ++s, ++gstep) {
        const int chunk = s % n_chunks;
        if (chunk == 0) {
          k = __ffs(rem) - 1;
          rem &= rem - 1;
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
        // this lane's quad of tile rows; rows without a pair repeat the
        // quad's first valid row (masked off in the MMA)
        const int r = warp * 64 + (lane & 15) * 4;
        const int4 e = *reinterpret_cast<const int4*>(rows + k * BMT + r);
        const int first = e.x >= 0 ? e.x : (e.y >= 0 ? e.y : (e.z >= 0 ? e.z : e.w));
        // every coordinate handed to the TMA lies inside its tensor (the
        // set-up validated the entries; a violation is reported, not issued)
        const bool in_rows = e.x < n_in && e.y < n_in && e.z < n_in && e.w < n_in;
        const bool in_cols = (chunk + 1) * KC <= c_in;
        bool fetch = lane < 16 && first >= 0;
        if (fetch && !(in_rows && in_cols)) {
          raise_status(status, TSC_STATUS_INTERNAL);
          fetch = false;
        }
        const bool wload = warp == 0 && lane == 16;
        const bool w_ok = k < K && n0 + TN <= c_out && in_cols;
        if (wload && !w_ok) raise_status(status, TSC_STATUS_INTERNAL);
        const unsigned quads = __ballot_sync(kFullMask, fetch);
        const bool w_issue = __shfl_sync(kFullMask, w_ok, 16);
        if (lane == 0)
          mbar_arrive_expect_tx(full, __popc(quads) * 4 * KC * 2 + (warp == 0 && w_issue ? C::B_BYTES : 0));
        __syncwarp();
        if (fetch) {
          tma_gather4(sa + r * (KC * 2), &tmap_f, chunk * KC, e.x >= 0 ? e.x : first, e.y >= 0 ? e.y : first,
                      e.z >= 0 ? e.z : first, e.w >= 0 ? e.w : first, full);
        } else if (wload && w_ok) {
          tma_load_3d(sa + C::A_BYTES, &tmap_w, chunk * KC, k, n0, full);
        }
      }
      if (!alive) break;
      // this warp has read the tile's entries: release the info block
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_iempty + 8 * ib);
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
        const int steps = __popc(rem) * n_chunks;
        const uint32_t* lmask = lmask_of(ib);
        // accumulator buffer b is zeroed and drained (epilogue arrival #use)
        if (!tc::mbar_wait(bar_aempty + 8 * b, use & 1, deadline, s_abort, status)) break;
        tc::tc_fence_after();
        const uint32_t acc0 = tmem + static_cast<uint32_t>(b * 2 * TN);
        bool ok = true;
        int k = 0;
        uint4 m[2];
        for (int s = 0; s < steps; ++s, ++gstep) {
          if (s % n_chunks == 0) {
            k = __ffs(rem) - 1;
            rem &= rem - 1;
            m[0] = *reinterpret_cast<const uint4*>(lmask + (k * 2 + 0) * 4);
            m[1] = *reinterpret_cast<const uint4*>(lmask + (k * 2 + 1) * 4);
          }
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
            if ((m[h].x & m[h].y & m[h].z & m[h].w) == kFullMask) continue;  // no pair in this half
#pragma unroll
            for (int kk = 0; kk < KC / 16; ++kk)
              tc::umma_f16_masked(acc0 + h * TN,
                                  tc::smem_desc<C::SWZ_MODE, C::SBO>(a_addr + h * (HALF * KC * 2) + kk * 32),
                                  tc::smem_desc<C::SWZ_MODE, C::SBO>(b_addr + kk * 32), idesc, m[h].x, m[h].y,
                                  m[h].z, m[h].w);
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
    int64_t n_ovf = 0;
    if (ovf != nullptr && meta != nullptr) {
      n_ovf = static_cast<int64_t>(__ldg(&meta[TSC_META_N_OVERFLOW]));
      if (n_ovf > ovf_cap) n_ovf = ovf_cap;
    }
    // one column tile: the additive term of the store (bias, or the
    // epilogue's shift) is the same for every tile -> shared memory
    const bool bias_smem = n_col_tiles == 1;
    const bool relu = epi.act == TSC_ACT_RELU;
    if (bias_smem) {
      for (int i = tid - EPI0; i < TN; i += NEPI)
        s_bias[i] = i >= c_out                ? 0.f
                    : epi.scale != nullptr ? __ldg(&epi.shift[i])
                    : bias != nullptr      ? to_f32(__ldg(&bias[i]))
                                           : 0.f;
      asm volatile("bar.sync 2, %0;" ::"r"(NEPI) : "memory");
    }

    // The tile of this CTA's jt-th slot: with a tile counter, the first
    // epilogue warp takes the next tile index from it and hands it to the
    // other three through tidx[jt & 1]; without one, tiles are dealt round
    // robin.  -1 = no more tiles.
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

    // Tile set-up of slot jt (tile t, or the end marker t = -1) into info
    // block jt & 1: this warp's 2 x 32 rows.
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
      int32_t* rows = rows_of(ib);
      int32_t* orow = orow_of(ib);
      uint32_t* lmask = lmask_of(ib);
      const int64_t row_tile = t / n_col_tiles;
      unsigned act = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = lrow + h * HALF;
        const int64_t tr = row_tile * BMT + r;
        const int o = tr < n_out ? (perm != nullptr ? __ldg(&perm[tr]) : static_cast<int>(tr)) : -1;
        const bool row_ok = o >= 0 && o < n_out;
        if (o >= n_out) raise_status(status, TSC_STATUS_INTERNAL);
        orow[r] = row_ok ? o : -1;
        int32_t j[KMAX];
#pragma unroll
        for (int kk = 0; kk < KMAX; ++kk) {
          j[kk] = -1;
          if (kk < K && row_ok) j[kk] = gmap != nullptr ? __ldg(&gmap[static_cast<int64_t>(kk) * n_out + o]) : o;
        }
#pragma unroll
        for (int kk = 0; kk < KMAX; ++kk) {
          if (kk >= K) break;
          int v = j[kk];
          if (v >= n_in) {
            raise_status(status, TSC_STATUS_KEY_RANGE);
            v = -1;
          }
          if (v < 0) v = -1;
          rows[kk * BMT + r] = v;
          const unsigned none = __ballot_sync(kFullMask, v < 0);
          if (lane == 0) lmask[(kk * 2 + h) * 4 + q] = none;
          act |= (none != kFullMask ? 1u : 0u) << kk;
        }
      }
      if (lane == 0) {
        reinterpret_cast<uint32_t*>(info0 + ib * Info::BYTES + Info::OFF_KMASK)[q] = act;
        *reinterpret_cast<int32_t*>(info0 + ib * Info::BYTES + Info::OFF_TILE) = static_cast<int32_t>(t);
      }
      tc::mbar_arrive(bar_ifull + 8 * ib);
    };

    // zero both accumulator buffers (MMAs always accumulate), set up the first
    // tile, hand the buffers to the MMA issuer (arrival #0), then set up the
    // second tile while the first one runs
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
    int64_t tq0 = grab(0);  // tiles of info blocks 0 and 1
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
              const T* wrow = W + (static_cast<int64_t>(n) * K + k) * c_in;
              const T* frow = F + static_cast<int64_t>(j) * c_in;
              float s = 0.f;
              for (int c = 0; c < c_in; ++c) s = fmaf(to_f32(frow[c]), to_f32(wrow[c]), s);
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
              if constexpr (GEN) {
                if (!bias_smem)
                  x = epi_apply(x, n + i, epi, bias);
                else
                  x = activate(epi.scale != nullptr ? fmaf(x, __ldg(&epi.scale[n + i]), s_bias[n + i])
                                                    : x + s_bias[n + i],
                               epi.act, epi.alpha);
              } else {
                if (bias_smem)
                  x += s_bias[n + i];
                else if (bias != nullptr)
                  x += to_f32(__ldg(&bias[n + i]));
                if (relu) x = fmaxf(x, 0.f);
              }
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
      // prepare the tile two ahead in this info block once the producers and
      // the MMA issuer have released it
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

}  // namespace tcp
}  // namespace tsc
