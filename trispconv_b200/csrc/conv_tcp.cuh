// Persistent tcgen05 implicit GEMM for sparse convolution (sm_100a).
//
// One CTA per SM walks a strided list of tiles.  A tile is 256 output rows
// x TN output channels, computed as two UMMA M=128 halves that share every
// weight stage (half the weight traffic of 128-row tiles).  Warp roles
// (288 threads):
//   warps 0-3  producers.  Thread p owns tile rows p and p+128: it loads their
//              gather-map entries for all offsets (batched, one round trip),
//              the tile's active-offset mask is OR-reduced across producers,
//              and for every (active offset, channel chunk) step the thread
//              cp.async-gathers its two rows into the shared-memory ring
//              (rows without a pair zero-filled), together with its share of
//              the weight slice W[:, k, chunk]; the copy engine arrives on
//              full[stage] when the copies land (cp.async.mbarrier.arrive.noinc).
//   warp 4     one thread issues tcgen05.mma (M=128, N=TN, K=16) for both
//              halves into a TMEM accumulator buffer; tcgen05.commit frees the
//              stage (empty[stage]) and, after the tile, signals acc_full[b].
//   warps 5-8  epilogue: tcgen05.ld of the finished buffer (warp w reads TMEM
//              lanes 32*(w%4)..+31 of both halves), overflow pairs, bias,
//              ReLU, 16-byte stores; then acc_empty[b].
// Two accumulator buffers (when 4*TN <= 512 TMEM columns) let the epilogue of
// one tile run under the MMAs of the next.  All mbarrier waits are bounded.
#pragma once

#include <cuda.h>

#include "conv_tc.cuh"

namespace tsc {
namespace tcp {

constexpr int BMT = 256;       // rows per tile
constexpr int HALF = 128;      // rows per UMMA
constexpr int NPROD = 128;     // producer threads
constexpr int NEPI = 128;      // epilogue threads
constexpr int NT = NPROD + 32 + NEPI;
constexpr int KMAX = 27;       // offsets per map (3x3x3 and smaller; 32-bit active mask)

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(mma::smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// TMA gather of 4 feature rows (y0..y3; an out-of-range row index reads the
// zero fill) x box-width channels starting at channel x, into 4 consecutive
// swizzled shared-memory rows at dst.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* tmap, int x, int y0, int y1, int y2,
                                            int y3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(bar)
      : "memory");
}

// TMA tile load of the weight slice W[n0:n0+TN, k, c0:c0+KC] (KRSC viewed as
// a 3-D tensor {C_in, K, C_out}); out-of-range channels read the zero fill.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* tmap, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

template <int TN, int KC>
struct Cfg {
  static constexpr int NACC = (4 * TN <= 512) ? 2 : 1;
  static constexpr int TMEM_COLS = NACC * 2 * TN;  // 128, 256 or 512
  static constexpr int A_BYTES = BMT * KC * 2;
  static constexpr int B_BYTES = TN * KC * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int RING_TARGET = 160 * 1024;
  static constexpr int NS = RING_TARGET / STAGE > 16 ? 16 : (RING_TARGET / STAGE < 2 ? 2 : RING_TARGET / STAGE);
  static constexpr int PIPE = NS * STAGE;
  // control block: full[NS], empty[NS], tinfo_full[2], acc_full[2], acc_empty[2],
  // tmem addr, abort, steps[2], active mask scratch
  static constexpr int OFF_EMPTY = 8 * NS;
  static constexpr int OFF_TINFO = 16 * NS;
  static constexpr int OFF_AFULL = OFF_TINFO + 16;
  static constexpr int OFF_AEMPTY = OFF_AFULL + 16;
  static constexpr int OFF_TMEM = OFF_AEMPTY + 16;
  static constexpr int OFF_ABORT = OFF_TMEM + 4;
  static constexpr int OFF_STEPS = OFF_ABORT + 4;   // int[2]
  static constexpr int OFF_MASK = OFF_STEPS + 8;    // uint32 scratch for the OR reduction
  static constexpr int CTRL = (OFF_MASK + 4 + 127) / 128 * 128;
  static constexpr int OROW = 2 * BMT * 4;          // out rows per accumulator buffer
  static constexpr int BIAS = 256 * 4;              // fp32 bias of the column tile
  static constexpr int ROWS = 2 * KMAX * BMT * 4;   // gather rows, double-buffered
  static constexpr int TOTAL = 1024 + PIPE + CTRL + OROW + BIAS + ROWS;
  static constexpr int SWZ_MODE = KC == 64 ? 2 : (KC == 32 ? 4 : 6);
  static constexpr int SBO = 8 * KC * 2;
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <typename T, int TN, int KC>
__global__ void __launch_bounds__(NT, 1)
k_conv_tcp(const __grid_constant__ CUtensorMap tmap_f, const __grid_constant__ CUtensorMap tmap_w,
           const T* __restrict__ F, int64_t n_in, int c_in, const T* __restrict__ W,
           const T* __restrict__ bias, const int32_t* __restrict__ gmap, const int32_t* __restrict__ perm, int K,
           int64_t n_out, int c_out, const int32_t* __restrict__ ovf, int64_t ovf_cap,
           const int64_t* __restrict__ meta, T* __restrict__ out, int flags, int64_t* __restrict__ status) {
  using C = Cfg<TN, KC>;
  constexpr int NS = C::NS;
  constexpr int NACC = C::NACC;
  constexpr int UPR = KC * 2 / 16;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u32 = mma::smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_u32 & 1023u)) & 1023u;
  unsigned char* ring = smem_raw + pad;
  const uint32_t ring_u32 = raw_u32 + pad;
  unsigned char* ctrl = ring + C::PIPE;
  const uint32_t ctrl_u32 = ring_u32 + C::PIPE;
  const uint32_t bar_full = ctrl_u32;
  const uint32_t bar_empty = ctrl_u32 + C::OFF_EMPTY;
  const uint32_t bar_tinfo = ctrl_u32 + C::OFF_TINFO;
  const uint32_t bar_afull = ctrl_u32 + C::OFF_AFULL;
  const uint32_t bar_aempty = ctrl_u32 + C::OFF_AEMPTY;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(ctrl + C::OFF_TMEM);
  volatile int* s_abort = reinterpret_cast<volatile int*>(ctrl + C::OFF_ABORT);
  int* s_steps = reinterpret_cast<int*>(ctrl + C::OFF_STEPS);
  unsigned* s_mask = reinterpret_cast<unsigned*>(ctrl + C::OFF_MASK);
  int32_t* s_orow = reinterpret_cast<int32_t*>(ctrl + C::CTRL);                        // [2][BMT]
  float* s_bias = reinterpret_cast<float*>(ctrl + C::CTRL + C::OROW);                  // [TN]
  int32_t* s_rows = reinterpret_cast<int32_t*>(ctrl + C::CTRL + C::OROW + C::BIAS);    // [2][K][BMT]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const unsigned long long deadline = tc::globaltimer() + tc::kWaitNs;
  const int64_t n_row_tiles = (n_out + BMT - 1) / BMT;
  const int n_col_tiles = (c_out + TN - 1) / TN;
  const int64_t n_tiles = n_row_tiles * n_col_tiles;
  const int n_chunks = (c_in + KC - 1) / KC;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(bar_full + 8 * s, NPROD / 32);  // one arrive.expect_tx per producer warp
      tc::mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar_tinfo + 8 * b, NPROD);
      tc::mbar_init(bar_afull + 8 * b, 1);
      tc::mbar_init(bar_aempty + 8 * b, NEPI);
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
    // Control flow is collective across the 128 producers (named barriers):
    // a failed wait clears `alive`, after which the thread skips all work but
    // still reaches every barrier.
    //
    // Thread p owns tile rows p and p+128.  The gather entries of the NEXT
    // tile are copied with 4-byte cp.async into the other half of the
    // double-buffered rows table while this tile's steps are produced, so no
    // dependent global round trip separates two tiles.
    int64_t gstep = 0;  // steps produced so far (ring position)
    int it = 0;
    bool alive = true;
    auto out_rows = [&](int64_t t, int (&o)[2]) {
      const int64_t row_tile = t / n_col_tiles;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t tr = row_tile * BMT + tid + h * HALF;
        o[h] = (t < n_tiles && tr < n_out) ? (perm != nullptr ? __ldg(&perm[tr]) : static_cast<int>(tr)) : -1;
      }
    };
    auto prefetch_rows = [&](const int (&o)[2], int rb) {
      int32_t* dst = s_rows + rb * (K * BMT);
      for (int k = 0; k < K; ++k) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int32_t* d = dst + k * BMT + tid + h * HALF;
          if (o[h] >= 0 && gmap != nullptr)
            cp_async4(d, gmap + static_cast<int64_t>(k) * n_out + o[h]);
          else
            *d = o[h];  // identity map (K == 1), or -1 past the last row
        }
      }
      mma::cp_commit();
    };
    int o_cur[2], o_nxt[2];
    out_rows(blockIdx.x, o_cur);
    prefetch_rows(o_cur, 0);
    for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
      const int b = it % NACC;
      const int use = it / NACC;
      const int rb = it & 1;
      const int64_t row_tile = t / n_col_tiles;
      const int n0 = static_cast<int>(t - row_tile * n_col_tiles) * TN;
      // the other rows buffer held tile it-1, whose entries this thread has read
      out_rows(t + gridDim.x, o_nxt);
      prefetch_rows(o_nxt, rb ^ 1);
      tc::cp_wait_n<1>();  // this tile's entries (committed one tile earlier) have landed
      // buffer b (out rows, step count, offsets) is free once the epilogue
      // released its previous tile; the epilogue's first arrival marks the
      // freshly zeroed accumulator
      if (alive) alive = tc::mbar_wait(bar_aempty + 8 * b, use & 1, deadline, s_abort, status);
      int32_t* rows = s_rows + rb * (K * BMT);
      unsigned mask = 0;
      for (int k = 0; k < K; ++k) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int32_t* p = rows + k * BMT + tid + h * HALF;
          const int j = *p;
          if (j >= n_in) {
            raise_status(status, TSC_STATUS_KEY_RANGE);
            *p = -1;
          } else if (j >= 0) {
            mask |= 1u << k;
          }
        }
      }
      if (alive) {
#pragma unroll
        for (int h = 0; h < 2; ++h) s_orow[b * BMT + tid + h * HALF] = o_cur[h];
      }
      // ---- tile's active offsets: OR over the 128 producers -------------------
      mask = __reduce_or_sync(kFullMask, mask);
      if (tid == 0) *s_mask = 0;
      named_bar_sync(1, NPROD);
      if (lane == 0) atomicOr(s_mask, mask);
      named_bar_sync(1, NPROD);
      const unsigned kmask = *s_mask;
      const int steps = alive ? __popc(kmask) * n_chunks : 0;
      if (alive) {
        if (tid == 0) s_steps[b] = steps;
        tc::mbar_arrive(bar_tinfo + 8 * b);
      }
      // ---- steps -----------------------------------------------------------------
      unsigned rem = kmask;
      int k = 0;
      for (int s = 0; s < steps && alive; ++s, ++gstep) {
        const int chunk = s % n_chunks;
        if (chunk == 0) {
          k = __ffs(rem) - 1;
          rem &= rem - 1;
        }
        const int stage = static_cast<int>(gstep % NS);
        const int64_t fill = gstep / NS;
        if (fill > 0 && !tc::mbar_wait(bar_empty + 8 * stage, static_cast<uint32_t>((fill - 1) & 1), deadline,
                                       s_abort, status)) {
          alive = false;
          break;
        }
        const int c0 = chunk * KC;
        const uint32_t sa = ring_u32 + stage * C::STAGE;
        const uint32_t sb = sa + C::A_BYTES;
        const uint32_t full = bar_full + 8 * stage;
        // warp w gathers tile rows [64w, 64w+64): lanes 0-15 one 4-row TMA
        // gather each; warp 0 also loads the weight slice.  Row entries of
        // other producers are visible after the mask barriers.
        if (lane == 0) mbar_arrive_expect_tx(full, 64 * KC * 2 + (warp == 0 ? C::B_BYTES : 0));
        __syncwarp();
        if (lane < 16) {
          const int r = warp * 64 + lane * 4;
          const int32_t* e = rows + k * BMT + r;
          // rows without a pair use the out-of-range row index n_in: the TMA
          // unit fills them with zeros and reads no memory for them
          const int oob = static_cast<int>(n_in);
          const int y0 = e[0] >= 0 ? e[0] : oob;
          const int y1 = e[1] >= 0 ? e[1] : oob;
          const int y2 = e[2] >= 0 ? e[2] : oob;
          const int y3 = e[3] >= 0 ? e[3] : oob;
          tma_gather4(sa + r * (KC * 2), &tmap_f, c0, y0, y1, y2, y3, full);
        } else if (warp == 0 && lane == 16) {
          tma_load_3d(sb, &tmap_w, c0, k, n0, full);
        }
      }
      if (*s_abort) alive = false;
      o_cur[0] = o_nxt[0];
      o_cur[1] = o_nxt[1];
      // s_mask is reset at the start of the next tile: every producer must
      // have read it first
      named_bar_sync(1, NPROD);
    }
    tc::cp_wait_all();
  } else if (warp == 4) {
    // ================================ MMA issuer ================================
    if (lane == 0) {
      constexpr uint32_t idesc = tc::instr_desc<T, TN>();
      int64_t gstep = 0;
      int it = 0;
      for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
        const int b = it % NACC;
        const int use = it / NACC;
        if (!tc::mbar_wait(bar_tinfo + 8 * b, use & 1, deadline, s_abort, status)) break;
        const int steps = s_steps[b];
        // accumulator buffer b is zeroed and drained (epilogue arrival #use)
        if (!tc::mbar_wait(bar_aempty + 8 * b, use & 1, deadline, s_abort, status)) break;
        tc::tc_fence_after();
        const uint32_t acc0 = tmem + static_cast<uint32_t>(b * 2 * TN);
        bool ok = true;
        for (int s = 0; s < steps; ++s, ++gstep) {
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
          for (int kk = 0; kk < KC / 16; ++kk) {
            const unsigned long long bd = tc::smem_desc<C::SWZ_MODE, C::SBO>(b_addr + kk * 32);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              // the accumulator starts at zero (epilogue-cleared), so every MMA accumulates
              tc::umma_f16(acc0 + h * TN,
                           tc::smem_desc<C::SWZ_MODE, C::SBO>(a_addr + h * (HALF * KC * 2) + kk * 32), bd, idesc,
                           1u);
            }
          }
          tc::umma_commit(bar_empty + 8 * stage);
        }
        if (!ok) break;
        tc::umma_commit(bar_afull + 8 * b);
      }
    }
  } else {
    // ================================= epilogue =================================
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int lrow = q * 32 + lane;
    const bool relu = (flags & TSC_CONV_RELU) != 0;
    int64_t n_ovf = 0;
    if (ovf != nullptr && meta != nullptr) {
      n_ovf = static_cast<int64_t>(__ldg(&meta[TSC_META_N_OVERFLOW]));
      if (n_ovf > ovf_cap) n_ovf = ovf_cap;
    }
    // one column tile: the bias is the same for every tile -> shared memory
    const bool bias_smem = n_col_tiles == 1;
    if (bias_smem) {
      for (int i = tid - (NPROD + 32); i < TN; i += NEPI)
        s_bias[i] = (bias != nullptr && i < c_out) ? to_f32(__ldg(&bias[i])) : 0.f;
      named_bar_sync(2, NEPI);
    }
    // zero both accumulator buffers (MMAs always accumulate; rows without a
    // pair are masked off) and hand them to the MMA issuer: arrival #0
    for (int b = 0; b < NACC; ++b) {
      __syncwarp();
#pragma unroll 1
      for (int h = 0; h < 2; ++h)
#pragma unroll 1
        for (int c0 = 0; c0 < TN; c0 += 32)
          tc::tmem_st32_zero(tmem + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(b * 2 * TN + h * TN + c0));
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_aempty + 8 * b);
    }
    int it = 0;
    for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
      const int b = it % NACC;
      const int use = it / NACC;
      const int64_t row_tile = t / n_col_tiles;
      const int n0 = static_cast<int>(t - row_tile * n_col_tiles) * TN;
      const bool ok1 = tc::mbar_wait(bar_tinfo + 8 * b, use & 1, deadline, s_abort, status);
      const bool ok2 = ok1 && tc::mbar_wait(bar_afull + 8 * b, use & 1, deadline, s_abort, status);
      if (!__all_sync(kFullMask, ok2)) break;
      tc::tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int o = s_orow[b * BMT + h * HALF + lrow];
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
