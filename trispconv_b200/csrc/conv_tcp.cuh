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

#include "conv_tc.cuh"

namespace tsc {
namespace tcp {

constexpr int BMT = 256;       // rows per tile
constexpr int HALF = 128;      // rows per UMMA
constexpr int NPROD = 128;     // producer threads
constexpr int NEPI = 128;      // epilogue threads
constexpr int NT = NPROD + 32 + NEPI;
constexpr int KMAX = 32;       // offsets per map (one 32-bit active mask)

template <int TN, int KC>
struct Cfg {
  static constexpr int NACC = (4 * TN <= 512) ? 2 : 1;
  static constexpr int TMEM_COLS = NACC * 2 * TN;  // 128, 256 or 512
  static constexpr int A_BYTES = BMT * KC * 2;
  static constexpr int B_BYTES = TN * KC * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int RING_TARGET = 168 * 1024;
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
  static constexpr int OFF_MASK = OFF_STEPS + 8;    // uint32
  static constexpr int CTRL = (OFF_MASK + 4 + 127) / 128 * 128;
  static constexpr int OROW = 2 * BMT * 4;          // out rows per accumulator buffer
  static constexpr int ROWS = KMAX * BMT * 4;       // gather rows of the tile being produced
  static constexpr int TOTAL = 1024 + PIPE + CTRL + OROW + ROWS;
  static constexpr int SWZ_MODE = KC == 64 ? 2 : (KC == 32 ? 4 : 6);
  static constexpr int SBO = 8 * KC * 2;
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <typename T, int TN, int KC>
__global__ void __launch_bounds__(NT, 1)
k_conv_tcp(const T* __restrict__ F, int64_t n_in, int c_in, const T* __restrict__ W,
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
  int32_t* s_orow = reinterpret_cast<int32_t*>(ctrl + C::CTRL);            // [2][BMT]
  int32_t* s_rows = reinterpret_cast<int32_t*>(ctrl + C::CTRL + C::OROW);  // [K][BMT]

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
      tc::mbar_init(bar_full + 8 * s, NPROD);
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
    int64_t gstep = 0;  // steps produced so far (ring position)
    int it = 0;
    bool alive = true;
    for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
      const int b = it % NACC;
      const int use = it / NACC;
      const int64_t row_tile = t / n_col_tiles;
      const int n0 = static_cast<int>(t - row_tile * n_col_tiles) * TN;
      // out rows of buffer b are free once the epilogue released tile it-NACC
      if (alive && use > 0) alive = tc::mbar_wait(bar_aempty + 8 * b, (use - 1) & 1, deadline, s_abort, status);
      // ---- stage this thread's two rows: out row ids + gather entries ----
      int o2[2];
      unsigned mask = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t tr = row_tile * BMT + tid + h * HALF;
        o2[h] = (alive && tr < n_out) ? (perm != nullptr ? __ldg(&perm[tr]) : static_cast<int>(tr)) : -1;
        if (alive) s_orow[b * BMT + tid + h * HALF] = o2[h];
      }
      for (int k0 = 0; k0 < K; k0 += 8) {
        int jj[8][2];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int k = k0 + q;
            int j = -1;
            if (k < K && o2[h] >= 0)
              j = gmap != nullptr ? __ldg(&gmap[static_cast<int64_t>(k) * n_out + o2[h]]) : o2[h];
            jj[q][h] = j;
          }
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int k = k0 + q;
          if (k >= K) break;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            int j = jj[q][h];
            if (j >= n_in) {
              raise_status(status, TSC_STATUS_KEY_RANGE);
              j = -1;
            }
            s_rows[k * BMT + tid + h * HALF] = j;
            if (j >= 0) mask |= 1u << k;
          }
        }
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
        unsigned char* sa = ring + stage * C::STAGE;
        unsigned char* sb = sa + C::A_BYTES;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = tid + h * HALF;
          const int j = s_rows[k * BMT + r];
          unsigned char* drow = sa + r * (KC * 2);
          const T* srow = F + static_cast<int64_t>(j < 0 ? 0 : j) * c_in;
#pragma unroll
          for (int q = 0; q < UPR; ++q) {
            const int c = c0 + q * 8;
            const bool valid = j >= 0 && c < c_in;
            mma::cp_async<16>(drow + (mma::swz<KC>(r, q) << 4), valid ? srow + c : F, valid);
          }
        }
        for (int u = tid; u < TN * UPR; u += NPROD) {
          const int nn = u / UPR;
          const int q = u - nn * UPR;
          const int c = c0 + q * 8;
          const int n = n0 + nn;
          const bool valid = n < c_out && c < c_in;
          mma::cp_async<16>(sb + nn * (KC * 2) + (mma::swz<KC>(nn, q) << 4),
                            valid ? W + (static_cast<int64_t>(n) * K + k) * c_in + c : W, valid);
        }
        tc::cp_arrive_noinc(bar_full + 8 * stage);
      }
      if (*s_abort) alive = false;
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
        if (use > 0 && !tc::mbar_wait(bar_aempty + 8 * b, (use - 1) & 1, deadline, s_abort, status)) break;
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
            const uint32_t acc = (s > 0 || kk > 0) ? 1u : 0u;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              tc::umma_f16(acc0 + h * TN,
                           tc::smem_desc<C::SWZ_MODE, C::SBO>(a_addr + h * (HALF * KC * 2) + kk * 32), bd,
                           idesc, acc);
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
      const int steps = s_steps[b];
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int o = s_orow[b * BMT + h * HALF + lrow];
#pragma unroll 1
        for (int c0 = 0; c0 < TN; c0 += 32) {
          float v[32];
          __syncwarp();
          if (steps > 0) {
            tc::tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * 2 * TN + h * TN + c0),
                          v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
          }
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
              if (bias != nullptr) x += to_f32(__ldg(&bias[n + i]));
              if (relu) x = fmaxf(x, 0.f);
              pk.hv[i] = from_f32<T>(x);
            }
            *reinterpret_cast<uint4*>(out + static_cast<int64_t>(o) * c_out + n) = pk.u;
          }
        }
      }
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
