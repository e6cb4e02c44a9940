// Persistent tcgen05 implicit GEMM with per-plane input halos and the A
// operand in tensor memory (sm_100a), for 3x3x3 kernels with 64 input
// channels on maps whose output rows are spatially ordered (the outputs of a
// strided map, and the submanifold maps built on them).
//
// Why: the TMA-gather kernel (conv_tcp.cuh) fetches an input row from L2 once
// per pair, ~11 times per row on a 3x3x3 submanifold map, and runs at the
// per-SM gather rate.  Here the 256 output rows of a tile are served from
// sub-halos: for each plane of the kernel (kz, 9 offsets) the distinct input
// rows the tile's pairs of that plane read, listed once per kernel map by
// tsc_tile_halo (halo.cu) in ascending row order.  A sub-halo (~300 rows on
// the config-3 maps, a third of the pairs it serves) is fetched once with TMA
// gather4 into a 128-byte-swizzled shared-memory buffer; two buffers let the
// plane after next load while the current one is used.  For every
// (offset, row) the A operand row is then copied from the sub-halo into
// tensor memory (ld.shared into registers, tcgen05.st), and the MMA reads A
// from tensor memory and the weight slice (B) from shared memory, so shared
// memory carries only the halo reads and B.
//
// Warp roles (448 threads, one CTA per SM, tiles dealt round robin):
//   warp 0      weight producer: per (tile, active offset) the KRSC slice
//               W[0:TN, k, 0:64] by one TMA tile load into a weight stage.
//   warp 1      MMA issuer: per step 2 halves x 4 tcgen05.mma (M=128, N=TN,
//               K=16) from the A stage in tensor memory and the weight
//               stage, with the per-row disable-output-lane mask of the
//               offset; commits free the stage and, per tile, fill an
//               accumulator.
//   warps 2-5   epilogue: tcgen05.ld of a finished accumulator, clear it for
//               reuse, bias, ReLU, 16-byte stores.
//   warps 6-13  assemblers, two per tensor-memory lane quadrant: warp w owns
//               lanes 32*(w%4)..+31 of half (w-6)/4, i.e. tile row
//               128*((w-6)/4) + 32*(w%4) + lane.  Per step each thread copies
//               its row's 128-byte input from the sub-halo (a row beyond the
//               halo capacity straight from global memory) into the A stage
//               and the warp publishes its rows without a pair as the MMA
//               lane mask.  They also load the sub-halos: once all eight
//               have read a plane's buffer, each lane issues the gather4 of
//               one quad of the sub-halo two planes ahead into it (the lists
//               are read one plane earlier, so no global load is waited on).
// Tensor memory: accumulators (2 x 2 x 64 or 1 x 2 x 128 columns) and four
// A stages of 64 columns (2 halves x 32 columns of packed fp16/bf16 pairs).
// All waits are bounded (tc::mbar_wait); no role uses a named barrier after
// the start.
#pragma once

#include <cuda.h>

#include "conv_tcp.cuh"

namespace tsc {
namespace tmh {

constexpr int BMT = 256;           // output rows per tile
constexpr int HALF = 128;          // rows per UMMA
constexpr int KC = 64;             // input channels: the UMMA K of one offset (4 x 16)
constexpr int PLANES = 3;          // kz planes of a 3x3x3 kernel
constexpr int KPG = 9;             // offsets per plane
constexpr int KVOL = PLANES * KPG;
constexpr int NHB = 2;             // sub-halo buffers
constexpr int ROW_BYTES = KC * 2;  // 128
constexpr int A_COLS = 2 * (KC / 2);  // tensor-memory columns of one A stage
constexpr int W_WGT = 0, W_MMA = 1, W_EPI0 = 2, W_ASM0 = 6;
constexpr int NASM = 8;            // assembler warps
constexpr int NWARPS = W_ASM0 + NASM;
constexpr int NT = NWARPS * 32;
constexpr int SMEM_MAX = 227 * 1024;
constexpr int16_t kNoPair = -1;
constexpr int16_t kOutsideHalo = -2;

// NS_ A (tensor memory) + weight (shared memory) stages; two accumulator
// buffers when they fit beside the stages in the 512 tensor-memory columns.
template <int TN, int NS_>
struct Cfg {
  static_assert(TN == 64 || TN == 128, "tile width");
  static constexpr int NS = NS_;
  static constexpr int TMEM_COLS = 512;
  static constexpr int NACC = 2 * 2 * TN + NS * A_COLS <= TMEM_COLS ? 2 : 1;
  static constexpr int A0 = NACC * 2 * TN;  // first A-stage column
  static_assert(A0 + NS * A_COLS <= TMEM_COLS, "tensor memory");
  static constexpr int HALO = TN == 64 ? 640 : 512;  // rows per sub-halo buffer
  static constexpr int HALO_BYTES = HALO * ROW_BYTES;
  static constexpr int W_BYTES = TN * KC * 2;
  static constexpr int OFF_HALO = 0;
  static constexpr int OFF_W = OFF_HALO + NHB * HALO_BYTES;
  static constexpr int OFF_MASK = OFF_W + NS * W_BYTES;  // uint32 [NS][half][quadrant]
  static constexpr int OFF_BIAS = OFF_MASK + NS * 8 * 4;  // float [TN]
  static constexpr int OFF_BAR = OFF_BIAS + TN * 4;
  // hfull[2] hempty[2] wfull[NS] afull[NS] sempty[NS] accfull[2] accempty[2]
  static constexpr int NBAR = 2 + 2 + 3 * NS + 2 + 2;
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  static constexpr int OFF_ABORT = OFF_TMEM + 4;
  static constexpr int TOTAL = 1024 /*alignment slack*/ + OFF_ABORT + 4;
  static_assert(OFF_W % 1024 == 0 && W_BYTES % 1024 == 0 && HALO_BYTES % 1024 == 0, "swizzle atoms");
  static_assert(OFF_BAR % 8 == 0, "barrier alignment");
  static_assert(TOTAL <= SMEM_MAX, "shared memory");
};

// tcgen05.mma with A in tensor memory (a_tmem: lane 0, first column of the
// 128 x 16 operand, two 16-bit elements per 32-bit column), B from shared
// memory, accumulate into d, rows whose bit is set in {m0..m3} unchanged.
__device__ __forceinline__ void umma_ts_masked(uint32_t d, uint32_t a_tmem, unsigned long long b, uint32_t idesc,
                                               uint32_t m0, uint32_t m1, uint32_t m2, uint32_t m3) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, 1, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%4, %5, %6, %7}, p; }"
      ::"r"(d), "r"(a_tmem), "l"(b), "r"(idesc), "r"(m0), "r"(m1), "r"(m2), "r"(m3)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// Sub-halo slots of one plane for the tile row o (kNoPair past n_out).
__device__ __forceinline__ void load_plane_slots(const int16_t* __restrict__ hmap, int64_t n_out, int64_t o,
                                                 int plane, int (&s)[KPG]) {
#pragma unroll
  for (int j = 0; j < KPG; ++j)
    s[j] = o < n_out ? __ldg(&hmap[static_cast<int64_t>(plane * KPG + j) * n_out + o]) : kNoPair;
}

// The quad of sub-halo rows (and the sub-halo's row count) one lane issues
// for plane sequence number hs of this CTA, or an empty quad past its tiles.
struct HaloQuad {
  int4 rows;
  int count;
};

__device__ __forceinline__ HaloQuad load_halo_quad(const int32_t* __restrict__ halo_rows,
                                                   const int32_t* __restrict__ halo_count, int cap,
                                                   int64_t n_tiles, int64_t hs, int qd) {
  HaloQuad h{make_int4(0, 0, 0, 0), 0};
  const int64_t t = blockIdx.x + (hs / PLANES) * static_cast<int64_t>(gridDim.x);
  if (t >= n_tiles) return h;
  const int64_t hp = t * PLANES + hs % PLANES;
  h.count = __ldg(&halo_count[hp]);
  if (4 * qd < h.count && 4 * qd + 3 < cap)
    h.rows = __ldg(reinterpret_cast<const int4*>(halo_rows + hp * static_cast<int64_t>(cap)) + qd);
  return h;
}

// GEN: the general store epilogue (folded BatchNorm, any activation);
// without it bias + optional ReLU in the shortest code.
template <typename T, int TN, int NS_, bool GEN>
__global__ void __launch_bounds__(NT, 1)
k_conv_tmh(const __grid_constant__ CUtensorMap tmap_f, const __grid_constant__ CUtensorMap tmap_w,
           const T* __restrict__ F, int64_t n_in, const T* __restrict__ bias, const int32_t* __restrict__ gmap,
           int64_t n_out, const int32_t* __restrict__ halo_rows, const int32_t* __restrict__ halo_count,
           const uint32_t* __restrict__ plane_kmask, const int16_t* __restrict__ hmap, int cap,
           T* __restrict__ out, int flags, EpiParams epi, int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  using C = Cfg<TN, NS_>;
  constexpr int NS = C::NS;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u32 = mma::smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_u32 & 1023u)) & 1023u;
  unsigned char* base = smem_raw + pad;
  const uint32_t base_u32 = raw_u32 + pad;
  uint32_t* s_mask = reinterpret_cast<uint32_t*>(base + C::OFF_MASK);
  float* s_bias = reinterpret_cast<float*>(base + C::OFF_BIAS);
  const uint32_t bar_hfull = base_u32 + C::OFF_BAR;
  const uint32_t bar_hempty = bar_hfull + 8 * NHB;
  const uint32_t bar_wfull = bar_hempty + 8 * NHB;
  const uint32_t bar_afull = bar_wfull + 8 * NS;
  const uint32_t bar_sempty = bar_afull + 8 * NS;
  const uint32_t bar_accfull = bar_sempty + 8 * NS;
  const uint32_t bar_accempty = bar_accfull + 16;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(base + C::OFF_TMEM);
  volatile int* s_abort = reinterpret_cast<volatile int*>(base + C::OFF_ABORT);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const unsigned long long deadline = 0;  // waits are bounded by a cycle count
  const int64_t n_tiles = (n_out + BMT - 1) / BMT;
  const int64_t n_planes = n_tiles > blockIdx.x ? ((n_tiles - 1 - blockIdx.x) / gridDim.x + 1) * PLANES : 0;

  if (tid == 0) {
    for (int b = 0; b < NHB; ++b) {
      tc::mbar_init(bar_hfull + 8 * b, NASM);   // one arrive.expect_tx per assembler warp
      tc::mbar_init(bar_hempty + 8 * b, NASM);  // one arrival per assembler warp
    }
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(bar_wfull + 8 * s, 1);
      tc::mbar_init(bar_afull + 8 * s, NASM);
      tc::mbar_init(bar_sempty + 8 * s, 1);  // tcgen05.commit
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar_accfull + 8 * b, 1);
      tc::mbar_init(bar_accempty + 8 * b, 4);  // one arrival per epilogue warp
    }
    *s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp >= W_EPI0 && warp < W_ASM0) {
    for (int i = tid - W_EPI0 * 32; i < TN; i += 4 * 32)
      s_bias[i] = epi.scale != nullptr ? __ldg(&epi.shift[i]) : bias != nullptr ? to_f32(__ldg(&bias[i])) : 0.f;
  }
  if (warp == W_MMA) {
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(base_u32 + C::OFF_TMEM),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == W_WGT) {
    // =========================== weight producer ===========================
    if (lane == 0) {
      int64_t g = 0;
      bool alive = true;
      for (int64_t t = blockIdx.x; t < n_tiles && alive; t += gridDim.x) {
        unsigned rem = (__ldg(&plane_kmask[t * PLANES]) | __ldg(&plane_kmask[t * PLANES + 1]) |
                        __ldg(&plane_kmask[t * PLANES + 2])) & ((1u << KVOL) - 1u);
        while (rem) {
          const int k = __ffs(rem) - 1;
          rem &= rem - 1;
          const int stage = static_cast<int>(g % NS);
          const int64_t fill = g / NS;
          if (fill > 0 && !tc::mbar_wait(bar_sempty + 8 * stage, static_cast<uint32_t>((fill - 1) & 1), deadline,
                                         s_abort, status)) {
            alive = false;
            break;
          }
          tcp::mbar_arrive_expect_tx(bar_wfull + 8 * stage, C::W_BYTES);
          tcp::tma_load_3d(base_u32 + C::OFF_W + stage * C::W_BYTES, &tmap_w, 0, k, 0, bar_wfull + 8 * stage);
          ++g;
        }
      }
      // the MMA issuer's commits release the stages asynchronously: collect
      // the last one of every stage before the CTA may exit
      if (alive && !*s_abort) tc::drain_ring(bar_sempty, NS, g, deadline, s_abort, status);
    }
  } else if (warp == W_MMA) {
    // ============================== MMA issuer ==============================
    if (lane == 0) {
      constexpr uint32_t idesc = tc::instr_desc<T, TN>();
      int64_t g = 0;
      int it = 0;
      bool alive = true;
      for (int64_t t = blockIdx.x; t < n_tiles && alive; t += gridDim.x, ++it) {
        unsigned rem = (__ldg(&plane_kmask[t * PLANES]) | __ldg(&plane_kmask[t * PLANES + 1]) |
                        __ldg(&plane_kmask[t * PLANES + 2])) & ((1u << KVOL) - 1u);
        const int b = it % C::NACC;
        const int use = it / C::NACC;
        if (!tc::mbar_wait(bar_accempty + 8 * b, use & 1, deadline, s_abort, status)) break;
        tc::tc_fence_after();
        const uint32_t acc0 = tmem + static_cast<uint32_t>(b * 2 * TN);
        while (rem) {
          rem &= rem - 1;
          const int stage = static_cast<int>(g % NS);
          const uint32_t par = static_cast<uint32_t>((g / NS) & 1);
          if (!tc::mbar_wait(bar_wfull + 8 * stage, par, deadline, s_abort, status) ||
              !tc::mbar_wait(bar_afull + 8 * stage, par, deadline, s_abort, status)) {
            alive = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t w_addr = base_u32 + C::OFF_W + stage * C::W_BYTES;
          const uint4 m0 = *reinterpret_cast<const uint4*>(s_mask + stage * 8);
          const uint4 m1 = *reinterpret_cast<const uint4*>(s_mask + stage * 8 + 4);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint4 m = h ? m1 : m0;
            if ((m.x & m.y & m.z & m.w) == kFullMask) continue;  // no pair in this half
            const uint32_t a_col = tmem + static_cast<uint32_t>(C::A0 + stage * A_COLS + h * (KC / 2));
#pragma unroll
            for (int kk = 0; kk < KC / 16; ++kk)
              umma_ts_masked(acc0 + h * TN, a_col + kk * 8, tc::smem_desc<2, 1024>(w_addr + kk * 32), idesc, m.x,
                             m.y, m.z, m.w);
          }
          tc::umma_commit(bar_sempty + 8 * stage);
          ++g;
        }
        if (!alive) break;
        tc::umma_commit(bar_accfull + 8 * b);
      }
    }
  } else if (warp < W_ASM0) {
    // =============================== epilogue ===============================
    const int q = warp & 3;
    const int lrow = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    // both accumulator buffers start at zero (the MMAs always accumulate)
    for (int b = 0; b < C::NACC; ++b)
#pragma unroll 1
      for (int c0 = 0; c0 < 2 * TN; c0 += 32)
        tc::tmem_st32_zero(tmem + lane_base + static_cast<uint32_t>(b * 2 * TN + c0));
    tc::tmem_wait_st();
    tc::tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < C::NACC; ++b) tc::mbar_arrive(bar_accempty + 8 * b);
    int it = 0;
    for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
      const int b = it % C::NACC;
      const int use = it / C::NACC;
      if (!__all_sync(kFullMask, tc::mbar_wait(bar_accfull + 8 * b, use & 1, deadline, s_abort, status))) break;
      tc::tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int64_t o = t * BMT + h * HALF + lrow;
#pragma unroll 1
        for (int c0 = 0; c0 < TN; c0 += 32) {
          float v[32];
          __syncwarp();
          const uint32_t taddr = tmem + lane_base + static_cast<uint32_t>(b * 2 * TN + h * TN + c0);
          tc::tmem_ld32(taddr, v);
          tc::tmem_st32_zero(taddr);  // ready for the buffer's next tile
          if (o >= n_out) continue;
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            union {
              uint4 u;
              T hv[8];
            } pk;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int n = c0 + qq * 8 + i;
              float x;
              if constexpr (GEN) {
                x = activate(epi.scale != nullptr ? fmaf(v[qq * 8 + i], __ldg(&epi.scale[n]), s_bias[n])
                                                  : v[qq * 8 + i] + s_bias[n],
                             epi.act, epi.alpha);
              } else {
                x = v[qq * 8 + i] + s_bias[n];
                if (epi.act == TSC_ACT_RELU) x = fmaxf(x, 0.f);
              }
              pk.hv[i] = from_f32<T>(x);
            }
            *reinterpret_cast<uint4*>(out + o * TN + c0 + qq * 8) = pk.u;
          }
        }
      }
      tc::tmem_wait_st();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_accempty + 8 * b);
    }
  } else {
    // ============================== assemblers ==============================
    const int a = warp - W_ASM0;             // 0 .. NASM-1
    const int q = warp & 3;                  // tensor-memory lane quadrant
    const int h = a >> 2;                    // half of the tile this warp builds
    const int r = h * HALF + q * 32 + lane;  // this thread's tile row
    const uint32_t a_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(C::A0 + h * (KC / 2));
    const int qd = a * 32 + lane;            // the sub-halo quad this lane loads
    static_assert(NASM * 32 * 4 >= C::HALO, "one quad per assembler lane covers a sub-halo");
    bool alive = true;

    // gather4 of this lane's quad of plane hs into halo buffer hs & 1; every
    // assembler warp arrives once per plane with the bytes of its quads
    auto issue = [&](int64_t hs, const HaloQuad& hq) {
      const int b = static_cast<int>(hs & 1);
      int cnt = hq.count;
      if (cnt < 0 || cnt > C::HALO || cnt > cap) {
        if (lane == 0 && a == 0) raise_status(status, TSC_STATUS_INTERNAL);
        cnt = 0;
      }
      const bool mine = 4 * qd < cnt;
      const unsigned quads = __ballot_sync(kFullMask, mine);
      if (lane == 0)
        tcp::mbar_arrive_expect_tx(bar_hfull + 8 * b, static_cast<uint32_t>(__popc(quads) * 4 * ROW_BYTES));
      __syncwarp();
      if (mine) {
        int4 rr = hq.rows;
        const bool in = rr.x >= 0 && rr.x < n_in && rr.y >= 0 && rr.y < n_in && rr.z >= 0 && rr.z < n_in &&
                        rr.w >= 0 && rr.w < n_in;
        if (!in) {  // never issue a coordinate outside the tensor
          raise_status(status, TSC_STATUS_INTERNAL);
          rr = make_int4(0, 0, 0, 0);
        }
        tcp::tma_gather4(base_u32 + C::OFF_HALO + b * C::HALO_BYTES + qd * (4 * ROW_BYTES), &tmap_f, 0, rr.x, rr.y,
                         rr.z, rr.w, bar_hfull + 8 * b);
      }
    };

    {
      const HaloQuad q0 = load_halo_quad(halo_rows, halo_count, cap, n_tiles, 0, qd);
      const HaloQuad q1 = load_halo_quad(halo_rows, halo_count, cap, n_tiles, 1, qd);
      if (n_planes > 0) issue(0, q0);
      if (n_planes > 1) issue(1, q1);
    }
    HaloQuad pend = load_halo_quad(halo_rows, halo_count, cap, n_tiles, 2, qd);  // plane hs + 2
    int cur[KPG], nxt[KPG];
    unsigned pk_cur = 0u, pk_nxt = 0u;
    uint32_t v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0u;
    if (n_planes > 0) {
      load_plane_slots(hmap, n_out, static_cast<int64_t>(blockIdx.x) * BMT + r, 0, cur);
      pk_cur = __ldg(&plane_kmask[static_cast<int64_t>(blockIdx.x) * PLANES]);
    }
    int64_t g = 0;
    for (int64_t hs = 0; hs < n_planes && alive; ++hs) {
      const int64_t t = blockIdx.x + (hs / PLANES) * static_cast<int64_t>(gridDim.x);
      const int p = static_cast<int>(hs % PLANES);
      const int b = static_cast<int>(hs & 1);
      // prefetch: the next plane's slots and offset mask, the quad of plane hs + 3
      if (hs + 1 < n_planes) {
        const int64_t t1 = blockIdx.x + ((hs + 1) / PLANES) * static_cast<int64_t>(gridDim.x);
        const int p1 = static_cast<int>((hs + 1) % PLANES);
        load_plane_slots(hmap, n_out, t1 * BMT + r, p1, nxt);
        pk_nxt = __ldg(&plane_kmask[t1 * PLANES + p1]);
      }
      const HaloQuad pend3 = load_halo_quad(halo_rows, halo_count, cap, n_tiles, hs + 3, qd);
      if (!__all_sync(kFullMask, tc::mbar_wait(bar_hfull + 8 * b, static_cast<uint32_t>((hs >> 1) & 1), deadline,
                                               s_abort, status))) {
        alive = false;
        break;
      }
      const uint32_t hb = base_u32 + C::OFF_HALO + b * C::HALO_BYTES;
      const int64_t o = t * BMT + r;
#pragma unroll
      for (int j = 0; j < KPG; ++j) {
        const int k = p * KPG + j;
        if (!((pk_cur >> k) & 1u)) continue;
        const int stage = static_cast<int>(g % NS);
        const int64_t fill = g / NS;
        if (fill > 0 && !__all_sync(kFullMask, tc::mbar_wait(bar_sempty + 8 * stage,
                                                             static_cast<uint32_t>((fill - 1) & 1), deadline,
                                                             s_abort, status))) {
          alive = false;
          break;
        }
        tc::tc_fence_after();
        const int slot = cur[j];
        bool has = false;
        if (slot >= 0 && slot < C::HALO) {
          const uint32_t src = hb + static_cast<uint32_t>(slot) * ROW_BYTES;
          const uint32_t sw = static_cast<uint32_t>(slot & 7);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 x = lds128(src + ((static_cast<uint32_t>(c) ^ sw) << 4));
            v[4 * c + 0] = x.x;
            v[4 * c + 1] = x.y;
            v[4 * c + 2] = x.z;
            v[4 * c + 3] = x.w;
          }
          has = true;
        } else if (slot == kOutsideHalo) {
          // a row beyond the sub-halo's capacity: read it from global memory
          const int jr = o < n_out ? __ldg(&gmap[static_cast<int64_t>(k) * n_out + o]) : -1;
          if (jr >= 0 && jr < n_in) {
            const uint4* src = reinterpret_cast<const uint4*>(F + static_cast<int64_t>(jr) * KC);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint4 x = __ldg(src + c);
              v[4 * c + 0] = x.x;
              v[4 * c + 1] = x.y;
              v[4 * c + 2] = x.z;
              v[4 * c + 3] = x.w;
            }
            has = true;
          } else {
            raise_status(status, TSC_STATUS_INTERNAL);
          }
        } else if (slot != kNoPair) {
          raise_status(status, TSC_STATUS_INTERNAL);
        }
        // rows without a pair store whatever the registers hold: the MMA
        // leaves their accumulator rows unchanged
        tmem_st32(a_base + static_cast<uint32_t>(stage * A_COLS), v);
        const unsigned none = __ballot_sync(kFullMask, !has);
        if (lane == 0) s_mask[stage * 8 + h * 4 + q] = none;
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_afull + 8 * stage);
        ++g;
      }
      if (!alive) break;
      // this plane's sub-halo has been read by this warp; once all assembler
      // warps have, the buffer takes the sub-halo of plane hs + 2
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_hempty + 8 * b);
      if (hs + 2 < n_planes) {
        if (!__all_sync(kFullMask, tc::mbar_wait(bar_hempty + 8 * b, static_cast<uint32_t>((hs >> 1) & 1), deadline,
                                                 s_abort, status))) {
          alive = false;
          break;
        }
        issue(hs + 2, pend);
      }
      pend = pend3;
#pragma unroll
      for (int j = 0; j < KPG; ++j) cur[j] = nxt[j];
      pk_cur = pk_nxt;
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == W_MMA) {
    __syncwarp();
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

}  // namespace tmh
}  // namespace tsc
