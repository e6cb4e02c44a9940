// Register-gather implicit GEMM for layers with few input channels
// (C_in in {4, 8, 16, 32}, C_out in {16, 32, 64}, K <= 64 offsets).
//
// For such layers a gathered input row is 8-64 bytes and one kernel offset
// contributes at most 16 x 32 multiply-adds per output row, so staging the
// gathered rows in shared memory (cp.async or TMA) and synchronising the CTA
// per offset costs more than the arithmetic.  Here every lane loads the A
// fragment of mma.sync.m16n8k16 straight from global memory into registers:
//
// * The A fragment of lane (group g = lane/4, quad q = lane%4) holds, per
//   row, the k16 positions {2q, 2q+1, 2q+8, 2q+9}.  The K dimension of the
//   implicit GEMM (offset, channel) is permuted so that these four positions
//   are four CONSECUTIVE channels of one offset: one 8-byte load per row and
//   k16 block (one 16-byte load covering two blocks when C_in = 32).  The
//   B operand uses the same permutation, so the product is unchanged.
// * The weights of all offsets stay in shared memory in that fragment order
//   (one 16-byte ld.shared per lane gives the B registers of two n8 tiles).
// * Each warp owns 16*MT output rows.  It stages its rows' gather-map slice
//   in shared memory with batched loads, ORs the active offsets over the
//   warp, and walks only those; missing neighbours are zero registers and
//   cost no memory traffic.  G offsets are loaded before their MMAs run, so
//   each lane keeps 2*MT*G loads in flight.
// * No CTA barrier after the weight load: warps walk row blocks on their own
//   (persistent grid).  The epilogue adds the duplicate-coordinate overflow
//   pairs, applies the store epilogue in fp32 and writes 4-byte pairs.
#pragma once

#include "tsc_common.cuh"

namespace tsc {
namespace rg {

constexpr int KMAX = 64;

// k16 blocks of the implicit GEMM for K offsets
template <int CIN>
__host__ __device__ constexpr int n_blocks(int K) {
  return (K * CIN + 15) / 16;
}
// loop units: one feature load per row each (an offset when C_in >= 16,
// else one k16 block spanning 16 / C_in offsets)
template <int CIN>
__host__ __device__ constexpr int n_units(int K) {
  return CIN >= 16 ? K : n_blocks<CIN>(K);
}
template <int CIN>
constexpr int kBlocksPerUnit = CIN >= 16 ? CIN / 16 : 1;

// Offset and first channel of the four consecutive channels that lane quad q
// holds in k16 block b.
template <int CIN>
__host__ __device__ __forceinline__ int blk_off(int b, int q) {
  if constexpr (CIN == 32) return b >> 1;
  if constexpr (CIN == 16) return b;
  if constexpr (CIN == 8) return 2 * b + (q >> 1);
  return 4 * b + q;
}
template <int CIN>
__host__ __device__ __forceinline__ int blk_ch(int b, int q) {
  if constexpr (CIN == 32) return 8 * q + 4 * (b & 1);
  if constexpr (CIN == 16) return 4 * q;
  if constexpr (CIN == 8) return 4 * (q & 1);
  return 0;
}
// Offset and first channel of the per-row load of unit u (16 bytes at
// channel 8q for C_in = 32, 8 bytes otherwise).
template <int CIN>
__device__ __forceinline__ int unit_off(int u, int q) {
  return CIN >= 16 ? u : blk_off<CIN>(u, q);
}
template <int CIN>
__device__ __forceinline__ int unit_ch(int u, int q) {
  if constexpr (CIN == 32) return 8 * q;
  return blk_ch<CIN>(u, q);
}

// Units whose offsets have a pair in the warp's rows.
template <int CIN>
__device__ __forceinline__ unsigned long long unit_mask(unsigned long long omask, int K) {
  if constexpr (CIN >= 16) {
    return omask;
  } else {
    constexpr int OPU = 16 / CIN;  // offsets per unit
    constexpr unsigned long long GROUP = (1ull << OPU) - 1;
    unsigned long long um = 0;
    const int nu = n_units<CIN>(K);
    for (int u = 0; u < nu; ++u)
      if ((omask >> (u * OPU)) & GROUP) um |= 1ull << u;
    return um;
  }
}

template <int CIN>
struct Load;
template <>
struct Load<32> {
  using type = uint4;
};
template <>
struct Load<16> {
  using type = uint2;
};
template <>
struct Load<8> {
  using type = uint2;
};
template <>
struct Load<4> {
  using type = uint2;
};

__device__ __forceinline__ void zero(uint4& v) { v = make_uint4(0u, 0u, 0u, 0u); }
__device__ __forceinline__ void zero(uint2& v) { v = make_uint2(0u, 0u); }
__device__ __forceinline__ void ldg(uint4& v, const void* p) { v = __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ void ldg(uint2& v, const void* p) { v = __ldg(reinterpret_cast<const uint2*>(p)); }

// A registers {a0 (r0, lo), a1 (r1, lo), a2 (r0, hi), a3 (r1, hi)} of k16
// block bb of a unit from the two rows' loads.
__device__ __forceinline__ void afrag(uint32_t (&a)[4], const uint4& r0, const uint4& r1, int bb) {
  a[0] = bb == 0 ? r0.x : r0.z;
  a[1] = bb == 0 ? r1.x : r1.z;
  a[2] = bb == 0 ? r0.y : r0.w;
  a[3] = bb == 0 ? r1.y : r1.w;
}
__device__ __forceinline__ void afrag(uint32_t (&a)[4], const uint2& r0, const uint2& r1, int) {
  a[0] = r0.x;
  a[1] = r1.x;
  a[2] = r0.y;
  a[3] = r1.y;
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                 uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Shared memory: the resident weights, [n_blocks][TN/16][32 lanes] uint4.
template <int CIN, int TN>
struct Smem {
  static __host__ __device__ constexpr size_t bytes(int K) {
    return static_cast<size_t>(n_blocks<CIN>(K)) * (TN / 16) * 32 * 16;
  }
};

// Offsets per unit, and the lane's offset inside its unit (C_in < 16: the
// four lane quads read different offsets of one k16 block).
template <int CIN>
constexpr int kOffsetsPerUnit = CIN >= 16 ? 1 : 16 / CIN;
template <int CIN>
__device__ __forceinline__ int lane_off(int q) {
  if constexpr (CIN >= 16) return 0;
  if constexpr (CIN == 8) return q >> 1;
  return q;
}

// Gather-map entries of G units starting at u0 for the lane's 2*MT rows:
// mrow[mt][h] points at the row's entry for the lane's offset of unit 0
// (NULL for rows past n_out), a unit adds u * kOffsetsPerUnit * n_out.
// -1: no pair, the unit lies past the last one, or the lane's offset is past
// K.  ident: no gather map (K = 1 identity), the row index itself.
template <int CIN, int MT, int G>
__device__ __forceinline__ void load_rows(int (&j)[G][MT][2], const int32_t* const (&mrow)[MT][2],
                                          const int (&o)[MT][2], bool ident, int u0, int nu, int K,
                                          int64_t unit_stride, int loff) {
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int u = u0 + g;
    const bool ok = u < nu && (kOffsetsPerUnit<CIN> == 1 || u * kOffsetsPerUnit<CIN> + loff < K);
    const int64_t step = static_cast<int64_t>(u) * unit_stride;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        int v = -1;
        if (ok && mrow[mt][h] != nullptr) v = ident ? o[mt][h] : __ldg(mrow[mt][h] + step);
        j[g][mt][h] = v;
      }
  }
}

// One warp owns 16*MT output rows and TN/WN output channels; WN warps of a
// CTA share a row block (each loads its rows; the second load hits L1).
// MINB CTAs per SM bound the registers (65536 / (NT * MINB) per thread).
template <typename T, int CIN, int TN, int MT, int G, int NT, int WN, int MINB>
__global__ void __launch_bounds__(NT, MINB)
k_conv_rg(const T* __restrict__ F, int n_in, const T* __restrict__ W, const T* __restrict__ bias,
          const int32_t* __restrict__ gmap, const int32_t* __restrict__ perm, int K, int n_out,
          const int32_t* __restrict__ ovf, int64_t ovf_cap, const int64_t* __restrict__ meta, T* __restrict__ out,
          EpiParams epi, int64_t* __restrict__ status) {
  using LT = typename Load<CIN>::type;
  constexpr int TNW = TN / WN;  // channels of one warp
  constexpr int NF = TNW / 8;
  constexpr int RW = 16 * MT;
  constexpr int BPU = kBlocksPerUnit<CIN>;
  constexpr int GROUPS = NT / 32 / WN;  // row blocks a CTA works on at once
  static_assert(TNW % 16 == 0, "column split");

  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) unsigned char smem[];
  const int nb = n_blocks<CIN>(K);
  const int nu = n_units<CIN>(K);
  const uint4* s_w = reinterpret_cast<const uint4*>(smem);
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int grp = lane >> 2;
  const int q = lane & 3;
  const int wcol = warp % WN;

  // ---- resident weights in fragment order ----------------------------------
  // entry (b, nf2, l): {b0, b1} of n8 tile 2*nf2 and of tile 2*nf2 + 1 for
  // lane l, i.e. four consecutive channels of W[n][off] with n = nf*8 + l/4
  {
    uint4* w_out = reinterpret_cast<uint4*>(smem);
    for (int e = tid; e < nb * (TN / 16) * 32; e += NT) {
      const int l = e & 31;
      const int bn = e >> 5;
      const int b = bn / (TN / 16);
      const int nf2 = bn - b * (TN / 16);
      const int off = blk_off<CIN>(b, l & 3);
      const int ch = blk_ch<CIN>(b, l & 3);
      const int n = nf2 * 16 + (l >> 2);
      uint2 lo = make_uint2(0u, 0u), hi = make_uint2(0u, 0u);
      if (off < K) {
        lo = __ldg(reinterpret_cast<const uint2*>(W + (static_cast<int64_t>(n) * K + off) * CIN + ch));
        hi = __ldg(reinterpret_cast<const uint2*>(W + (static_cast<int64_t>(n + 8) * K + off) * CIN + ch));
      }
      w_out[e] = make_uint4(lo.x, lo.y, hi.x, hi.y);
    }
  }
  __syncthreads();

  int64_t n_ovf = 0;
  if (ovf != nullptr && meta != nullptr) {
    n_ovf = static_cast<int64_t>(__ldg(&meta[TSC_META_N_OVERFLOW]));
    if (n_ovf > ovf_cap) n_ovf = ovf_cap;
  }
  const T* Fq = F + unit_ch<CIN>(0, q);  // the lane's channel offset is the same for every unit
  const int loff = lane_off<CIN>(q);
  const int64_t unit_stride = static_cast<int64_t>(kOffsetsPerUnit<CIN>) * n_out;
  const bool ident = gmap == nullptr;
  // identity map: any non-NULL marker; load_rows never dereferences it
  const int32_t* const gmap_self = reinterpret_cast<const int32_t*>(out);
  const uint4* s_wc = s_w + (wcol * (TNW / 16)) * 32 + lane;
  const int n_blk = (n_out + RW - 1) / RW;
  const int stride = gridDim.x * GROUPS;
  for (int blk = blockIdx.x * GROUPS + warp / WN; blk < n_blk; blk += stride) {
    const int t0 = blk * RW;
    int o[MT][2];
    const int32_t* mrow[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = t0 + mt * 16 + h * 8 + grp;
        int ov = t < n_out ? (perm != nullptr ? __ldg(&perm[t]) : t) : -1;
        if (t < n_out && static_cast<unsigned>(ov) >= static_cast<unsigned>(n_out)) {
          raise_status(status, TSC_STATUS_INTERNAL);  // a row order that is not a permutation of the rows
          ov = -1;
        }
        o[mt][h] = ov;
        mrow[mt][h] = o[mt][h] < 0 ? nullptr
                      : (ident ? gmap_self : gmap + static_cast<int64_t>(loff) * n_out + o[mt][h]);
      }

    float acc[MT][NF][4];
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < NF; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

    bool bad = false;  // a gather index at or past n_in (a corrupt map)
    // loads and MMAs of the G units at u0 whose row indices are j
    auto process = [&](const int (&j)[G][MT][2], int u0) {
      LT av[G][MT][2];
      bool any[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        bool a = false;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int jj = j[g][mt][h];
            const bool v = static_cast<unsigned>(jj) < static_cast<unsigned>(n_in);
            bad |= jj >= n_in;
            if (v)
              ldg(av[g][mt][h], Fq + static_cast<int64_t>(jj) * CIN);
            else
              zero(av[g][mt][h]);
            a |= v;
          }
        any[g] = __any_sync(kFullMask, a);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        if (!any[g]) continue;  // warp-uniform
#pragma unroll
        for (int bb = 0; bb < BPU; ++bb) {
          const int b = (u0 + g) * BPU + bb;
          uint32_t af[MT][4];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) afrag(af[mt], av[g][mt][0], av[g][mt][1], bb);
#pragma unroll
          for (int nf2 = 0; nf2 < NF / 2; ++nf2) {
            const uint4 w = s_wc[(b * (TN / 16) + nf2) * 32];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              mma16816<T>(acc[mt][2 * nf2], af[mt], w.x, w.y);
              mma16816<T>(acc[mt][2 * nf2 + 1], af[mt], w.z, w.w);
            }
          }
        }
      }
    };

    // two row-index buffers: the next G units' indices load while this G
    // units' features load and multiply
    int ja[G][MT][2], jb[G][MT][2];
    load_rows<CIN, MT, G>(ja, mrow, o, ident, 0, nu, K, unit_stride, loff);
    for (int u0 = 0; u0 < nu; u0 += 2 * G) {
      if (u0 + G < nu) load_rows<CIN, MT, G>(jb, mrow, o, ident, u0 + G, nu, K, unit_stride, loff);
      process(ja, u0);
      if (u0 + G >= nu) break;
      if (u0 + 2 * G < nu) load_rows<CIN, MT, G>(ja, mrow, o, ident, u0 + 2 * G, nu, K, unit_stride, loff);
      process(jb, u0 + G);
    }
    if (__any_sync(kFullMask, bad) && lane == 0) raise_status(status, TSC_STATUS_KEY_RANGE);

    // ---- epilogue --------------------------------------------------------------
    const int n_base = wcol * TNW;
    // pairs that did not fit the gather map (duplicate input coordinates)
    for (int64_t e = 0; e < n_ovf; ++e) {
      const int k = __ldg(&ovf[3 * e + 0]);
      const int oo = __ldg(&ovf[3 * e + 1]);
      const int j = __ldg(&ovf[3 * e + 2]);
      if (k < 0 || k >= K || j < 0 || j >= n_in) continue;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (o[mt][h] != oo) continue;
          const T* frow = F + static_cast<int64_t>(j) * CIN;
#pragma unroll
          for (int nf = 0; nf < NF; ++nf)
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
              const T* wrow = W + (static_cast<int64_t>(n_base + nf * 8 + 2 * q + c2) * K + k) * CIN;
              float s = 0.f;
              for (int c = 0; c < CIN; ++c) s = fmaf(to_f32(frow[c]), to_f32(wrow[c]), s);
              acc[mt][nf][2 * h + c2] += s;
            }
        }
    }
    const bool simple = epi.scale == nullptr && epi.act <= TSC_ACT_RELU;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (o[mt][h] < 0) continue;
        uint32_t* dst = reinterpret_cast<uint32_t*>(out + static_cast<int64_t>(o[mt][h]) * TN + n_base);
#pragma unroll
        for (int nf = 0; nf < NF; ++nf) {
          const int n = n_base + nf * 8 + 2 * q;
          float v0 = acc[mt][nf][2 * h], v1 = acc[mt][nf][2 * h + 1];
          if (simple) {
            if (bias != nullptr) {
              v0 += to_f32(bias[n]);
              v1 += to_f32(bias[n + 1]);
            }
            if (epi.act == TSC_ACT_RELU) {
              v0 = fmaxf(v0, 0.f);
              v1 = fmaxf(v1, 0.f);
            }
          } else {
            v0 = epi_apply(v0, n, epi, bias);
            v1 = epi_apply(v1, n + 1, epi, bias);
          }
          dst[(nf * 8 + 2 * q) >> 1] = pack2<T>(v0, v1);
        }
      }
  }
}

}  // namespace rg
}  // namespace tsc
