// Warp-level tensor-core implicit GEMM (mma.sync m16n8k16, fp16/bf16 in,
// fp32 accumulate) for sparse convolution.
//
// One CTA owns BM = 128 output rows x TN output channels.  The gather map
// slice of the tile (K x 128 input rows) is staged in shared memory once;
// offsets with no pair in the tile are skipped.  For each remaining
// (offset k, input-channel chunk) step the gathered feature rows and the
// weight slice W[:, k, chunk] (KRSC, i.e. already "K-major" for the B
// operand) are copied with cp.async into a 4-stage ring of XOR-swizzled
// shared-memory tiles, then consumed with ldmatrix + mma.sync.  Rows whose
// gather index is -1 are zero-filled by the copy engine (src-size 0), so
// they cost no memory traffic.  The epilogue stages the fp32 tile in shared
// memory, adds the rare duplicate-coordinate overflow pairs, applies bias
// and ReLU, and writes 16-byte chunks of each output row.
#pragma once

#include "tsc_common.cuh"

namespace tsc {
namespace mma {

constexpr int BM = 128;
constexpr int NT = 256;
constexpr int NS = 4;
constexpr int KMAX = 64;  // kernel volumes handled by this path

// RB output rows per CTA (BM, or 2*BM to share each weight slice between
// more rows).
template <int TN, int KC, int RB = BM>
struct Cfg {
  static constexpr int A_BYTES = RB * KC * 2;
  static constexpr int B_BYTES = TN * KC * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int PIPE = NS * STAGE;
  static constexpr int OUT_LD = TN + 8;  // fp32 epilogue row stride
  static constexpr int EPI = RB * OUT_LD * 4;
  static constexpr int MAIN = PIPE > EPI ? PIPE : EPI;
  // rows [K][RB] int32 + out rows [RB] + active list [KMAX] + misc[8]
  static constexpr int TOTAL = MAIN + (KMAX * RB + RB + KMAX + 8) * 4;  // K = KMAX upper bound
  static constexpr int bytes(int K) { return MAIN + (K * RB + RB + KMAX + 8) * 4; }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

template <int CH>
__device__ __forceinline__ void cp_async(void* dst, const void* src, bool valid) {
  const uint32_t d = smem_u32(dst);
  const int sz = valid ? CH : 0;
  if constexpr (CH == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(sz));
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d), "l"(src), "r"(sz));
  }
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }

template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
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

// XOR swizzle of 16-byte chunks inside a shared-memory row of KC halves so
// that the 8 rows an ldmatrix phase touches land in 8 distinct bank groups.
template <int KC>
__device__ __forceinline__ int swz(int row, int chunk) {
  constexpr int C = KC * 2 / 16;  // chunks per row: 2, 4 or 8
  return chunk ^ ((row / (8 / C)) % C);
}

template <typename T, int TN, int KC, int CH, int RB = BM>
__global__ void __launch_bounds__(NT)
k_conv_mma(const T* __restrict__ F, int64_t n_in, int c_in, const T* __restrict__ W,
           const T* __restrict__ bias, const int32_t* __restrict__ gmap, const int32_t* __restrict__ perm,
           int K, int64_t n_out, int c_out, const int32_t* __restrict__ ovf, int64_t ovf_cap,
           const int64_t* __restrict__ meta, T* __restrict__ out, int flags, EpiParams epi, int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  using C = Cfg<TN, KC, RB>;
  static_assert(RB <= NT && RB % BM == 0, "rows per CTA");
  constexpr int WN = (TN == 128) ? 2 : 1;
  constexpr int WM = 8 / WN;
  constexpr int WTM = RB / WM;
  constexpr int WTN = TN / WN;
  constexpr int MF = WTM / 16;
  constexpr int NF = WTN / 8;
  constexpr int UPR = KC * 2 / CH;  // copy units per shared-memory row
  static_assert(NF % 2 == 0, "B fragments are loaded in pairs");

  extern __shared__ __align__(128) unsigned char smem[];
  int32_t* s_rows = reinterpret_cast<int32_t*>(smem + C::MAIN);  // [K][RB]
  int32_t* s_orow = s_rows + K * RB;                              // [RB] output row ids (-1 = none)
  int32_t* s_klist = s_orow + RB;                                 // active offsets
  int32_t* s_misc = s_klist + KMAX;                               // [0] n_active, [1] hit row

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t tile0 = static_cast<int64_t>(blockIdx.x) * RB;
  const int n0 = blockIdx.y * TN;

  // ---- stage the tile's output rows and gather-map slice ------------------
  if (tid < KMAX) s_klist[tid] = 0;  // used as per-offset "any pair" flags first
  if (tid < RB) {
    const int64_t t = tile0 + tid;
    int32_t ov = t < n_out ? (perm != nullptr ? __ldg(&perm[t]) : static_cast<int32_t>(t)) : -1;
    if (t < n_out && static_cast<int64_t>(static_cast<uint32_t>(ov)) >= n_out) {
      raise_status(status, TSC_STATUS_INTERNAL);  // a row order that is not a permutation of the rows
      ov = -1;
    }
    s_orow[tid] = ov;
  }
  __syncthreads();
  for (int e = tid; e < K * RB; e += NT) {
    const int k = e / RB;
    const int r = e - k * RB;
    const int o = s_orow[r];
    int j = -1;
    if (o >= 0) {
      j = gmap != nullptr ? __ldg(&gmap[static_cast<int64_t>(k) * n_out + o]) : o;
      if (j >= n_in) {
        raise_status(status, TSC_STATUS_KEY_RANGE);
        j = -1;
      }
    }
    s_rows[e] = j;
    if (j >= 0) s_klist[k] = 1;
  }
  __syncthreads();
  if (tid == 0) {
    int n = 0;
    for (int k = 0; k < K; ++k)
      if (s_klist[k]) s_klist[n++] = k;
    s_misc[0] = n;
  }
  __syncthreads();
  const int n_chunks = (c_in + KC - 1) / KC;
  const int steps = s_misc[0] * n_chunks;

  // ---- producer: cp.async one (k, channel chunk) step into a stage --------
  // Each thread copies the same UA feature units and UB weight units in every
  // step; their rows, channels and swizzled destinations are fixed per thread
  // and computed once here, so a step only looks up the gather row.
  constexpr int UA = RB * UPR / NT;
  constexpr int UB = (TN * UPR + NT - 1) / NT;
  static_assert(RB * UPR % NT == 0, "feature copy units per thread");
  int a_row[UA], a_ch[UA], a_dst[UA];
#pragma unroll
  for (int i = 0; i < UA; ++i) {
    const int u = tid + i * NT;
    const int r = u / UPR;
    const int q = u - r * UPR;
    const int byte = q * CH;
    a_row[i] = r;
    a_ch[i] = q * (CH / 2);
    a_dst[i] = r * (KC * 2) + (swz<KC>(r, byte >> 4) << 4) + (byte & 15);
  }
  int b_n[UB], b_ch[UB], b_dst[UB];
#pragma unroll
  for (int i = 0; i < UB; ++i) {
    const int u = tid + i * NT;
    const int nn = u / UPR;
    const int q = u - nn * UPR;
    const int byte = q * CH;
    b_n[i] = u < TN * UPR ? n0 + nn : -1;
    b_ch[i] = q * (CH / 2);
    b_dst[i] = nn * (KC * 2) + (swz<KC>(nn, byte >> 4) << 4) + (byte & 15);
  }
  auto load_stage = [&](int s, int buf) {
    const int k = s_klist[s / n_chunks];
    const int c0 = (s % n_chunks) * KC;
    unsigned char* sa = smem + buf * C::STAGE;
    unsigned char* sb = sa + C::A_BYTES;
    const int32_t* rows_k = s_rows + k * RB;
#pragma unroll
    for (int i = 0; i < UA; ++i) {
      const int c = c0 + a_ch[i];
      const int j = rows_k[a_row[i]];
      const bool valid = j >= 0 && c < c_in;
      cp_async<CH>(sa + a_dst[i], valid ? F + static_cast<int64_t>(j) * c_in + c : F, valid);
    }
#pragma unroll
    for (int i = 0; i < UB; ++i) {
      if (b_n[i] < 0) continue;
      const int c = c0 + b_ch[i];
      const int n = b_n[i];
      const bool valid = n < c_out && c < c_in;
      cp_async<CH>(sb + b_dst[i], valid ? W + (static_cast<int64_t>(n) * K + k) * c_in + c : W, valid);
    }
  };

  float acc[MF][NF][4];
#pragma unroll
  for (int a = 0; a < MF; ++a)
#pragma unroll
    for (int b = 0; b < NF; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

  const int wm = warp / WN;
  const int wn = warp % WN;

#pragma unroll
  for (int s = 0; s < NS - 1; ++s) {
    if (s < steps) load_stage(s, s);
    cp_commit();
  }
  for (int s = 0; s < steps; ++s) {
    cp_wait<NS - 2>();
    __syncthreads();
    const int nxt = s + NS - 1;
    if (nxt < steps) load_stage(nxt, nxt % NS);
    cp_commit();
    const unsigned char* sa = smem + (s % NS) * C::STAGE;
    const unsigned char* sb = sa + C::A_BYTES;
#pragma unroll
    for (int kk = 0; kk < KC / 16; ++kk) {
      uint32_t af[MF][4];
#pragma unroll
      for (int mf = 0; mf < MF; ++mf) {
        const int row = wm * WTM + mf * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int chunk = kk * 2 + (lane >> 4);
        ldsm_x4(af[mf], smem_u32(sa + row * (KC * 2) + (swz<KC>(row, chunk) << 4)));
      }
#pragma unroll
      for (int nf2 = 0; nf2 < NF / 2; ++nf2) {
        uint32_t bf[4];
        const int g = lane >> 3;
        const int row = wn * WTN + nf2 * 16 + (g >> 1) * 8 + (lane & 7);
        const int chunk = kk * 2 + (g & 1);
        ldsm_x4(bf, smem_u32(sb + row * (KC * 2) + (swz<KC>(row, chunk) << 4)));
#pragma unroll
        for (int mf = 0; mf < MF; ++mf) {
          mma16816<T>(acc[mf][2 * nf2], af[mf], bf[0], bf[1]);
          mma16816<T>(acc[mf][2 * nf2 + 1], af[mf], bf[2], bf[3]);
        }
      }
    }
  }
  cp_wait<0>();
  __syncthreads();

  // ---- epilogue: fp32 tile in shared memory --------------------------------
  float* s_out = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int mf = 0; mf < MF; ++mf) {
#pragma unroll
    for (int nf = 0; nf < NF; ++nf) {
      const int row = wm * WTM + mf * 16 + (lane >> 2);
      const int col = wn * WTN + nf * 8 + (lane & 3) * 2;
      *reinterpret_cast<float2*>(&s_out[row * C::OUT_LD + col]) = make_float2(acc[mf][nf][0], acc[mf][nf][1]);
      *reinterpret_cast<float2*>(&s_out[(row + 8) * C::OUT_LD + col]) =
          make_float2(acc[mf][nf][2], acc[mf][nf][3]);
    }
  }
  __syncthreads();

  // Pairs that did not fit the gather map (duplicate input coordinates).
  if (ovf != nullptr && meta != nullptr) {
    int64_t n_ovf = static_cast<int64_t>(__ldg(&meta[TSC_META_N_OVERFLOW]));
    if (n_ovf > ovf_cap) n_ovf = ovf_cap;
    for (int64_t e = 0; e < n_ovf; ++e) {
      const int k = __ldg(&ovf[3 * e + 0]);
      const int o = __ldg(&ovf[3 * e + 1]);
      const int j = __ldg(&ovf[3 * e + 2]);
      if (tid == 0) s_misc[1] = -1;
      __syncthreads();
      if (tid < RB && s_orow[tid] == o) s_misc[1] = tid;
      __syncthreads();
      const int r = s_misc[1];
      if (r >= 0 && k >= 0 && k < K && j >= 0 && j < n_in && tid < TN && n0 + tid < c_out) {
        const T* wrow = W + (static_cast<int64_t>(n0 + tid) * K + k) * c_in;
        const T* frow = F + static_cast<int64_t>(j) * c_in;
        float s = 0.f;
        for (int c = 0; c < c_in; ++c) s = fmaf(to_f32(frow[c]), to_f32(wrow[c]), s);
        s_out[r * C::OUT_LD + tid] += s;
      }
      __syncthreads();
    }
  }

  constexpr int CPR_OUT = TN / 8;  // 16-byte output chunks per row
  for (int u = tid; u < RB * CPR_OUT; u += NT) {
    const int r = u / CPR_OUT;
    const int q = u - r * CPR_OUT;
    const int o = s_orow[r];
    const int n = n0 + q * 8;
    if (o < 0 || n >= c_out) continue;
    const float* src = &s_out[r * C::OUT_LD + q * 8];
    union {
      uint4 v;
      T h[8];
    } pk;
    epi_store8(src, n, epi, bias, pk.h);
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(o) * c_out + n) = pk.v;
  }
}

// ---------------------------------------------------------------------------
// Persistent variant with resident weights (layers whose whole weight slice
// of one column tile fits in shared memory: C_in <= KC, one channel chunk).
// Each CTA loads W[n0:n0+TN, :, :] once, in the swizzled B-tile layout, and
// then walks row tiles; the ring carries only the gathered feature rows.
// Compared with k_conv_mma this removes the per-tile weight reload and the
// per-CTA launch cost; it pays off only for small weight blocks (below).
// ---------------------------------------------------------------------------

template <int TN, int KC>
struct CfgW {
  static constexpr int A_BYTES = BM * KC * 2;
  static constexpr int PIPE = NS * A_BYTES;
  static constexpr int OUT_LD = TN + 8;
  static constexpr int EPI = BM * OUT_LD * 4;
  static constexpr int MAIN = PIPE > EPI ? PIPE : EPI;
  static constexpr int WSLICE = TN * KC * 2;  // one offset's B tile
  static constexpr int bytes(int K) { return MAIN + K * WSLICE + (K * BM + BM + KMAX + 8) * 4; }
};

// Largest resident weight block taken.  Measured on the config-3 maps: 16->16
// (14 KB) is 15 % faster resident, 16->32 (28 KB) breaks even, and 32->32
// (55 KB) and 32->64 (111 KB) are slower, because the larger shared-memory
// footprint halves the CTAs per SM that hide the gather latency.
constexpr int kMaxResidentWeightBytes = 16 * 1024;

template <typename T, int TN, int KC, int CH>
__global__ void __launch_bounds__(NT)
k_conv_mmaw(const T* __restrict__ F, int64_t n_in, int c_in, const T* __restrict__ W,
            const T* __restrict__ bias, const int32_t* __restrict__ gmap, const int32_t* __restrict__ perm,
            int K, int64_t n_out, int c_out, const int32_t* __restrict__ ovf, int64_t ovf_cap,
            const int64_t* __restrict__ meta, T* __restrict__ out, int flags, EpiParams epi, int64_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  using C = CfgW<TN, KC>;
  constexpr int WN = (TN == 128) ? 2 : 1;
  constexpr int WM = 8 / WN;
  constexpr int WTM = BM / WM;
  constexpr int WTN = TN / WN;
  constexpr int MF = WTM / 16;
  constexpr int NF = WTN / 8;
  constexpr int UPR = KC * 2 / CH;  // copy units per shared-memory row
  static_assert(NF % 2 == 0, "B fragments are loaded in pairs");

  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* s_w = smem + C::MAIN;                                             // [K][TN][KC]
  int32_t* s_rows = reinterpret_cast<int32_t*>(s_w + static_cast<int64_t>(K) * C::WSLICE);  // [K][BM]
  int32_t* s_orow = s_rows + K * BM;
  int32_t* s_klist = s_orow + BM;
  int32_t* s_misc = s_klist + KMAX;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int n0 = blockIdx.y * TN;
  const int64_t n_row_tiles = (n_out + BM - 1) / BM;

  // ---- resident weights: W[n0 + nn, k, 0:c_in] for all k --------------------
  for (int u = tid; u < K * TN * UPR; u += NT) {
    const int k = u / (TN * UPR);
    const int rem = u - k * (TN * UPR);
    const int nn = rem / UPR;
    const int q = rem - nn * UPR;
    const int c = q * (CH / 2);
    const int n = n0 + nn;
    const bool valid = n < c_out && c < c_in;
    const int byte = q * CH;
    unsigned char* dst = s_w + k * C::WSLICE + nn * (KC * 2) + (swz<KC>(nn, byte >> 4) << 4) + (byte & 15);
    const T* src = valid ? W + (static_cast<int64_t>(n) * K + k) * c_in + c : W;
    cp_async<CH>(dst, src, valid);
  }
  cp_commit();

  const int wm = warp / WN;
  const int wn = warp % WN;

  // feature copy units of this thread (fixed across steps and tiles)
  constexpr int UA = BM * UPR / NT;
  static_assert(BM * UPR % NT == 0, "feature copy units per thread");
  int a_row[UA], a_ch[UA], a_dst[UA];
#pragma unroll
  for (int i = 0; i < UA; ++i) {
    const int u = tid + i * NT;
    const int r = u / UPR;
    const int q = u - r * UPR;
    const int byte = q * CH;
    a_row[i] = r;
    a_ch[i] = q * (CH / 2);
    a_dst[i] = r * (KC * 2) + (swz<KC>(r, byte >> 4) << 4) + (byte & 15);
  }

  for (int64_t tile = blockIdx.x; tile < n_row_tiles; tile += gridDim.x) {
    const int64_t tile0 = tile * BM;
    // ---- the tile's output rows and gather-map slice -------------------------
    if (tid < KMAX) s_klist[tid] = 0;
    if (tid < BM) {
      const int64_t t = tile0 + tid;
      int32_t ov = t < n_out ? (perm != nullptr ? __ldg(&perm[t]) : static_cast<int32_t>(t)) : -1;
      if (t < n_out && static_cast<int64_t>(static_cast<uint32_t>(ov)) >= n_out) {
        raise_status(status, TSC_STATUS_INTERNAL);  // a row order that is not a permutation of the rows
        ov = -1;
      }
      s_orow[tid] = ov;
    }
    __syncthreads();
    for (int e = tid; e < K * BM; e += NT) {
      const int k = e / BM;
      const int r = e - k * BM;
      const int o = s_orow[r];
      int j = -1;
      if (o >= 0) {
        j = gmap != nullptr ? __ldg(&gmap[static_cast<int64_t>(k) * n_out + o]) : o;
        if (j >= n_in) {
          raise_status(status, TSC_STATUS_KEY_RANGE);
          j = -1;
        }
      }
      s_rows[e] = j;
      if (j >= 0) s_klist[k] = 1;
    }
    __syncthreads();
    if (tid == 0) {
      int na = 0;
      for (int k = 0; k < K; ++k)
        if (s_klist[k]) s_klist[na++] = k;
      s_misc[0] = na;
    }
    __syncthreads();
    const int steps = s_misc[0];

    auto load_stage = [&](int s, int buf) {
      const int k = s_klist[s];
      unsigned char* sa = smem + buf * C::A_BYTES;
      const int32_t* rows_k = s_rows + k * BM;
#pragma unroll
      for (int i = 0; i < UA; ++i) {
        const int j = rows_k[a_row[i]];
        const bool valid = j >= 0 && a_ch[i] < c_in;
        cp_async<CH>(sa + a_dst[i], valid ? F + static_cast<int64_t>(j) * c_in + a_ch[i] : F, valid);
      }
    };

    float acc[MF][NF][4];
#pragma unroll
    for (int a = 0; a < MF; ++a)
#pragma unroll
      for (int b = 0; b < NF; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

#pragma unroll
    for (int s = 0; s < NS - 1; ++s) {
      if (s < steps) load_stage(s, s);
      cp_commit();
    }
    for (int s = 0; s < steps; ++s) {
      cp_wait<NS - 2>();
      __syncthreads();
      const int nxt = s + NS - 1;
      if (nxt < steps) load_stage(nxt, nxt % NS);
      cp_commit();
      const unsigned char* sa = smem + (s % NS) * C::A_BYTES;
      const unsigned char* sb = s_w + s_klist[s] * C::WSLICE;
#pragma unroll
      for (int kk = 0; kk < KC / 16; ++kk) {
        uint32_t af[MF][4];
#pragma unroll
        for (int mf = 0; mf < MF; ++mf) {
          const int row = wm * WTM + mf * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int chunk = kk * 2 + (lane >> 4);
          ldsm_x4(af[mf], smem_u32(sa + row * (KC * 2) + (swz<KC>(row, chunk) << 4)));
        }
#pragma unroll
        for (int nf2 = 0; nf2 < NF / 2; ++nf2) {
          uint32_t bf[4];
          const int g = lane >> 3;
          const int row = wn * WTN + nf2 * 16 + (g >> 1) * 8 + (lane & 7);
          const int chunk = kk * 2 + (g & 1);
          ldsm_x4(bf, smem_u32(sb + row * (KC * 2) + (swz<KC>(row, chunk) << 4)));
#pragma unroll
          for (int mf = 0; mf < MF; ++mf) {
            mma16816<T>(acc[mf][2 * nf2], af[mf], bf[0], bf[1]);
            mma16816<T>(acc[mf][2 * nf2 + 1], af[mf], bf[2], bf[3]);
          }
        }
      }
    }
    cp_wait<0>();
    __syncthreads();

    // ---- epilogue: fp32 tile in shared memory (over the ring) --------------
    float* s_out = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int mf = 0; mf < MF; ++mf) {
#pragma unroll
      for (int nf = 0; nf < NF; ++nf) {
        const int row = wm * WTM + mf * 16 + (lane >> 2);
        const int col = wn * WTN + nf * 8 + (lane & 3) * 2;
        *reinterpret_cast<float2*>(&s_out[row * C::OUT_LD + col]) = make_float2(acc[mf][nf][0], acc[mf][nf][1]);
        *reinterpret_cast<float2*>(&s_out[(row + 8) * C::OUT_LD + col]) =
            make_float2(acc[mf][nf][2], acc[mf][nf][3]);
      }
    }
    __syncthreads();

    // Pairs that did not fit the gather map (duplicate input coordinates).
    if (ovf != nullptr && meta != nullptr) {
      int64_t n_ovf = static_cast<int64_t>(__ldg(&meta[TSC_META_N_OVERFLOW]));
      if (n_ovf > ovf_cap) n_ovf = ovf_cap;
      for (int64_t e = 0; e < n_ovf; ++e) {
        const int k = __ldg(&ovf[3 * e + 0]);
        const int o = __ldg(&ovf[3 * e + 1]);
        const int j = __ldg(&ovf[3 * e + 2]);
        if (tid == 0) s_misc[1] = -1;
        __syncthreads();
        if (tid < BM && s_orow[tid] == o) s_misc[1] = tid;
        __syncthreads();
        const int r = s_misc[1];
        if (r >= 0 && k >= 0 && k < K && j >= 0 && j < n_in && tid < TN && n0 + tid < c_out) {
          const T* wrow = W + (static_cast<int64_t>(n0 + tid) * K + k) * c_in;
          const T* frow = F + static_cast<int64_t>(j) * c_in;
          float sacc = 0.f;
          for (int c = 0; c < c_in; ++c) sacc = fmaf(to_f32(frow[c]), to_f32(wrow[c]), sacc);
          s_out[r * C::OUT_LD + tid] += sacc;
        }
        __syncthreads();
      }
    }

    constexpr int CPR_OUT = TN / 8;  // 16-byte output chunks per row
    for (int u = tid; u < BM * CPR_OUT; u += NT) {
      const int r = u / CPR_OUT;
      const int q = u - r * CPR_OUT;
      const int o = s_orow[r];
      const int n = n0 + q * 8;
      if (o < 0 || n >= c_out) continue;
      const float* src = &s_out[r * C::OUT_LD + q * 8];
      union {
        uint4 v;
        T h[8];
      } pk;
      epi_store8(src, n, epi, bias, pk.h);
      *reinterpret_cast<uint4*>(out + static_cast<int64_t>(o) * c_out + n) = pk.v;
    }
    __syncthreads();  // s_out, s_orow and s_rows are rewritten by the next tile
  }
  cp_wait<0>();
}

}  // namespace mma
}  // namespace tsc
