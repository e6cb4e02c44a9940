// Blackwell (sm_100a) tensor-core implicit GEMM for sparse convolution:
// tcgen05.mma with the accumulator in tensor memory.
//
// One CTA = 128 output rows x TN output channels (UMMA M=128, N=TN, K=16).
// Warp roles (160 threads):
//   warps 0-3  producers: gather feature rows (gather map -> cp.async, rows
//              without a pair zero-filled) and the weight slice W[:, k, chunk]
//              (KRSC = K-major B operand) into a 4-stage shared-memory ring in
//              the canonical UMMA K-major 128/64/32-byte-swizzled layout; after
//              the copies land: fence.proxy.async + mbarrier arrive (full[s]).
//              Afterwards the same 128 threads are the epilogue: thread r owns
//              output row r = TMEM lane r, reads it with tcgen05.ld, adds
//              bias (+ duplicate-coordinate overflow pairs), ReLU, stores.
//   warp 4     one elected thread issues tcgen05.mma for each (offset, channel
//              chunk) step and tcgen05.commit -> empty[s] (stage free) and,
//              at the end, -> done.
// Every mbarrier wait is bounded by a deadline on %globaltimer; a timeout
// sets TSC_STATUS_WAIT_TIMEOUT, raises a CTA-wide abort flag, and all roles
// leave their loops so TMEM is still freed and the kernel returns.
#pragma once

#include "conv_mma.cuh"
#include "tsc_common.cuh"

namespace tsc {
namespace tc {

constexpr int BM = 128;
constexpr int NPROD = 128;          // producer / epilogue threads (warps 0-3)
constexpr int NT = NPROD + 32;      // + MMA warp
constexpr int KMAX = 64;
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s per kernel
constexpr long long kWaitCycles = 4000000000ll;        // bounded barrier waits (~2 s)
constexpr long long kTestWaitCycles = 200000ll;        // TSC_CONV_TEST_WAIT_TIMEOUT (~0.1 ms)

template <int TN, int KC>
struct Cfg {
  static constexpr int A_BYTES = BM * KC * 2;
  static constexpr int B_BYTES = TN * KC * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;  // multiple of 1024
  // ring of ~96 KB (two CTAs per SM) for N <= 64, ~192 KB for wider tiles
  static constexpr int RING = (TN <= 64 ? 96 : 192) * 1024;
  static constexpr int NS = RING / STAGE > 12 ? 12 : (RING / STAGE < 2 ? 2 : RING / STAGE);
  static constexpr int PIPE = NS * STAGE;
  // control block after the ring: barriers full[NS] @0, empty[NS] @8*NS,
  // done @16*NS, then tmem address, abort flag, number of active offsets;
  // followed by active offsets, out rows and gather rows [K][BM]
  static constexpr int OFF_EMPTY = 8 * NS;
  static constexpr int OFF_DONE = 16 * NS;
  static constexpr int OFF_TMEM = OFF_DONE + 8;
  static constexpr int OFF_ABORT = OFF_TMEM + 4;
  static constexpr int OFF_NACTIVE = OFF_ABORT + 4;
  static constexpr int CTRL = (OFF_NACTIVE + 4 + 127) / 128 * 128;
  static constexpr int TOTAL_FIXED = 1024 /*alignment slack*/ + PIPE + CTRL + (KMAX + BM) * 4;
  static constexpr int TMEM_COLS = TN < 32 ? 32 : TN;
  static constexpr int SWZ_MODE = KC == 64 ? 2 : (KC == 32 ? 4 : 6);  // UMMA layout type
  static constexpr int SBO = 8 * KC * 2;                             // bytes between 8-row groups
};

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread for up to `hint_ns` (it resumes as
// soon as the phase completes).  A suspended waiter issues no instructions,
// so waiting roles do not take issue slots from the warps doing work on the
// same SM sub-partition.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

constexpr uint32_t kSuspendNs = 50000;  // upper bound of one suspension

// Bounded wait: false on timeout (about `limit` SM cycles after the wait
// began, kWaitCycles by default) or when another role aborted.  The
// `deadline` argument is unused and kept for the call sites' symmetry.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned long long deadline,
                                          volatile int* abort_flag, int64_t* status,
                                          long long limit = kWaitCycles) {
  (void)deadline;
  if (mbar_try_wait(bar, parity)) return true;
  // SM cycle counter (cheap to read, unlike %globaltimer): ~2 s at 2 GHz.
  const long long start = clock64();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, limit < kWaitCycles ? 1000u : kSuspendNs)) return true;
    if (*abort_flag) return false;
    if (clock64() - start > limit) {
      raise_status(status, TSC_STATUS_WAIT_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Arrive on `bar` when all prior cp.async of this thread have completed; the
// arrival counts against the barrier's expected count (.noinc).
__device__ __forceinline__ void cp_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

template <int N>
__device__ __forceinline__ void cp_wait_n() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// UMMA shared-memory descriptor, K-major, swizzled (layout type SWZ), 8-row
// groups SBO bytes apart; LBO is unused for swizzled K-major layouts (1).
template <int SWZ, int SBO>
__device__ __forceinline__ unsigned long long smem_desc(uint32_t addr) {
  return static_cast<unsigned long long>((addr >> 4) & 0x3FFFu) | (1ull << 16) |
         (static_cast<unsigned long long>((SBO >> 4) & 0x3FFF) << 32) | (1ull << 46) |
         (static_cast<unsigned long long>(SWZ) << 61);
}

// Instruction descriptor for kind::f16: D fp32, A/B fp16 (0) or bf16 (1),
// both K-major, M = 128, N = TN.
template <typename T, int TN>
__host__ __device__ constexpr uint32_t instr_desc() {
  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(TN >> 3) << 17) |
         (static_cast<uint32_t>(BM >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, unsigned long long a, unsigned long long b,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same, with a disable-output-lane mask: accumulator rows (TMEM lanes) whose
// bit is set in {m0..m3} (lane i -> m[i / 32] bit i % 32) are left unchanged.
__device__ __forceinline__ void umma_f16_masked(uint32_t tmem_d, unsigned long long a, unsigned long long b,
                                                uint32_t idesc, uint32_t m0, uint32_t m1, uint32_t m2,
                                                uint32_t m3) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, 1, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%4, %5, %6, %7}, p; }"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(m0), "r"(m1), "r"(m2), "r"(m3)
      : "memory");
}

__device__ __forceinline__ void tmem_st32_zero(uint32_t taddr) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
      "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Ring tail: waits until the tcgen05.commit arrivals that released the last
// fill of every stage have landed on empty[stage].  A commit arrives
// asynchronously when its MMAs complete; without this wait the CTA could exit
// first and the arrival would land in the shared memory of the next CTA that
// the SM runs (another launch's barriers, TMEM address or row tables).
// `steps` ring steps were produced and consumed in total.
__device__ __forceinline__ void drain_ring(uint32_t bar_empty, int ns, int64_t steps, unsigned long long deadline,
                                           volatile int* abort_flag, int64_t* status) {
  for (int s = 0; s < ns && s < steps; ++s) {
    const int64_t fills = steps / ns + (s < steps % ns ? 1 : 0);
    if (!mbar_wait(bar_empty + 8 * s, static_cast<uint32_t>((fills - 1) & 1), deadline, abort_flag, status)) return;
  }
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <typename T, int TN, int KC>
__global__ void __launch_bounds__(NT, 1)
k_conv_tc(const T* __restrict__ F, int64_t n_in, int c_in, const T* __restrict__ W,
          const T* __restrict__ bias, const int32_t* __restrict__ gmap, const int32_t* __restrict__ perm, int K,
          int64_t n_out, int c_out, const int32_t* __restrict__ ovf, int64_t ovf_cap,
          const int64_t* __restrict__ meta, T* __restrict__ out, int flags, EpiParams epi, int64_t* __restrict__ status) {
  using C = Cfg<TN, KC>;
  constexpr int NS = C::NS;
  constexpr int UPR = KC * 2 / 16;  // 16-byte chunks per shared-memory row
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte aligned ring (swizzle atoms are address-based)
  const uint32_t raw_u32 = mma::smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_u32 & 1023u)) & 1023u;
  unsigned char* ring = smem_raw + pad;
  const uint32_t ring_u32 = raw_u32 + pad;
  unsigned char* ctrl = ring + C::PIPE;
  const uint32_t ctrl_u32 = ring_u32 + C::PIPE;
  static_assert(C::OFF_NACTIVE + 4 <= C::CTRL, "control block overflow");
  const uint32_t bar_full = ctrl_u32;
  const uint32_t bar_empty = ctrl_u32 + C::OFF_EMPTY;
  const uint32_t bar_done = ctrl_u32 + C::OFF_DONE;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(ctrl + C::OFF_TMEM);
  volatile int* s_abort = reinterpret_cast<volatile int*>(ctrl + C::OFF_ABORT);
  int* s_nactive = reinterpret_cast<int*>(ctrl + C::OFF_NACTIVE);
  int32_t* s_klist = reinterpret_cast<int32_t*>(ctrl + C::CTRL);
  int32_t* s_orow = s_klist + KMAX;
  int32_t* s_rows = s_orow + BM;  // [K][BM]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int64_t tile0 = static_cast<int64_t>(blockIdx.x) * BM;
  const int n0 = blockIdx.y * TN;
  const unsigned long long deadline = globaltimer() + kWaitNs;

  // ---- set-up: barriers, TMEM, gather-map slice ----------------------------
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
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_full + 8 * s, NPROD);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_done, 1);
    *s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 4) {
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     static_cast<uint32_t>(ctrl_u32 + C::OFF_TMEM)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
    int n = 0;
    for (int k = 0; k < K; ++k)
      if (s_klist[k]) s_klist[n++] = k;
    *s_nactive = n;
  }
  __syncthreads();
  const uint32_t tmem = *s_tmem;
  const int n_chunks = (c_in + KC - 1) / KC;
  const int steps = *s_nactive * n_chunks;

  if (warp < 4) {
    // ---- producers -----------------------------------------------------------
    // Each thread's copies for a stage end with cp.async.mbarrier.arrive.noinc
    // on full[stage] (init count NPROD): the copy engine arrives for the thread
    // once its copies have landed, so producers run ahead over every free stage.
    for (int s = 0; s < steps; ++s) {
      const int stage = s % NS;
      const int fill = s / NS;
      if (fill > 0 && !mbar_wait(bar_empty + 8 * stage, (fill - 1) & 1, deadline, s_abort, status)) break;
      const int k = s_klist[s / n_chunks];
      const int c0 = (s % n_chunks) * KC;
      unsigned char* sa = ring + stage * C::STAGE;
      unsigned char* sb = sa + C::A_BYTES;
      for (int u = tid; u < BM * UPR; u += NPROD) {
        const int r = u / UPR;
        const int q = u - r * UPR;
        const int c = c0 + q * 8;
        const int j = s_rows[k * BM + r];
        const bool valid = j >= 0 && c < c_in;
        unsigned char* dst = sa + r * (KC * 2) + (mma::swz<KC>(r, q) << 4);
        mma::cp_async<16>(dst, valid ? F + static_cast<int64_t>(j) * c_in + c : F, valid);
      }
      for (int u = tid; u < TN * UPR; u += NPROD) {
        const int nn = u / UPR;
        const int q = u - nn * UPR;
        const int c = c0 + q * 8;
        const int n = n0 + nn;
        const bool valid = n < c_out && c < c_in;
        unsigned char* dst = sb + nn * (KC * 2) + (mma::swz<KC>(nn, q) << 4);
        mma::cp_async<16>(dst, valid ? W + (static_cast<int64_t>(n) * K + k) * c_in + c : W, valid);
      }
      cp_arrive_noinc(bar_full + 8 * stage);
    }
    cp_wait_all();
  } else if (lane == 0) {
    // ---- MMA issuer ------------------------------------------------------------
    constexpr uint32_t idesc = instr_desc<T, TN>();
    for (int s = 0; s < steps; ++s) {
      const int stage = s % NS;
      if (!mbar_wait(bar_full + 8 * stage, (s / NS) & 1, deadline, s_abort, status)) break;
      tc_fence_after();
      const uint32_t a_addr = ring_u32 + stage * C::STAGE;
      const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
      for (int kk = 0; kk < KC / 16; ++kk) {
        umma_f16(tmem, smem_desc<C::SWZ_MODE, C::SBO>(a_addr + kk * 32),
                 smem_desc<C::SWZ_MODE, C::SBO>(b_addr + kk * 32), idesc, (s > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(bar_empty + 8 * stage);
    }
    umma_commit(bar_done);
  }

  // ---- epilogue: warps 0-3, thread r <-> TMEM lane r <-> tile row r --------
  if (warp < 4) {
    const bool ok = __all_sync(kFullMask, mbar_wait(bar_done, 0, deadline, s_abort, status));
    // every MMA has completed: collect the ring's last empty arrivals
    if (tid == 0 && ok && !*s_abort) drain_ring(bar_empty, NS, steps, deadline, s_abort, status);
    tc_fence_after();
    const int r = tid;
    const int o = s_orow[r];
    int64_t n_ovf = 0;
    if (ovf != nullptr && meta != nullptr) {
      n_ovf = static_cast<int64_t>(__ldg(&meta[TSC_META_N_OVERFLOW]));
      if (n_ovf > ovf_cap) n_ovf = ovf_cap;
    }
#pragma unroll 1
    for (int c0 = 0; c0 < TN; c0 += 32) {
      float v[32];
      __syncwarp();
      if (ok && steps > 0) {
        tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c0, v);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      if (o >= n_out) {
        raise_status(status, TSC_STATUS_INTERNAL);
        continue;
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
      for (int q = 0; q < 4; ++q) {
        const int n = n0 + c0 + q * 8;
        if (n >= c_out) break;
        union {
          uint4 u;
          T h[8];
        } pk;
#pragma unroll
        for (int i = 0; i < 8; ++i) pk.h[i] = from_f32<T>(epi_apply(v[q * 8 + i], n + i, epi, bias));
        *reinterpret_cast<uint4*>(out + static_cast<int64_t>(o) * c_out + n) = pk.u;
      }
    }
  }

  // ---- teardown ------------------------------------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

}  // namespace tc
}  // namespace tsc
