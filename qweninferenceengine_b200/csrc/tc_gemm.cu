// tc_gemm.cu -- batched Q4 / fp16 projections on tcgen05 tensor cores.
//
// CTA = 128 output rows x nb activation rows, K split over grid.y.  NG groups
// of four warps (NG = 4 for Q4 launches, 2 for the fp16 LM head) plus three:
//   warp 4NG    producer: one lane issues the 1-D bulk copies.  Q4 weights go
//               to a deep ring of raw 4608-byte chunks (up to 32; usually
//               every chunk of the CTA), all issued before griddepcontrol.wait
//               -- weights do not depend on the previous kernel of the stream,
//               so they stream in while it still runs -- and refilled as soon
//               as a chunk has been read by the dequantising warps.
//               Activations go to their own ring (up to 12 stages) and fp16
//               weights to a shared-memory A ring; the MMAs free both.
//   warps 0..4NG-1  Q4: the groups take units (one or two 64-k chunks) in
//               turn; thread r of a group dequantises both 32-weight blocks of
//               row r per chunk (16 nibble pairs each -> fp16 via the 0x6400
//               exponent trick, (q - 8) exact, one rounding for the product
//               with the block scale) and stores the row's 64 values into
//               tensor-memory lane r with one tcgen05.st (one A stage per
//               group).  Then the epilogue: warp w reads tensor-memory lanes
//               32(w%4).. (its rows) for its group's share of the columns
//   warps 4NG+1, 4NG+2  the first allocates tensor memory; each MMA warp takes
//               alternate units, one lane issuing 4 MMAs (M=128, N=nb, K=16)
//               per chunk (A from tensor memory, or from shared memory for
//               fp16) into the warp's own fp32 accumulator and committing the
//               A stage (aempty) and the activation stage (xempty) back.  Two
//               issuing warps because a lone MMA warp's wait -> issue -> commit
//               loop, not the tensor pipe, set the rate at N=64; the epilogue
//               adds the two accumulators in a fixed order.  Where two
//               accumulators and the A stages do not fit in tensor memory
//               (nb > 128), the second MMA warp idles.
// Three rings because each refill sits on its own loop of latencies: a raw
// weight chunk is refilled one HBM latency after its dequantisation, an
// activation chunk one L2 latency (~1.5 us with every CTA reading the same
// chunk) after its MMAs.  With one ring for everything, that loop bounded the
// kernel at ring depth / 1.9 us chunks.
// D[n][b] = sum_k A[n][k] X[b][k]: A (weights) and X (activations) are both
// K-major, so one tcgen05.mma.kind::f16 per 16 k computes W . X^T.
//
// Numerics against gemv_q4_0 (matmul.metal:44-45): the reference forms
// (q-8)*scale exactly in fp32; here the product is rounded once to fp16
// (relative error <= 2^-11) before the fp32-accumulating MMA.  The fp16 LM
// head (matmul.metal:75-113) is exact up to summation order.
//
// All waits are bounded (2 s of %globaltimer); a timeout records
// kDevWaitTimeout, sets a CTA-wide abort flag that the other roles honour, and
// the kernel still waits for its own bulk copies and MMAs before it frees
// tensor memory and returns.
#include "qwen_common.cuh"
#include "qwen_internal.h"
#include "tc_gemm.h"

namespace qwen {
namespace {

constexpr int kTcMaxStages = 4;      // A stages in tensor memory (Q4)
constexpr int kTcMaxF16Stages = 4;   // A ring (fp16 weights straight from HBM)
constexpr int kTcMaxXStages = 12;    // activation ring
constexpr int kTcMaxRawStages = 32;  // Q4 raw-weight ring
constexpr size_t kTcSmemBudget = 227 * 1024;
// Warp layout for NG groups of four dequantising/epilogue warps: warps
// 0 .. 4NG-1, then the producer warp, then the two MMA warps.  Q4 launches use
// four groups; the fp16 LM head (no dequantisation) two, so that two CTAs with
// 60 registers per thread still fit one SM.
constexpr int kDeqGroups = 4;                      // Q4 launches
constexpr int kF16DeqGroups = 2;                   // fp16 launches
__host__ __device__ constexpr int tc_threads(int ng) { return ng * 128 + 3 * 32; }
constexpr int kDeqGroupWarps = 4;    // one dequantising group: 128 threads, one per tile row
constexpr uint32_t kTmemAStageCols = kTcChunkK / 2;  // a Q4 A stage: 64 fp16 per lane
constexpr unsigned long long kTcWaitNs = 2000000000ull;

// ------------------------------------------------------------ tcgen05 PTX --
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D (tensor memory) (+)= A(smem desc) . B(smem desc)^T, fp16 in, fp32 out.
__device__ __forceinline__ void tc_mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same with A (M x K, K-major) read from tensor memory at a_tmem: lane m holds
// row m, two fp16 of k per 32-bit column.
__device__ __forceinline__ void tc_mma_f16_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 consecutive 32-bit columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]),
      "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]),
      "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// Arrive on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// 16 consecutive fp32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  // The wait names the registers so no use of them is scheduled before it.
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 B apart (SBO), LBO unused for swizzled K-major, descriptor version 1.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator, A = B = fp16, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t f16_idesc(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded parity wait.  honour_abort: give up as soon as another role did.
__device__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err,
                        bool honour_abort = true) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = gtime();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (honour_abort && *abort) return false;
      if (gtime() - t0 > kTcWaitNs) {
        *abort = 1;
        raise_error(err, kDevWaitTimeout);
        return false;
      }
    }
  }
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// 8 nibble-permuted weights -> 4 half2 (k0,k1) (k2,k3) (k4,k5) (k6,k7) at
// o[0..3], each (q - 8) * scale rounded once.
__device__ __forceinline__ void dequant8(uint32_t w, __half2 s2, uint32_t* o) {
  const __half2 off = __floats2half2_rn(1032.0f, 1032.0f);
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t v = ((w >> (4 * s)) & 0x000F000Fu) | 0x64006400u;  // 1024 + q
    o[s] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(v), off), s2));
  }
}

template <int NG>
__global__ void __launch_bounds__(tc_threads(NG), 1) k_tc_gemm(TcGemmArgs a) {
  constexpr int kDeqThreads = NG * 128;         // dequant + epilogue threads
  constexpr int kProducerWarp = NG * 4;
  constexpr int kMmaWarp = kProducerWarp + 1;   // allocates tensor memory; MMA warps +0, +1
  extern __shared__ uint8_t tc_smem[];
  const bool q4 = a.q4;
  const int U = a.unit;                // 64-k chunks per pipeline unit (Q4: 1 or 2; fp16: 1)
  const int S = a.stages;              // A stages: tensor memory (Q4) or shared memory (fp16)
  const int XS = a.xstages;            // activation ring depth
  const int RS = q4 ? a.raw_stages : 0;  // raw Q4 ring depth
  const int NW = q4 ? RS : S;          // weight-landing barriers (raw ring, or A ring for fp16)
  const int SA = q4 ? 0 : S;           // shared-memory A stages
  const uint32_t pad = (1024u - (smem_u32(tc_smem) & 1023u)) & 1023u;
  uint8_t* sA = tc_smem + pad;                             // [SA][128 rows][128 B] (fp16)
  uint8_t* sX = sA + SA * kF16TcChunkBytes;                // [XS][nb rows][128 B]
  const int nb = a.nb;
  const uint32_t xbytes = (uint32_t)nb * 128u;
  const size_t act_chunk_bytes = (size_t)(a.act_stride_rows > 0 ? a.act_stride_rows : nb) * 128u;
  const uint32_t xunit = (uint32_t)U * xbytes;             // activation bytes per unit
  const uint32_t runit = (uint32_t)U * kQ4TcChunkBytes;    // raw Q4 bytes per unit
  uint8_t* sR = sX + XS * xunit;                           // [RS][U][4608] (Q4)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sR + RS * runit);
  uint64_t* wfull = bars;          // [NW] weight chunk landed
  uint64_t* rempty = wfull + NW;   // [RS] raw chunk read by its dequantising group
  uint64_t* xfull = rempty + RS;   // [XS] activation chunk landed
  uint64_t* xempty = xfull + XS;   // [XS] MMAs reading the activation chunk completed
  uint64_t* deq = xempty + XS;     // [S]  Q4: A stage written and its activations landed
  uint64_t* aempty = deq + S;      // [S]  MMAs reading the A stage completed
  uint64_t* accum = aempty + S;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_chunks = a.k / kTcChunkK;
  const int cps = n_chunks / a.splits;
  const int nu = cps / U;  // pipeline units of this CTA
  const int c0 = blockIdx.y * cps;
  const int tile = blockIdx.x;
  // Tensor memory: one fp32 accumulator per MMA warp, acc_cols columns each,
  // then (Q4) the A stages, 32 columns per chunk (64 fp16 of k per lane).
  const int MW = a.mma_warps;
  const uint32_t acc_cols = nb <= 32 ? 32u : nb <= 64 ? 64u : nb <= 128 ? 128u : 256u;
  const uint32_t a_base = acc_cols * (uint32_t)MW;
  const uint32_t need = a_base + (q4 ? (uint32_t)(S * U) * kTmemAStageCols : 0u);
  const uint32_t ncols = need <= 32 ? 32u : need <= 64 ? 64u : need <= 128 ? 128u : need <= 256 ? 256u : 512u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NW; ++s) mbar_init(wfull + s, 1);
    for (int s = 0; s < RS; ++s) mbar_init(rempty + s, kDeqGroupWarps);
    for (int s = 0; s < XS; ++s) {
      mbar_init(xfull + s, 1);
      mbar_init(xempty + s, 1);
    }
    for (int s = 0; s < S; ++s) {
      mbar_init(deq + s, kDeqGroupWarps);
      mbar_init(aempty + s, 1);
    }
    mbar_init(accum, 2);  // both MMA warps
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tslot, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (threadIdx.x == 0) pdl_launch_dependents();
  if (warp == kProducerWarp) {
    // ---------------------------------------------------------- producer --
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint32_t cbytes = q4 ? kQ4TcChunkBytes : kF16TcChunkBytes;  // weight bytes per chunk
      // Unit i: chunks c0 + U i .. +U-1, adjacent in the weight blob (one copy)
      // but not always in the activation tiles (one copy per chunk).
      auto load_w = [&](int i) {
        const int s = i % NW;
        const uint32_t bytes = cbytes * (uint32_t)U;
        mbar_arrive_expect_tx(wfull + s, bytes);
        uint8_t* wdst = q4 ? sR + s * runit : sA + s * kF16TcChunkBytes;
        bulk_g2s_stream(wdst, a.w + ((size_t)tile * n_chunks + c0 + (size_t)i * U) * cbytes, bytes,
                        wfull + s, pol);
      };
      auto load_x = [&](int i) {
        const int s = i % XS;
        mbar_arrive_expect_tx(xfull + s, xunit);
        for (int j = 0; j < U; ++j)
          bulk_g2s(sX + s * xunit + j * xbytes, a.act + (size_t)(c0 + i * U + j) * act_chunk_bytes,
                   xbytes, xfull + s);
      };
      int nw = nu < NW ? nu : NW, nx = nu < XS ? nu : XS;  // units issued
      for (int i = 0; i < nw; ++i) load_w(i);  // weights do not depend on earlier kernels
      pdl_wait();
      for (int i = 0; i < nx; ++i) load_x(i);
      // Refill in the order the slots free up: the weight slot of chunk t once
      // it was read (Q4: dequantised, which precedes its MMAs; fp16: its MMAs
      // completed), then its activation slot once its MMAs completed.  While a
      // refill is due, nw == t + NW and nx == t + XS.
      for (int t = 0; nw < nu || nx < nu; ++t) {
        if (nw < nu) {
          const bool ok = q4 ? tc_wait(rempty + t % RS, (t / RS) & 1, abort, a.err)
                             : tc_wait(aempty + t % S, (t / S) & 1, abort, a.err);
          if (!ok) break;
          load_w(nw++);
        }
        if (nx < nu) {
          if (!tc_wait(xempty + t % XS, (t / XS) & 1, abort, a.err)) break;
          load_x(nx++);
        }
      }
      // Every issued copy lands before the CTA may exit.
      for (int j = nw > NW ? nw - NW : 0; j < nw; ++j)
        tc_wait(wfull + j % NW, (j / NW) & 1, abort, a.err, false);
      for (int j = nx > XS ? nx - XS : 0; j < nx; ++j)
        tc_wait(xfull + j % XS, (j / XS) & 1, abort, a.err, false);
    }
    __syncwarp();
  } else if (warp >= kMmaWarp) {
    // --------------------------------------------------------------- MMA --
    // MMA warp m takes units m, m + MW, ... into accumulator m.  The warp
    // loops converged (every lane waits); lane 0 issues.  One wait per Q4
    // unit: deq[s] completes only after the unit's activations landed.
    const int m = warp - kMmaWarp;
    const uint32_t idesc = f16_idesc(kTcM, nb);
    const uint32_t dacc = tmem + (uint32_t)m * acc_cols;
    bool issued = false;
    for (int i = m; m < MW && i < nu; i += MW) {
      const int s = i % S, xs = i % XS;
      bool ok = tc_wait(q4 ? deq + s : wfull + s, (i / S) & 1, abort, a.err);
      if (!q4) ok = ok && tc_wait(xfull + xs, (i / XS) & 1, abort, a.err);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint64_t bd = sw128_kmajor_desc(smem_u32(sX + xs * xunit));
        if (q4) {
          for (int j = 0; j < U; ++j) {
            const uint32_t at = tmem + a_base + (uint32_t)(s * U + j) * kTmemAStageCols;
            const uint64_t bj = bd + (uint64_t)((j * xbytes) >> 4);  // next activation tile
#pragma unroll
            for (int kk = 0; kk < kTcChunkK / 16; ++kk)  // 8 columns (16 k) of A, +32 B of X
              tc_mma_f16_ta(dacc, at + 8u * kk, bj + 2 * kk, idesc,
                            (i != m || j != 0 || kk != 0) ? 1u : 0u);
          }
        } else {
          const uint64_t ad = sw128_kmajor_desc(smem_u32(sA + s * kF16TcChunkBytes));
#pragma unroll
          for (int kk = 0; kk < kTcChunkK / 16; ++kk)  // +32 B of k per MMA inside the atom
            tc_mma_f16(dacc, ad + 2 * kk, bd + 2 * kk, idesc, (i != m || kk != 0) ? 1u : 0u);
        }
        tc_commit(aempty + s);
        tc_commit(xempty + xs);
      }
      issued = true;
      __syncwarp();
    }
    // accum completes once both warps' MMAs have (a warp without any arrives
    // directly).
    if (lane == 0) {
      if (issued)
        tc_commit(accum);
      else
        mbar_arrive(accum);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------- dequant (Q4 only) --
    // Group h (warps 4h..4h+3) takes units h, h+4, ...; thread r of the
    // group dequantises row r into tensor-memory lane r (warp 4h+q owns lanes
    // 32q..32q+31).  Waits are made warp-uniform so that the per-warp
    // arrivals (lane 0 after __syncwarp) and the warp-collective tcgen05.st
    // stay well-formed on abort.
    const int r = threadIdx.x & (kTcM - 1), h = threadIdx.x >> 7;
    const int q = (threadIdx.x >> 5) & 3;
    if (q4) {
      const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + a_base;
      for (int i = h; i < nu; i += NG) {
        const int s = i % S, rs = i % RS;
        if (!__all_sync(0xffffffffu, tc_wait(wfull + rs, (i / RS) & 1, abort, a.err))) break;
        bool failed = false;
        for (int j = 0; j < U; ++j) {
          const uint8_t* raw = sR + rs * runit + j * kQ4TcChunkBytes;
          const uint4 p0 = *reinterpret_cast<const uint4*>(raw + r * 16);
          const uint4 p1 = *reinterpret_cast<const uint4*>(raw + 2048 + r * 16);
          const __half2 sc = *reinterpret_cast<const __half2*>(raw + 4096 + r * 4);
          const __half2 s0 = __low2half2(sc), s1 = __high2half2(sc);
          uint32_t v[32];
          dequant8(p0.x, s0, v + 0);
          dequant8(p0.y, s0, v + 4);
          dequant8(p0.z, s0, v + 8);
          dequant8(p0.w, s0, v + 12);
          dequant8(p1.x, s1, v + 16);
          dequant8(p1.y, s1, v + 20);
          dequant8(p1.z, s1, v + 24);
          dequant8(p1.w, s1, v + 28);
          if (j == U - 1) {
            __syncwarp();
            if (lane == 0) mbar_arrive(rempty + rs);  // the raw slot may be refilled
          }
          if (j == 0) {
            if (i >= S &&
                !__all_sync(0xffffffffu, tc_wait(aempty + s, ((i / S) - 1) & 1, abort, a.err))) {
              failed = true;
              break;
            }
            tc_fence_after();
          }
          tmem_st32(lane_base + (uint32_t)(s * U + j) * kTmemAStageCols, v);
        }
        if (failed) break;
        tmem_wait_st();
        tc_fence_before();
        // One warp of the group also waits for the unit's activations, so the
        // MMA warp needs a single wait per unit.
        if (q == 0 &&
            !__all_sync(0xffffffffu, tc_wait(xfull + i % XS, (i / XS) & 1, abort, a.err)))
          break;
        __syncwarp();
        if (lane == 0) mbar_arrive(deq + s);
      }
    }
    // ---------------------------------------------------------- epilogue --
    // Warp w reads tensor-memory lanes 32(w%4) .. +31 (rows r) and the column
    // groups of half w/4: groups of 16 columns [g0, g1).
    pdl_wait();  // outputs are written only after the previous kernel completed
    const bool landed = tc_wait(accum, 0, abort, a.err, false);
    tc_fence_after();
    // tcgen05.ld is warp-collective: the decision is the warp's, not the lane's.
    const bool go = __all_sync(0xffffffffu, landed && !*abort);
    // Column groups of 16 split over the four dequantising groups.
    const int groups = nb / 16, gq = (groups + NG - 1) / NG;
    const int g0 = min(groups, h * gq), g1 = min(groups, g0 + gq);
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    // The second accumulator holds units 1, 3, ... (none when nu == 1).
    const bool two = MW == 2 && nu > 1;
    auto ld_acc = [&](uint32_t col, float (&v)[16]) {
      tmem_ld16(lane_addr + col, v);
      if (two) {
        float w[16];
        tmem_ld16(lane_addr + acc_cols + col, w);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] += w[j];
      }
    };
    if (a.swiglu_act) {
      // half(gate) and half(up) of every row and column to shared memory
      // [b][128] (the activation ring is idle once the accumulators are
      // complete); then all 256 threads form 8 outputs each per 16-byte
      // store.  The tile's 64 gate rows are k = 64 tile .. +63 of the down
      // projection's input: exactly activation chunk `tile`, stored whole.
      __half* gu = reinterpret_cast<__half*>(sX);
      if (go)
        for (int c = 16 * g0; c < 16 * g1; c += 16) {
          float v[16];
          ld_acc((uint32_t)c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) gu[(c + j) * 128 + r] = f2h(v[j]);
        }
      asm volatile("bar.sync 2, %0;" ::"r"(kDeqThreads) : "memory");  // the epilogue warps
      if (go) {
        uint8_t* chunk = a.swiglu_act + (size_t)tile * a.swiglu_nb * 128;
        for (int it = threadIdx.x; it < a.nb_valid * 8; it += kDeqThreads) {
          const int b = it >> 3, jj = it & 7;
          const uint4 g8 = *reinterpret_cast<const uint4*>(gu + b * 128 + jj * 8);
          const uint4 u8 = *reinterpret_cast<const uint4*>(gu + b * 128 + 64 + jj * 8);
          const uint32_t gw[4] = {g8.x, g8.y, g8.z, g8.w}, uw[4] = {u8.x, u8.y, u8.z, u8.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 g2 = __half22float2(u32_as_h2(gw[e])), u2 = __half22float2(u32_as_h2(uw[e]));
            o[e] = h2_as_u32(__floats2half2_rn(silu_ref(g2.x) * u2.x, silu_ref(g2.y) * u2.y));
          }
          *reinterpret_cast<uint4*>(chunk + (size_t)b * 128 + (((uint32_t)jj ^ (uint32_t)(b & 7)) << 4)) =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    } else if (go) {
      const size_t row = (size_t)tile * kTcM + r;
      for (int c = 16 * g0; c < 16 * g1; c += 16) {
        float v[16];
        ld_acc((uint32_t)c, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int b = c + j;
          if (b < a.nb_valid) {
            if (a.part)
              a.part[((size_t)blockIdx.y * a.nb_valid + b) * a.n_rows + row] = v[j];
            else
              a.out[(size_t)b * a.ld_out + row] = f2h(v[j]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem, ncols);
}

// ----------------------------------------------------------- repacking ---
// Nibble order inside a 32-bit word: byte s holds (k_2s low, k_2s+1 high);
// the blob stores k_2s at nibble s and k_2s+1 at nibble 4+s.
__device__ __forceinline__ uint32_t permute_nibbles(uint32_t w) {
  uint32_t o = 0;
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t b = (w >> (8 * s)) & 0xFFu;
    o |= (b & 0xFu) << (4 * s);
    o |= (b >> 4) << (16 + 4 * s);
  }
  return o;
}

// Source row tile * R + r goes to tile row dst_off + r (R = rows per tile taken
// from the source: 128, or 64 for the gate/up pairing).
__global__ void k_repack_q4_tc(const uint8_t* __restrict__ packed, const __half* __restrict__ scales,
                               int n_rows, int k, uint8_t* __restrict__ blob, int R, int dst_off) {
  const int nc = k / kTcChunkK;
  const size_t total = (size_t)(n_rows / R) * nc * 2 * R;
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int r = (int)(idx % R);
  const int h = (int)((idx / R) % 2);
  const size_t tc = idx / (2 * (size_t)R);  // tile * nc + chunk
  const int c = (int)(tc % nc);
  const size_t row = (tc / nc) * R + r;
  const int rr = dst_off + r;
  const uint4 src = *reinterpret_cast<const uint4*>(packed + row * (k / 2) + (size_t)(c * 2 + h) * 16);
  const uint4 dst = make_uint4(permute_nibbles(src.x), permute_nibbles(src.y),
                               permute_nibbles(src.z), permute_nibbles(src.w));
  uint8_t* chunk = blob + tc * kQ4TcChunkBytes;
  *reinterpret_cast<uint4*>(chunk + h * 2048 + rr * 16) = dst;
  *reinterpret_cast<__half*>(chunk + 4096 + rr * 4 + h * 2) = scales[row * (k / 32) + c * 2 + h];
}

__global__ void k_repack_f16_tc(const __half* __restrict__ w, int n_rows, int k,
                                uint8_t* __restrict__ blob) {
  const int nc = k / kTcChunkK;
  const size_t total = (size_t)(n_rows / kTcM) * nc * kTcM * 8;
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int j = (int)(idx % 8);
  const int r = (int)((idx / 8) % kTcM);
  const size_t tc = idx / (8 * kTcM);
  const int c = (int)(tc % nc);
  const size_t row = (tc / nc) * kTcM + r;
  const uint4 v = *reinterpret_cast<const uint4*>(w + row * k + (size_t)c * kTcChunkK + j * 8);
  *reinterpret_cast<uint4*>(blob + tc * kF16TcChunkBytes + r * 128 + ((j ^ (r & 7)) << 4)) = v;
}

__global__ void k_pack_act(const __half* __restrict__ x, long long ld, int rows, int k, int nb,
                           uint8_t* __restrict__ act) {
  const size_t total = (size_t)(k / kTcChunkK) * nb * 8;
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int j = (int)(idx % 8);
  const int b = (int)((idx / 8) % nb);
  const size_t c = idx / (8 * (size_t)nb);
  uint4 v = make_uint4(0, 0, 0, 0);
  if (b < rows) v = *reinterpret_cast<const uint4*>(x + (size_t)b * ld + c * kTcChunkK + j * 8);
  *reinterpret_cast<uint4*>(act + (c * nb + b) * 128 + ((j ^ (b & 7)) << 4)) = v;
}

__global__ void k_splits_to_f16(const float* __restrict__ part, int splits, int nbv, int n,
                                const __half* __restrict__ bias, __half* __restrict__ y,
                                long long ld) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (size_t)nbv * n) return;
  const int col = (int)(idx % n);
  const size_t b = idx / n;
  float s = 0.0f;
  for (int sp = 0; sp < splits; ++sp) s += part[((size_t)sp * nbv + b) * n + col];
  if (bias) s += h2f(bias[col]);
  y[b * ld + col] = f2h(s);
}

inline unsigned blocks_for(size_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace

size_t tc_gemm_smem_bytes(int nb, bool q4, int stages, int xstages, int raw_stages, int unit) {
  const int rs = q4 ? raw_stages : 0;
  const int nw = q4 ? rs : stages;
  const int sa = q4 ? 0 : stages;  // Q4 A stages live in tensor memory
  return 1024 + (size_t)sa * kF16TcChunkBytes + (size_t)xstages * unit * nb * 128 +
         (size_t)rs * unit * kQ4TcChunkBytes + 8 * (size_t)(nw + rs + 2 * xstages + 2 * stages + 1) +
         8;
}

// Ring depths (in pipeline units of `unit` chunks) for nu units per CTA within
// 227 KB of shared memory.  Q4: 4 A stages in tensor memory; the activation
// ring (at most 12 chunks, at least min(nu, 4) units) with room left for
// min(nu, 8) raw units, then the raw ring with the rest (at most 32 units; a
// multiple of the dequantising group count unless it holds every unit).  fp16:
// activation ring of min(nu, 4), shared-memory A ring (HBM weights) of up to
// 4: at 64 activation rows two CTAs then share an SM, which the LM head's many
// tiles need more than depth.
void tc_gemm_rings(int nb, bool q4, int nu, int unit, int* stages, int* xstages, int* raw_stages) {
  auto lim = [](int v, int hi) { return v < hi ? v : hi; };
  if (!q4) {
    const int xs = lim(nu, 4) < 2 ? 2 : lim(nu, 4);
    int st = kTcMaxF16Stages;
    while (st > 2 && tc_gemm_smem_bytes(nb, false, st, xs, 0, 1) > kTcSmemBudget) --st;
    *stages = st;
    *xstages = xs;
    *raw_stages = 0;
    return;
  }
  const int st = kTcMaxStages;
  const int rs_min = lim(nu, 8);
  // At least min(nu, st) activation stages: a dequantising warp waits for the
  // activations of unit i once the MMAs of unit i - st completed, so the
  // previous fill of its slot (unit i - xs) has landed and the parity wait
  // cannot alias it.
  const int xs_min = lim(nu, st) < 2 ? 2 : lim(nu, st);
  int xs = lim(nu, kTcMaxXStages / unit);
  if (xs < xs_min) xs = xs_min;
  while (xs > xs_min && tc_gemm_smem_bytes(nb, true, st, xs, rs_min, unit) > kTcSmemBudget) --xs;
  // A refilled activation ring has an even depth: with two MMA warps (units
  // alternate between them) the MMAs of unit i - st having completed implies
  // those of unit i - xs only when the two units share a warp.
  if (xs < nu && (xs & 1)) --xs;
  int rs = lim(nu, kTcMaxRawStages);
  while (rs > 2 && tc_gemm_smem_bytes(nb, true, st, xs, rs, unit) > kTcSmemBudget) --rs;
  // A ring that is refilled must have a depth that is a multiple of the group
  // count: unit i then reuses the slot of unit i - rs of the same dequantising
  // group, which that group has already read, so its parity wait can never
  // alias a fill two phases back.
  if (rs < nu) rs -= rs % kDeqGroups;
  if (rs == 0) rs = kDeqGroups < nu ? kDeqGroups : nu;
  *stages = st;
  *xstages = xs;
  *raw_stages = rs;
}

// Launch plan of a GEMM with cps chunks per CTA: unit size, ring depths, MMA
// warps and dequantising groups, shared memory.  smem > the budget: no plan.
struct TcLaunchPlan {
  int unit, stages, xstages, raw_stages, mma_warps, groups;
  size_t smem;
};
static TcLaunchPlan tc_gemm_plan(int nb, bool q4, int cps) {
  TcLaunchPlan pl{};
  pl.groups = q4 ? kDeqGroups : kF16DeqGroups;
  // Two-chunk units (half the waits and commits per MMA) where the chunk count
  // is even and the rings still fit; else single chunks.
  for (int u = (q4 && cps % 2 == 0) ? 2 : 1; u >= 1; --u) {
    pl.unit = u;
    tc_gemm_rings(nb, q4, cps / u, u, &pl.stages, &pl.xstages, &pl.raw_stages);
    pl.smem = tc_gemm_smem_bytes(nb, q4, pl.stages, pl.xstages, pl.raw_stages, u);
    if (pl.smem <= kTcSmemBudget) break;
  }
  // A second MMA warp (and accumulator) where both accumulators and the A
  // stages fit in the 512 tensor-memory columns.
  const int acc = nb <= 32 ? 32 : nb <= 64 ? 64 : nb <= 128 ? 128 : 256;
  const int astage = q4 ? pl.stages * pl.unit * 32 : 0;
  pl.mma_warps = (2 * acc + astage <= 512) ? 2 : 1;
  return pl;
}

int launch_tc_gemm(const TcGemmArgs& a, cudaStream_t st) {
  if (!a.w || !a.act || a.n_rows <= 0 || a.n_rows % kTcM || a.k <= 0 || a.k % kTcChunkK ||
      a.nb < 16 || a.nb > kTcMaxNb || a.nb % 16 || a.nb_valid < 1 || a.nb_valid > a.nb ||
      a.splits < 1 || (a.k / kTcChunkK) % a.splits ||
      (a.act_stride_rows != 0 && (a.act_stride_rows < a.nb || a.act_stride_rows % 16)))
    return -1;
  const int outs = (a.part ? 1 : 0) + (a.out ? 1 : 0) + (a.swiglu_act ? 1 : 0);
  if (outs != 1 || (!a.part && a.splits != 1) ||
      (a.swiglu_act && (a.swiglu_nb < a.nb_valid || !a.q4)))
    return -1;
  TcGemmArgs args = a;
  const TcLaunchPlan pl = tc_gemm_plan(a.nb, a.q4, (a.k / kTcChunkK) / a.splits);
  if (pl.smem > kTcSmemBudget) return -1;
  args.unit = pl.unit;
  args.stages = pl.stages;
  args.xstages = pl.xstages;
  args.raw_stages = pl.raw_stages;
  args.mma_warps = pl.mma_warps;
  const size_t smem = pl.smem;
  void (*kernel)(TcGemmArgs) = a.q4 ? k_tc_gemm<kDeqGroups> : k_tc_gemm<kF16DeqGroups>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_rows / kTcM, a.splits);
  cfg.blockDim = dim3(tc_threads(a.q4 ? kDeqGroups : kF16DeqGroups));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args) == cudaSuccess ? 0 : -1;
}

int launch_repack_q4_tc_rows(const uint8_t* packed, const __half* scales, int n_rows, int k,
                             uint8_t* blob, int src_rows_per_tile, int dst_row_offset,
                             cudaStream_t st) {
  const int R = src_rows_per_tile;
  if (R < 1 || R > kTcM || dst_row_offset < 0 || dst_row_offset + R > kTcM || n_rows % R ||
      k % kTcChunkK)
    return -1;
  const size_t total = (size_t)(n_rows / R) * (k / kTcChunkK) * 2 * R;
  k_repack_q4_tc<<<blocks_for(total, 256), 256, 0, st>>>(packed, scales, n_rows, k, blob, R,
                                                         dst_row_offset);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_repack_q4_tc(const uint8_t* packed, const __half* scales, int n_rows, int k,
                        uint8_t* blob, cudaStream_t st) {
  return launch_repack_q4_tc_rows(packed, scales, n_rows, k, blob, kTcM, 0, st);
}

int launch_repack_f16_tc(const __half* w, int n_rows, int k, uint8_t* blob, cudaStream_t st) {
  if (n_rows % kTcM || k % kTcChunkK) return -1;
  const size_t total = (size_t)(n_rows / kTcM) * (k / kTcChunkK) * kTcM * 8;
  k_repack_f16_tc<<<blocks_for(total, 256), 256, 0, st>>>(w, n_rows, k, blob);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_pack_act(const __half* x, long long ld, int rows, int k, int nb, uint8_t* act,
                    cudaStream_t st) {
  if (k % kTcChunkK || nb % 16 || rows > nb || ld % 8) return -1;
  const size_t total = (size_t)(k / kTcChunkK) * nb * 8;
  k_pack_act<<<blocks_for(total, 256), 256, 0, st>>>(x, ld, rows, k, nb, act);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_splits_to_f16(const float* part, int splits, int nb_valid, int n_rows,
                         const __half* bias, __half* y, long long ld_y, cudaStream_t st) {
  const size_t total = (size_t)nb_valid * n_rows;
  k_splits_to_f16<<<blocks_for(total, 256), 256, 0, st>>>(part, splits, nb_valid, n_rows, bias, y,
                                                           ld_y);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace qwen

// Test hook (not part of the public header): the plan launch_tc_gemm would use
// for nb activation rows and cps chunks per CTA, as {unit, stages, xstages,
// raw_stages, mma_warps, dequant groups, shared memory bytes}.  Host
// arithmetic only.  Returns 0, or -1 when no plan fits shared memory.
extern "C" int qwen_tc_gemm_plan(int nb, int q4, int cps, long long* out7) {
  if (!out7 || nb < 16 || nb > qwen::kTcMaxNb || nb % 16 || cps < 1) return -1;
  const auto pl = qwen::tc_gemm_plan(nb, q4 != 0, cps);
  const long long v[7] = {pl.unit, pl.stages, pl.xstages, pl.raw_stages, pl.mma_warps, pl.groups,
                          (long long)pl.smem};
  for (int i = 0; i < 7; ++i) out7[i] = v[i];
  return pl.smem <= qwen::kTcSmemBudget ? 0 : -1;
}
