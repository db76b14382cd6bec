// tc_gemm.cu -- batched Q4 / fp16 projections on tcgen05 tensor cores.
//
// CTA = 128 output rows x nb activation rows, K split over grid.y.  Ten warps:
//   warp 8      producer: one lane issues the 1-D bulk copies of each K chunk
//               into a 4-stage ring: the weight blob chunk (completion on
//               wfull[s]) and the activation chunk (xfull[s]).  Launched as a
//               programmatic dependent, the first stages' weights are fetched
//               before griddepcontrol.wait, i.e. while the previous kernel of
//               the stream still runs; activations only after it.
//   warps 0..7  Q4: thread (h, r) dequantises block h of row r of the chunk
//               (16 nibble pairs -> fp16 via the 0x6400 exponent trick, (q - 8)
//               exact, one rounding for the product with the block scale) into
//               the 128-byte-swizzled A tile; then the epilogue: warp w reads
//               tensor-memory lanes 32(w%4).. (its rows) for half w/4 of the
//               columns
//   warp 9      allocates tensor memory; one lane issues 4 MMAs
//               (M=128, N=nb, K=16) per chunk and commits each stage back to
//               the producer through empty[s]
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

constexpr int kTcMaxStages = 4;  // deeper rings measured slower (one CTA per SM instead of two)
constexpr int kTcThreads = 320;   // warps 0-7 dequant + epilogue, 8 producer, 9 MMA
constexpr int kDeqThreads = 256;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
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

// 8 nibble-permuted weights -> 4 half2 (k0,k1) (k2,k3) (k4,k5) (k6,k7),
// each (q - 8) * scale rounded once.
__device__ __forceinline__ uint4 dequant8(uint32_t w, __half2 s2) {
  const __half2 off = __floats2half2_rn(1032.0f, 1032.0f);
  uint32_t o[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t v = ((w >> (4 * s)) & 0x000F000Fu) | 0x64006400u;  // 1024 + q
    o[s] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(v), off), s2));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(kTcThreads, 1) k_tc_gemm(TcGemmArgs a) {
  extern __shared__ uint8_t tc_smem[];
  const int S = a.stages;  // ring depth (host-sized to the shared memory budget)
  const uint32_t pad = (1024u - (smem_u32(tc_smem) & 1023u)) & 1023u;
  uint8_t* sA = tc_smem + pad;                             // [S][128 rows][128 B]
  uint8_t* sX = sA + S * kF16TcChunkBytes;         // [S][nb rows][128 B]
  const int nb = a.nb;
  const uint32_t xbytes = (uint32_t)nb * 128u;
  const size_t act_chunk_bytes = (size_t)(a.act_stride_rows > 0 ? a.act_stride_rows : nb) * 128u;
  uint8_t* sR = sX + S * xbytes;                   // [S][4608] (Q4)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sR + (a.q4 ? S * kQ4TcChunkBytes : 0));
  uint64_t* wfull = bars;
  uint64_t* xfull = bars + S;
  uint64_t* deq = bars + 2 * S;
  uint64_t* empty = bars + 3 * S;
  uint64_t* accum = bars + 4 * S;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 4 * S + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_chunks = a.k / kTcChunkK;
  const int cps = n_chunks / a.splits;
  const int c0 = blockIdx.y * cps;
  const int tile = blockIdx.x;
  const uint32_t ncols = nb <= 32 ? 32u : nb <= 64 ? 64u : nb <= 128 ? 128u : 256u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(wfull + s, 1);
      mbar_init(xfull + s, 1);
      mbar_init(deq + s, kDeqThreads);
      mbar_init(empty + s, 1);
    }
    mbar_init(accum, 1);
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
      const uint32_t wbytes = a.q4 ? kQ4TcChunkBytes : kF16TcChunkBytes;
      auto load_w = [&](int i) {
        const int s = i % S;
        mbar_arrive_expect_tx(wfull + s, wbytes);
        uint8_t* wdst = a.q4 ? sR + s * kQ4TcChunkBytes : sA + s * kF16TcChunkBytes;
        bulk_g2s_stream(wdst, a.w + ((size_t)tile * n_chunks + c0 + i) * wbytes, wbytes, wfull + s,
                        pol);
      };
      auto load_x = [&](int i) {
        const int s = i % S;
        mbar_arrive_expect_tx(xfull + s, xbytes);
        bulk_g2s(sX + s * xbytes, a.act + (size_t)(c0 + i) * act_chunk_bytes, xbytes, xfull + s);
      };
      const int pre = cps < S ? cps : S;
      for (int i = 0; i < pre; ++i) load_w(i);  // weights do not depend on earlier kernels
      pdl_wait();
      for (int i = 0; i < pre; ++i) load_x(i);
      int i = pre;
      for (; i < cps; ++i) {
        const int s = i % S;
        if (!tc_wait(empty + s, ((i / S) - 1) & 1, abort, a.err)) break;
        load_w(i);
        load_x(i);
      }
      // Every issued copy lands before the CTA may exit.
      for (int j = i > S ? i - S : 0; j < i; ++j) {
        tc_wait(wfull + j % S, (j / S) & 1, abort, a.err, false);
        tc_wait(xfull + j % S, (j / S) & 1, abort, a.err, false);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // --------------------------------------------------------------- MMA --
    if (lane == 0) {
      const uint32_t idesc = f16_idesc(kTcM, nb);
      for (int i = 0; i < cps; ++i) {
        const int s = i % S;
        if (!tc_wait(a.q4 ? deq + s : wfull + s, (i / S) & 1, abort, a.err)) break;
        if (!tc_wait(xfull + s, (i / S) & 1, abort, a.err)) break;
        tc_fence_after();
        const uint64_t ad = sw128_kmajor_desc(smem_u32(sA + s * kF16TcChunkBytes));
        const uint64_t bd = sw128_kmajor_desc(smem_u32(sX + s * xbytes));
#pragma unroll
        for (int kk = 0; kk < kTcChunkK / 16; ++kk)  // +32 B of k per MMA inside the atom
          tc_mma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
        tc_commit(empty + s);
      }
      tc_commit(accum);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------- dequant (Q4 only) --
    // Thread (h, r): block h (32 k) of row r of the chunk.
    const int r = threadIdx.x & (kTcM - 1), h = threadIdx.x >> 7;
    if (a.q4) {
      for (int i = 0; i < cps; ++i) {
        const int s = i % S;
        if (!tc_wait(wfull + s, (i / S) & 1, abort, a.err)) break;
        const uint8_t* raw = sR + s * kQ4TcChunkBytes;
        const uint4 pk = *reinterpret_cast<const uint4*>(raw + h * 2048 + r * 16);
        const __half2 s2 = __half2half2(*reinterpret_cast<const __half*>(raw + 4096 + r * 4 + h * 2));
        uint8_t* arow = sA + s * kF16TcChunkBytes + r * 128;
        const uint32_t sw = (uint32_t)(r & 7), j0 = 4u * (uint32_t)h;
        *reinterpret_cast<uint4*>(arow + (((j0 + 0u) ^ sw) << 4)) = dequant8(pk.x, s2);
        *reinterpret_cast<uint4*>(arow + (((j0 + 1u) ^ sw) << 4)) = dequant8(pk.y, s2);
        *reinterpret_cast<uint4*>(arow + (((j0 + 2u) ^ sw) << 4)) = dequant8(pk.z, s2);
        *reinterpret_cast<uint4*>(arow + (((j0 + 3u) ^ sw) << 4)) = dequant8(pk.w, s2);
        fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
        mbar_arrive(deq + s);
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
    const int groups = nb / 16, gsplit = (groups + 1) / 2;
    const int g0 = h == 0 ? 0 : gsplit, g1 = h == 0 ? gsplit : groups;
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    if (a.swiglu_act) {
      // Up rows (lanes 64..127) -> fp16 in shared memory [b][64] (the A ring
      // is idle once the accumulator is complete), then the gate-row warps
      // combine them.
      __half* ub = reinterpret_cast<__half*>(sA);
      if (go && r >= 64)
        for (int c = 16 * g0; c < 16 * g1; c += 16) {
          float v[16];
          tmem_ld16(lane_addr + (uint32_t)c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) ub[(c + j) * 64 + (r - 64)] = f2h(v[j]);
        }
      asm volatile("bar.sync 2, 256;" ::: "memory");  // the eight epilogue warps
      if (go && r < 64) {
        const int hrow = tile * 64 + r;  // k index of the down projection's input
        const int cc = hrow >> 6, jj = (hrow >> 3) & 7;
        for (int c = 16 * g0; c < 16 * g1; c += 16) {
          float v[16];
          tmem_ld16(lane_addr + (uint32_t)c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int b = c + j;
            if (b < a.nb_valid) {
              const float gt = h2f(f2h(v[j])), up = h2f(ub[b * 64 + r]);
              const size_t off = ((size_t)cc * a.swiglu_nb + b) * 128 +
                                 (((uint32_t)jj ^ (uint32_t)(b & 7)) << 4) + (hrow & 7) * 2;
              *reinterpret_cast<__half*>(a.swiglu_act + off) = f2h(silu_ref(gt) * up);
            }
          }
        }
      }
    } else if (go) {
      const size_t row = (size_t)tile * kTcM + r;
      for (int c = 16 * g0; c < 16 * g1; c += 16) {
        float v[16];
        tmem_ld16(lane_addr + (uint32_t)c, v);
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

size_t tc_gemm_smem_bytes(int nb, bool q4, int stages) {
  return 1024 + (size_t)stages * kF16TcChunkBytes + (size_t)stages * nb * 128 +
         (q4 ? (size_t)stages * kQ4TcChunkBytes : 0) + (4 * stages + 1) * 8 + 16;
}

// The deepest ring (up to 4 stages) that fits one CTA's shared memory.
int tc_gemm_stages(int nb, bool q4) {
  int st = kTcMaxStages;
  while (st > 2 && tc_gemm_smem_bytes(nb, q4, st) > 227 * 1024) --st;
  return st;
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
  args.stages = tc_gemm_stages(a.nb, a.q4);
  const size_t smem = tc_gemm_smem_bytes(a.nb, a.q4, args.stages);
  if (cudaFuncSetAttribute(k_tc_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_rows / kTcM, a.splits);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_tc_gemm, args) == cudaSuccess ? 0 : -1;
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
