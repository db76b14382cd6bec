// qwen_common.cuh -- shared device helpers for the sm_100a decode kernels.
//
// Model constants follow QwenConfig.swift:10-22.  PTX wrappers cover the
// Blackwell/Hopper async machinery used by the kernels: mbarriers with
// transaction counts, cp.async.bulk (TMA bulk copies global -> shared),
// programmatic dependent launch, acquire/release counters between CTAs, and
// the m16n8k16 f16 MMA used to contract dequantised int4 tiles.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qwen {

constexpr int kHidden = 1536;        // QwenConfig.hiddenDim
constexpr int kInter = 8960;         // QwenConfig.mlpIntermediate
constexpr int kLayers = 28;          // QwenConfig.numLayers
constexpr int kHeads = 12;           // QwenConfig.numAttnHeads
constexpr int kKVHeads = 2;          // QwenConfig.numKVHeads
constexpr int kHeadDim = 128;        // QwenConfig.headDim
constexpr int kKVDim = 256;          // QwenConfig.kDim
constexpr int kQKVRows = kHidden + 2 * kKVDim;  // 2048
constexpr int kVocab = 151936;       // QwenConfig.vocabSize (padded rows)
constexpr int kActualVocab = 151666; // QwenConfig.actualVocabSize
constexpr int kStopToken = 151645;   // <|im_end|>, InferenceEngine.swift:41,291,314
constexpr float kAttnScale = 0.088388f;  // attention.metal:30
constexpr float kRmsEps = 1e-6f;         // rmsnorm.metal:39

// Error codes written to the device error word (first error wins).
enum DeviceError : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,   // a bounded spin on an mbarrier or counter gave up
  kDevBadArgument = 2,   // a kernel saw an out-of-range size or index
};

// ---------------------------------------------------------------- fp16 ----
__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }
__device__ __forceinline__ __half f2h(float f) { return __float2half_rn(f); }
__device__ __forceinline__ uint16_t hbits(__half h) { return __half_as_ushort(h); }

// SiLU with the reference's clamps (activations.metal:9-27).
__device__ __forceinline__ float silu_ref(float x) {
  if (x > 15.0f) return x;
  if (x < -15.0f) return 0.0f;
  return x / (1.0f + expf(-x));
}

// --------------------------------------------------------------- errors ---
__device__ __forceinline__ void raise_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------------------------- mbarrier ---
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and records kDevWaitTimeout) after `limit`
// polls.  Every poll of try_wait already suspends for a hardware-defined
// interval, so the limit bounds the wait in time.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err,
                                          uint32_t limit = (1u << 22)) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  raise_error(err, kDevWaitTimeout);
  return false;
}

// ------------------------------------------------- TMA bulk copy (1-D) ----
// global -> shared, completion reported as transaction bytes on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Same, with an L2 eviction-first hint: streamed weights are read once per step.
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes,
                                                uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------------------------ dependent launch (PDL) --
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------ inter-CTA counters (gpu scope) -
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add_u32(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_acq_rel_add_u32(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}
// Bounded spin until *p >= target.  Returns false on timeout (error recorded).
__device__ __forceinline__ bool spin_until_geq(const uint32_t* p, uint32_t target, int* err,
                                               uint32_t limit = (1u << 24)) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (ld_acquire_u32(p) >= target) return true;
    if (i > 64) __nanosleep(64);
    // Another CTA already gave up: stop waiting for it.
    if (err && (i & 255) == 255 && *((volatile int*)err) != 0) return false;
  }
  raise_error(err, kDevWaitTimeout);
  return false;
}

// --------------------------------------------------------- MMA m16n8k16 ---
// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1, const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
        "f"(c[2]), "f"(c[3]));
}

// ------------------------------------------------------- int4 dequant -----
// One 32-bit word of a Q4 row holds 8 consecutive k (byte j: element 2j in the
// low nibble, 2j+1 in the high nibble; matmul.metal:37-39).  Returns four
// half2 values of (q - 8), exact in fp16:
//   out[0] = (k0, k4), out[1] = (k1, k5), out[2] = (k2, k6), out[3] = (k3, k7).
// The low nibbles become 1024+q via the fp16 exponent trick and are shifted by
// -1032; the high nibbles become 1024+16q and are mapped by q' = x/16 - 72.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t (&out)[4]) {
  const uint32_t kLo = 0x000f000fu, kHi = 0x00f000f0u, kEx = 0x64006400u;
  const uint32_t t0 = lop3_and_or(w, kLo, kEx);
  const uint32_t t1 = lop3_and_or(w, kHi, kEx);
  const uint32_t w8 = w >> 8;
  const uint32_t t2 = lop3_and_or(w8, kLo, kEx);
  const uint32_t t3 = lop3_and_or(w8, kHi, kEx);
  const uint32_t k1032 = 0x64086408u, kSixteenth = 0x2c002c00u, kMinus72 = 0xd480d480u;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(out[0]) : "r"(t0), "r"(k1032));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out[1]) : "r"(t1), "r"(kSixteenth), "r"(kMinus72));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(out[2]) : "r"(t2), "r"(k1032));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out[3]) : "r"(t3), "r"(kSixteenth), "r"(kMinus72));
}

// One Q4 block (32 k) for the 16 rows of an m16 tile, column-replicated x.
//   wg, wg8: the word this lane owns in rows g and g+8 (word t of the block,
//            t = lane & 3, i.e. k = 32b + 8t .. 8t+7)
//   xf:      the lane's x fragment for the block, 4 half2:
//            (x0,x4), (x1,x5), (x2,x6), (x3,x7) relative to 32b + 8t
// Returns the block's dot products for rows g (d[0]) and g+8 (d[2]), exact
// products accumulated in fp32, before the block scale.
__device__ __forceinline__ void q4_block_mma(uint32_t wg, uint32_t wg8, const uint4& xf,
                                             float (&d)[4]) {
  uint32_t ag[4], ag8[4];
  dequant_word(wg, ag);
  dequant_word(wg8, ag8);
  const float z[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t a1[4] = {ag[0], ag8[0], ag[1], ag8[1]};
  mma_16816(d, a1, xf.x, xf.y, z);
  const uint32_t a2[4] = {ag[2], ag8[2], ag[3], ag8[3]};
  mma_16816(d, a2, xf.z, xf.w, d);
}

// Build the x fragment of block b for lane quad t from 8 consecutive fp16 x
// values x[32b+8t .. 32b+8t+7] (v0..v7).
__device__ __forceinline__ uint4 make_xfrag(const __half (&v)[8]) {
  uint4 r;
  r.x = (uint32_t)hbits(v[0]) | ((uint32_t)hbits(v[4]) << 16);
  r.y = (uint32_t)hbits(v[1]) | ((uint32_t)hbits(v[5]) << 16);
  r.z = (uint32_t)hbits(v[2]) | ((uint32_t)hbits(v[6]) << 16);
  r.w = (uint32_t)hbits(v[3]) | ((uint32_t)hbits(v[7]) << 16);
  return r;
}

// Offset form of q4_block_mma for the fused kernels.  The MMA takes the raw
// exponent-trick halves -- 1024+q for the low nibbles, 1024+16q for the high
// nibbles -- against x for the low nibbles and x/16 for the high ones, and the
// constant part cancels through the accumulator input:
//   sum (q-8) x = D - c_b,  c_b = 1032 * sum_even x + 1152 * sum_odd (x/16)
// (exact in real arithmetic; the fp32 accumulation carries the 1024 offset,
// costing ~2^-24 * 4096 per block).  neg_c = -c_b of the block.
__device__ __forceinline__ void raw_word(uint32_t w, uint32_t (&out)[4]) {
  const uint32_t kLo = 0x000f000fu, kHi = 0x00f000f0u, kEx = 0x64006400u;
  out[0] = lop3_and_or(w, kLo, kEx);
  out[1] = lop3_and_or(w, kHi, kEx);
  const uint32_t w8 = w >> 8;
  out[2] = lop3_and_or(w8, kLo, kEx);
  out[3] = lop3_and_or(w8, kHi, kEx);
}
__device__ __forceinline__ void q4_block_mma_off(uint32_t wg, uint32_t wg8, const uint4& xf,
                                                 float neg_c, float (&d)[4]) {
  uint32_t ag[4], ag8[4];
  raw_word(wg, ag);
  raw_word(wg8, ag8);
  const float c[4] = {neg_c, neg_c, neg_c, neg_c};
  const uint32_t a1[4] = {ag[0], ag8[0], ag[1], ag8[1]};
  mma_16816(d, a1, xf.x, xf.y, c);
  const uint32_t a2[4] = {ag[2], ag8[2], ag[3], ag8[3]};
  mma_16816(d, a2, xf.z, xf.w, d);
}
// x fragment for the offset form: the high-nibble partners (odd k) are divided
// by 16 (an exact power-of-two scaling for normal fp16 values).
__device__ __forceinline__ uint4 make_xfrag_hi16(const __half (&v)[8]) {
  const __half k16 = __ushort_as_half((unsigned short)0x2c00u);  // 1/16
  __half h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = (i & 1) ? __hmul(v[i], k16) : v[i];
  return make_xfrag(h);
}
// -c_b of block b from its four offset-form fragments (fixed summation order).
__device__ __forceinline__ float block_neg_corr(const uint4* frag4) {
  float even = 0.f, odd = 0.f;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint4 f = frag4[t];
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&f.x));  // x0, x4
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&f.y));  // x1/16, x5/16
    const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&f.z));  // x2, x6
    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&f.w));  // x3/16, x7/16
    even += (a.x + a.y) + (c.x + c.y);
    odd += (b.x + b.y) + (d.x + d.y);
  }
  return -(1032.0f * even + 1152.0f * odd);
}

// Warp-wide sums.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace qwen
