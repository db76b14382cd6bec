// decode_fused.cu -- the whole decode step (28 layers + final norm + LM head)
// as one persistent kernel, one CTA per SM.
//
// Replaces the 506 dispatches of InferenceEngine.swift:103-264 per token.
//
// Inside a CTA (256 threads, 8 warps): Q4 dequant + m16n8k16 MMA GEMVs on a
// ring of shared-memory weight slots, with fused prologues (RMSNorm) and
// epilogues (bias, RoPE, KV-cache write, SwiGLU, residual add), and the
// split-K attention.  The ring streams this CTA's share of every weight byte
// of the step, in consumption order, with TMA bulk copies (cp.async.bulk +
// mbarrier transaction counts): the first 14 items at start, then item i + 14
// as soon as the warps have released item i, issued by the warp whose release
// completes it.  Weights do not depend on activations, so streaming runs ahead
// across the dependency waits.  (No separate producer warp: 8 warps are 2 per
// SM sub-partition, so a thread may hold 255 registers; 9 warps capped it at
// 168 and the GEMV loops spilled.)
//
// Cross-CTA data (x, q, new k/v, attention partials and output, the SwiGLU
// output h) travels as tagged words: a 32-bit word holds the fp16 value and a
// 16-bit tag of (step, write instance); a reader polls until every word it
// needs carries the expected tag.  Value and tag share one single-copy-atomic
// store, so no fences or grid barriers are needed and each dependency costs
// one L2 round trip.  Every wait is bounded; on timeout the kernel records
// QWEN_ERR_DEVICE_TIMEOUT, skips the remaining work (keeping every named
// barrier in step) and drains its in-flight copies before exiting.
//
// Rounding points follow the reference: q/k/v, o, gate/up, down outputs and
// logits are rounded to fp16 (matmul.metal:71,111), RoPE re-rounds q/k
// (rope.metal:37-38), the residual adds are fp16 adds (attention.metal:64),
// RMSNorm rounds twice (rmsnorm.metal:44), SwiGLU rounds once
// (activations.metal:26) and the attention output once (attention.metal:55).
#include <algorithm>
#include <cstring>

#include "engine.h"
#include "fused.h"
#include "qwen_common.cuh"
#include "status.h"

namespace qwen {

namespace {

constexpr int kNS = 14;                    // ring slots
// The down strip: kWarpsPerDownItem warps share each of the kDownItems items.
constexpr int kWarpsPerDownItem = kConsumerWarps / kDownItems;                 // 2
constexpr int kDownRowTilesPerWarp = kDownItemTiles / kWarpsPerDownItem;       // 12
static_assert(kWarpsPerDownItem * kDownItems == kConsumerWarps, "warps per down item");
// A round of the down strip: 6 row tiles, MMA chains in groups of three, stores by tile pairs.
constexpr int kDownRound = 6;
static_assert(kDownRowTilesPerWarp % kDownRound == 0, "down row tiles a warp: whole rounds");
// Rows of the layer output each CTA finishes, and the partial sums it reads.
// (CTA b finishes rows [b*1536/grid, (b+1)*1536/grid): at most ceil(1536/grid)
// <= ceil(1536/140) = 11 of them, as the grid has at least kMlpUnits CTAs.)
constexpr int kMaxReduceRows = (kHidden + kMlpUnits - 1) / kMlpUnits;
constexpr int kReducePerThread = (kMaxReduceRows * kMlpUnits + kFusedThreads - 1) / kFusedThreads;
constexpr int kUnionBytes = 20480;         // x fragments + corrections / attention buffers
constexpr int kMaxXFrags = kInter / 8;     // 1120 fragment units (K = 8960)
static_assert(kMaxXFrags * 16 <= kUnionBytes, "x fragments exceed the union");
// Every dependency wait gives up after FusedParams::wait_ns (2 s by default).
// The final drain of in-flight copies always allows 2 s: a CTA must not exit
// while a bulk copy may still write its shared memory.
constexpr uint64_t kDrainNs = 2000000000ull;

constexpr int kOffUnion = kNS * kSlotBytes;
constexpr int kOffXloc = kOffUnion + kUnionBytes;
constexpr int kOffXn = kOffXloc + kHidden * 2;
constexpr int kOffRed = kOffXn + kHidden * 2;
constexpr int kOffRed2 = kOffRed + kConsumerWarps * 16 * 4;
constexpr int kOffBars = kOffRed2 + 64;
constexpr int kOffMisc = kOffBars + 2 * kNS * 8;
constexpr int kMiscBytes = 128;
constexpr int kOffItems = kOffMisc + kMiscBytes;
// Trace stamps of this CTA (when tracing), kept in shared memory during the
// step and copied out at exit: a global store would make the next release's
// block-scope fence wait for it and distort what it measures.
constexpr int kMaxTraceStride = 3 + kLayers * kTraceStampsPerLayer + 2 + kAttnTraceStamps;
constexpr int kOffTrace = kOffItems + kMaxItemsPerCta * 8;
constexpr int kSmemBytes = kOffTrace + kMaxTraceStride * 8;

// attention buffers inside the union region
constexpr int kAVs = 0;                                   // [4][16][272] V rows
constexpr int kAPt = kAVs + kAttnWarpsFused * 16 * 272;   // [4][2][16*8] P^T hi/lo
constexpr int kAWm = kAPt + kAttnWarpsFused * 2 * 128 * 2;
constexpr int kAWl = kAWm + kAttnWarpsFused * 8 * 4;
constexpr int kAKnew = kAWl + kAttnWarpsFused * 8 * 4;    // [128] fp16 new k
constexpr int kAVnew = kAKnew + 256;                      // [128] fp16 new v
static_assert(kAVnew + 256 <= kUnionBytes, "attention buffers exceed the union region");
// MLP buffers inside the union region, after the gate/up x fragments (K = 1536).
constexpr int kOffHFrag = kHidden / 8 * 16;                  // [8] uint4: the unit's h fragments
constexpr int kOffMlpStage = kOffHFrag + kGUTilesPerUnit * 16;  // [rows][140] fp32 partials
static_assert(kOffMlpStage + kMaxReduceRows * kMlpUnits * 4 <= kUnionBytes,
              "MLP buffers exceed the union region");
// Merge factors, after the warp merge buffer (which aliases the dead V rows).
constexpr int kAFac = kAVs + kAttnWarpsFused * 6 * 128 * 4;  // 36 floats
constexpr int kACFac = kAFac + 256;                           // [74][2] + [6] floats
static_assert(kACFac + (kMaxAttnSplits * 2 + 8) * 4 <= kAPt, "merge factors exceed the V rows");
static_assert(kSmemBytes <= 232448, "shared memory budget");
static_assert(kAttnWarpsFused * 6 * 128 * 4 <= kAPt, "warp merge buffer aliases the V rows");

struct Misc {
  unsigned long long wait_ns;   // FusedParams::wait_ns
  int issued[kNS];              // bulk copies issued into each ring slot so far
  int abort;
  float scale;
  int cphase;           // phase the consumers are in (diagnostics)
  int last_rel[8];      // last item index each consumer warp released (diagnostics)
};

static_assert(sizeof(Misc) <= kMiscBytes, "Misc exceeds its shared-memory region");

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ void abar() { asm volatile("bar.sync 2, 128;" ::: "memory"); }


// ---------------------------------------------------------- tagged words --
__device__ __forceinline__ void st_tag16(uint32_t* p, uint16_t tag, __half v) {
  const uint32_t w = ((uint32_t)tag << 16) | (uint32_t)hbits(v);
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(w) : "memory");
}
__device__ __forceinline__ uint4 ld_tag4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_tag32(unsigned long long* p, uint16_t tag, float v) {
  const unsigned long long w =
      ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tag64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool tags_ok(const uint4& v, uint32_t tag) {
  return (v.x >> 16) == tag && (v.y >> 16) == tag && (v.z >> 16) == tag && (v.w >> 16) == tag;
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// True once this CTA or any other has given up.  A CTA that sees another's
// error raises its own abort flag first: a warp whose wait returned false
// releases its slot without the data having landed, and the flag is what stops
// that release from refilling the slot (release() checks it) -- a refill then
// could put a second copy in flight into the slot, or skip a ring lap so the
// exit drain would wait on the wrong phase.
__device__ __forceinline__ bool aborted(volatile Misc* m, const int* err) {
  if (m->abort != 0) return true;
  if (*((volatile const int*)err) != 0) {
    m->abort = 1;
    return true;
  }
  return false;
}
// Records the timeout and where it happened: err[1] = site, err[2] = CTA,
// err[3] = thread (the first failure wins).
__device__ __noinline__ void fail(volatile Misc* m, int* err, int site) {
  m->abort = 1;
  if (err && atomicCAS(err, 0, kDevWaitTimeout) == 0) {
    err[1] = site;
    err[2] = blockIdx.x;
    err[3] = threadIdx.x;
  }
}
// The abort flags and the time limit of a wait, looked at on one round in
// kWaitCheckEvery and never on the first: the abort check reads global
// memory, and a check on the first round would delay the round that sees the
// data by an L2 round trip whenever it arrives just after the first look.
// wait_check_slow returns the wait's start time (set at the first check) or
// kWaitStop once the wait must end (another CTA failed, or the limit passed).
constexpr uint32_t kWaitCheckEvery = 64;
constexpr uint64_t kWaitStop = ~0ull;
__device__ __noinline__ uint64_t wait_check_slow(uint64_t t0, volatile Misc* m, int* err, int site) {
  if (aborted(m, err)) return kWaitStop;
  const uint64_t now = globaltimer();
  if (t0 == 0) return now;
  if (now - t0 > m->wait_ns) {
    fail(m, err, site);
    return kWaitStop;
  }
  return t0;
}
__device__ __forceinline__ bool wait_check(uint32_t it, uint64_t& t0, volatile Misc* m, int* err,
                                           int site) {
  if (it % kWaitCheckEvery != kWaitCheckEvery - 1) return false;
  t0 = wait_check_slow(t0, m, err, site);
  return t0 == kWaitStop;
}

// Wait sites (x 100 + layer) reported by fail().
enum WaitSite : int {
  kSiteEmpty = 1, kSiteFull = 2, kSiteXIn = 3, kSiteQ = 4, kSiteKV = 5, kSiteCombine = 6,
  kSiteAttnOut = 7, kSiteXMid = 8, kSiteDownPart = 9, kSiteXFinal = 10
};

static_assert(kSiteDownPart == kFusedStallDownPart, "the stall hook's site is the partials poll");

// Polls units of 8 consecutive tagged fp16 words: unit u covers words
// [8u, 8u+8).  Thread `tid` of `nthr` owns units tid, tid+nthr, ... (at most
// MAXU).  f(u, v[8]) receives each unit once all its tags match.
template <int MAXU, class F>
__device__ __forceinline__ void poll_units(const uint32_t* src, int n_units, int tid, int nthr,
                                           uint32_t tag, volatile Misc* m, int* err, int site, F f) {
  uint32_t pending = 0;
  uint64_t t0 = 0;
#pragma unroll
  for (int j = 0; j < MAXU; ++j)
    if (tid + j * nthr < n_units) pending |= 1u << j;
  for (uint32_t it = 0; pending; ++it) {
    uint4 a[MAXU], b[MAXU];
#pragma unroll
    for (int j = 0; j < MAXU; ++j)
      if (pending & (1u << j)) {
        const uint32_t* p = src + 8 * (tid + j * nthr);
        a[j] = ld_tag4(p);
        b[j] = ld_tag4(p + 4);
      }
#pragma unroll
    for (int j = 0; j < MAXU; ++j)
      if ((pending & (1u << j)) && tags_ok(a[j], tag) && tags_ok(b[j], tag)) {
        __half v[8];
        const uint32_t w[8] = {a[j].x, a[j].y, a[j].z, a[j].w, b[j].x, b[j].y, b[j].z, b[j].w};
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = __ushort_as_half((unsigned short)(w[q] & 0xFFFFu));
        f(tid + j * nthr, v);
        pending &= ~(1u << j);
      }
    if (!pending) break;
    if (wait_check(it, t0, m, err, site)) return;
    // no sleep between rounds: a hop is on the step's critical path, and a
    // 32 ns back-off measured 0.8% slower end to end
  }
}

// The slow paths of the waits are out of line: the fast path (the data has
// landed) is what every item takes, and the step's per-layer code has to stay
// small enough for the SM's instruction cache.
__device__ __noinline__ bool slot_wait_slow(uint64_t* bar, uint32_t parity, volatile Misc* m,
                                            int* err, int site) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (wait_check(it, t0, m, err, site)) return false;
  }
}
__device__ __forceinline__ bool slot_wait(uint64_t* bar, uint32_t parity, volatile Misc* m,
                                          int* err, int site) {
  return mbar_try_wait(bar, parity) || slot_wait_slow(bar, parity, m, err, site);
}

// Waits for item i of this CTA's list to land in its ring slot.  A slot's
// mbarrier only tells the current phase from the previous one, so a warp
// that runs ahead (one that owns every 8th tile) first waits until item i has
// been issued into the slot (slot_item) -- from then on the slot's current
// phase is item i's and the parity wait is exact.
__device__ __noinline__ bool item_issue_wait_slow(int i, volatile const int* slot_item,
                                                  volatile Misc* m, int* err, int site) {
  uint64_t t0 = 0;
  for (uint32_t it = 0; slot_item[i % kNS] != i; ++it) {
    if (wait_check(it, t0, m, err, site)) return false;
    __nanosleep(32);
  }
  return true;
}
__device__ __forceinline__ bool item_wait(int i, uint64_t* full, volatile const int* slot_item,
                                          volatile Misc* m, int* err, int site) {
  if (slot_item[i % kNS] != i && !item_issue_wait_slow(i, slot_item, m, err, site)) return false;
  return slot_wait(&full[i % kNS], (i / kNS) & 1, m, err, site);
}


// RMSNorm of xloc (rmsnorm.metal:9-46): out = half(half(x * s) * gamma).
// Writes Q4 x fragments (frags) and/or plain fp16 (plain).  256 consumer threads.
// gamma_u: this thread's 8 gamma values (unit ct, threads < 192), loaded by
// the caller before its wait for x so the load is off the critical path.
__device__ __forceinline__ uint4 gamma_prefetch(const __half* __restrict__ gamma, int ct) {
  return ct < kHidden / 8 ? __ldg(reinterpret_cast<const uint4*>(gamma) + ct) : make_uint4(0, 0, 0, 0);
}

// RMSNorm of xloc (rmsnorm.metal:9-46): out = half(half(x * s) * gamma).
__device__ __forceinline__ void rmsnorm_out(const __half* xloc, uint4 gamma_u, float* red2,
                                            uint4* frags, __half* plain, int ct) {
  float ss = 0.f;
  for (int i = ct; i < kHidden; i += 256) {
    const float v = h2f(xloc[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((ct & 31) == 0) red2[ct >> 5] = ss;
  cbar();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) tot += red2[w];
  const float s = 1.0f / sqrtf(tot / 1536.0f + kRmsEps);
  if (ct < kHidden / 8) {
    __half v[8];
    const uint4 raw = reinterpret_cast<const uint4*>(xloc)[ct];
    const __half* xv = reinterpret_cast<const __half*>(&raw);
    const __half* gv = reinterpret_cast<const __half*>(&gamma_u);
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = __hmul(f2h(h2f(xv[q]) * s), gv[q]);
    if (frags) frags[ct] = make_xfrag(v);
    if (plain) reinterpret_cast<uint4*>(plain)[ct] = *reinterpret_cast<uint4*>(v);
  }
  cbar();
}

// Block pairs b = b_begin, b_begin + b_step, ... < b_end of a Q4 slot whose
// first block pair is k0 of its tile, for the lane's rows g and g+8.  Two
// block pairs per iteration keep four independent MMA chains in flight.
__device__ __forceinline__ void q4_bp(const uint8_t* slot, int k0, int b, const uint4* xf, int lane,
                                      float& ag, float& ag8) {
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* bp = slot + b * kBpBytes;
  const uint4 wv = *reinterpret_cast<const uint4*>(bp + lane * 16);
  const uint2 sv = *reinterpret_cast<const uint2*>(bp + 512 + g * 8);
  const int gp = k0 + b;
  const uint4 x0 = xf[(2 * gp) * 4 + t];
  const uint4 x1 = xf[(2 * gp + 1) * 4 + t];
  float d0[4], d1[4];
  q4_block_mma(wv.x, wv.y, x0, d0);
  q4_block_mma(wv.z, wv.w, x1, d1);
  const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&sv.x));
  const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&sv.y));
  ag = fmaf(s0.x, d0[0], ag);
  ag8 = fmaf(s0.y, d0[2], ag8);
  ag = fmaf(s1.x, d1[0], ag);
  ag8 = fmaf(s1.y, d1[2], ag8);
}

__device__ __forceinline__ void q4_chunk(const uint8_t* slot, int k0, int b_begin, int b_end,
                                         int b_step, const uint4* xf, int lane, float& acc_g,
                                         float& acc_g8) {
  float ga = 0.f, g8a = 0.f, gb = 0.f, g8b = 0.f;
  int b = b_begin;
  for (; b + b_step < b_end; b += 2 * b_step) {
    q4_bp(slot, k0, b, xf, lane, ga, g8a);
    q4_bp(slot, k0, b + b_step, xf, lane, gb, g8b);
  }
  if (b < b_end) q4_bp(slot, k0, b, xf, lane, ga, g8a);
  acc_g += ga + gb;
  acc_g8 += g8a + g8b;
}

// Same with three block pairs in flight: the single-tile phases (QKV, O) give
// each warp 3 strided block pairs, which q4_chunk runs as a pair then a tail,
// two dependent rounds; the down ranges (17-18 pairs a warp) gain from the
// third chain too now that registers do not spill.
// Warp w's share of a whole-tile item (24 block pairs, K-split over the 8
// warps): block pairs w, w + 8, w + 16, three MMA chains in flight.  Straight
// code: the step's per-layer code has to stay small enough for the SM's
// instruction cache, and a loop here unrolls into several copies.
static_assert(kBp1536 == 3 * kConsumerWarps, "a whole-tile item is three block pairs a warp");
__device__ __forceinline__ void q4_kslice3(const uint8_t* slot, int warp, const uint4* xf, int lane,
                                           float& acc_g, float& acc_g8) {
  float ga = 0.f, g8a = 0.f, gb = 0.f, g8b = 0.f, gc = 0.f, g8c = 0.f;
  q4_bp(slot, 0, warp, xf, lane, ga, g8a);
  q4_bp(slot, 0, warp + kConsumerWarps, xf, lane, gb, g8b);
  q4_bp(slot, 0, warp + 2 * kConsumerWarps, xf, lane, gc, g8c);
  acc_g += ga + gb + gc;
  acc_g8 += g8a + g8b + g8c;
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// Split-K attention of one (kv head, split) unit by consumer warps 0..3 (the
// arithmetic of k_attention_decode), then the combine of this unit's slice of
// the 768 outputs of its kv head from every split's partial.
__device__ __forceinline__ void attention_unit(const FusedParams& p, int layer, int kvh, int s, uint32_t S_eff,
                               uint32_t chunk, uint32_t L, uint16_t tag, uint8_t* uni, __half* qs,
                               volatile Misc* misc, int ct, unsigned long long* at) {
  auto astamp = [&](int k) {
    if (at && layer == p.n_layers / 2 && ct == 0) at[k] = globaltimer();
  };
  astamp(0);
  const int warp = ct >> 5, lane = ct & 31, g = lane >> 2, t = lane & 3;
  const uint32_t p0 = s * chunk, p1 = min(L, p0 + chunk);
  const uint32_t last = L - 1;
  const bool has_new = last >= p0 && last < p1;
  __half* knew = reinterpret_cast<__half*>(uni + kAKnew);
  __half* vnew = reinterpret_cast<__half*>(uni + kAVnew);
  const __half* kbase = p.kc + (size_t)layer * p.kv_layer_stride + kvh * kHeadDim;
  const __half* vbase = p.vc + (size_t)layer * p.kv_layer_stride + kvh * kHeadDim;
  uint8_t* vs = uni + kAVs + warp * (16 * 272);
  uint16_t* pth = reinterpret_cast<uint16_t*>(uni + kAPt) + warp * 256;
  uint16_t* ptl = pth + 128;
  // Stages the V rows [base, base+16) into shared memory (cp.async, zero past
  // p1) and loads the K rows of the lane's positions g, g+8 into registers.
  // Before the step's new row has arrived, position `last` is fetched from the
  // (stale) cache and patched afterwards.
  uint32_t kg[16], kg8[16];
  auto issue_kv = [&](uint32_t base, bool have_new) {
    const int r = lane >> 1, hs = lane & 1;
    const uint32_t pos = base + r;
    uint8_t* dst = vs + r * 272 + hs * 128;
    if (pos < p1 && have_new && pos == last) {
      // The step's new row is already in shared memory (vnew): a plain copy
      // (cp.async.*.shared.global only takes a global source).
      const uint4* src = reinterpret_cast<const uint4*>(vnew) + hs * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) reinterpret_cast<uint4*>(dst)[j] = src[j];
    } else if (pos < p1) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(vbase + (size_t)pos * kKVDim) + hs * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + 16 * j)),
                     "l"(src + 16 * j)
                     : "memory");
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) reinterpret_cast<uint4*>(dst)[j] = make_uint4(0, 0, 0, 0);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    const uint32_t pg = min(base + g, p1 - 1), pg8 = min(base + g + 8, p1 - 1);
    const uint4* sg = (have_new && pg == last)
                          ? reinterpret_cast<const uint4*>(knew + 32 * t)
                          : reinterpret_cast<const uint4*>(kbase + (size_t)pg * kKVDim + 32 * t);
    const uint4* sg8 = (have_new && pg8 == last)
                           ? reinterpret_cast<const uint4*>(knew + 32 * t)
                           : reinterpret_cast<const uint4*>(kbase + (size_t)pg8 * kKVDim + 32 * t);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 a = sg[j], b = sg8[j];
      kg[4 * j] = a.x; kg[4 * j + 1] = a.y; kg[4 * j + 2] = a.z; kg[4 * j + 3] = a.w;
      kg8[4 * j] = b.x; kg8[4 * j + 1] = b.y; kg8[4 * j + 2] = b.z; kg8[4 * j + 3] = b.w;
    }
  };
  const uint32_t first = p0 + warp * 16;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  uint32_t qf[16];
  // One copy of the sub-tile issue (the instruction cache): the first
  // sub-tile is issued before the waits for q and the new k / v rows, which
  // the first pass takes; a warp without positions only takes part in those.
  for (uint32_t base = first;; base += kAttnWarpsFused * 16) {
    if (base < p1) issue_kv(base, base != first);
    if (base == first) {
      // q of the 6 heads of this kv group, and the step's new k / v rows.
      poll_units<1>(p.q_ll + kvh * 768, 96, ct, 128, tag, misc, p.err, kSiteQ * 100 + layer,
                    [&](int u, const __half* v) {
                      reinterpret_cast<uint4*>(qs)[u] = *reinterpret_cast<const uint4*>(v);
                    });
      if (has_new) {
        poll_units<1>(p.kv_ll, 64, ct, 128, tag, misc, p.err, kSiteKV * 100 + layer,
                      [&](int u, const __half* v) {
                        const int w0 = 8 * u;  // words 0..255 = k, 256..511 = v
                        if (((w0 & 255) >> 7) != kvh) return;
                        __half* dst = (w0 < 256 ? knew : vnew) + (w0 & 127);
                        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(v);
                      });
      }
      abar();
      astamp(1);
      const uint4* qp = reinterpret_cast<const uint4*>(qs + (g < 6 ? g : 0) * kHeadDim + 32 * t);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 v = g < 6 ? qp[j] : make_uint4(0, 0, 0, 0);
        qf[4 * j] = v.x;
        qf[4 * j + 1] = v.y;
        qf[4 * j + 2] = v.z;
        qf[4 * j + 3] = v.w;
      }
    }
    if (base >= p1) break;
    if (base == first && last >= base && last < base + 16) {
      // patch the step's new row into the prefetched sub-tile
      const uint32_t pg = min(base + g, p1 - 1), pg8 = min(base + g + 8, p1 - 1);
      if (pg == last || pg8 == last) {
        const uint4* nk = reinterpret_cast<const uint4*>(knew + 32 * t);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 a = nk[j];
          if (pg == last) { kg[4 * j] = a.x; kg[4 * j + 1] = a.y; kg[4 * j + 2] = a.z; kg[4 * j + 3] = a.w; }
          if (pg8 == last) { kg8[4 * j] = a.x; kg8[4 * j + 1] = a.y; kg8[4 * j + 2] = a.z; kg8[4 * j + 3] = a.w; }
        }
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (base == first && last >= base && last < base + 16 && (int)(last - base) == (lane >> 1)) {
      const int hs = lane & 1;
      uint4* dst = reinterpret_cast<uint4*>(vs + (last - base) * 272 + hs * 128);
      const uint4* src = reinterpret_cast<const uint4*>(vnew) + hs * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) dst[j] = src[j];
    }
    __syncwarp();
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    {
#pragma unroll
      for (int st = 0; st < 8; ++st) {
        const uint32_t a[4] = {kg[2 * st], kg8[2 * st], kg[2 * st + 1], kg8[2 * st + 1]};
        mma_16816(sc, a, qf[2 * st], qf[2 * st + 1], sc);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[j] *= kAttnScale;
      if (base + g >= p1) sc[0] = sc[1] = -INFINITY;
      if (base + g + 8 >= p1) sc[2] = sc[3] = -INFINITY;
    }
    float pr[4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float mx = fmaxf(sc[hh], sc[2 + hh]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float m_new = fmaxf(m_run[hh], mx);
      const float corr = m_run[hh] == -INFINITY ? 0.f : expf(m_run[hh] - m_new);
      const float e0 = expf(sc[hh] - m_new), e1 = expf(sc[2 + hh] - m_new);
      pr[hh] = e0;
      pr[2 + hh] = e1;
      float sum = e0 + e1;
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      sum += __shfl_xor_sync(0xffffffffu, sum, 8);
      sum += __shfl_xor_sync(0xffffffffu, sum, 16);
      l_run[hh] = l_run[hh] * corr + sum;
      m_run[hh] = m_new;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i][hh] *= corr;
        o[i][2 + hh] *= corr;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int pos = g + (j >= 2 ? 8 : 0), head = 2 * t + (j & 1);
      const __half h = f2h(pr[j]);
      pth[pos * 8 + head] = hbits(h);
      ptl[pos * 8 + head] = hbits(f2h(pr[j] - h2f(h)));
    }
    __syncwarp();
    const uint32_t bh0 = (uint32_t)pth[(2 * t) * 8 + g] | ((uint32_t)pth[(2 * t + 1) * 8 + g] << 16);
    const uint32_t bh1 = (uint32_t)pth[(2 * t + 8) * 8 + g] | ((uint32_t)pth[(2 * t + 9) * 8 + g] << 16);
    const uint32_t bl0 = (uint32_t)ptl[(2 * t) * 8 + g] | ((uint32_t)ptl[(2 * t + 1) * 8 + g] << 16);
    const uint32_t bl1 = (uint32_t)ptl[(2 * t + 8) * 8 + g] | ((uint32_t)ptl[(2 * t + 9) * 8 + g] << 16);
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int prow = ri + ((mi >> 1) << 3), dcol = (mi & 1) << 3;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t a[4];
        ldmatrix_x4_trans(a, vs + prow * 272 + (16 * i + dcol) * 2);
        mma_16816(o[i], a, bh0, bh1, o[i]);
        mma_16816(o[i], a, bl0, bl1, o[i]);
      }
    }
    __syncwarp();
  }
  astamp(2);
  // ---- merge the 4 warps (shared memory), write this split's partial.
  float* wm = reinterpret_cast<float*>(uni + kAWm);
  float* wl = reinterpret_cast<float*>(uni + kAWl);
  if (g == 0) {
    wm[warp * 8 + 2 * t] = m_run[0];
    wm[warp * 8 + 2 * t + 1] = m_run[1];
    wl[warp * 8 + 2 * t] = l_run[0];
    wl[warp * 8 + 2 * t + 1] = l_run[1];
  }
  abar();  // every warp is done with its V rows: reuse them for the merge
  float* wo = reinterpret_cast<float*>(uni + kAVs);  // [4][6][128]
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int head = 2 * t + (j & 1), d = 16 * i + g + (j >= 2 ? 8 : 0);
      if (head < 6) wo[(warp * 6 + head) * kHeadDim + d] = o[i][j];
    }
  abar();
  astamp(3);
  // Rescale factors of the 4 warps per head, computed once (they depend on the
  // head only); factor 0 for a warp without positions.
  float* fac = reinterpret_cast<float*>(uni + kAFac);  // [4][6] factors, [6] max, [6] sum
  if (ct < 6) {
    const int head = ct;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarpsFused; ++w) M = fmaxf(M, wm[w * 8 + head]);
    float Ls = 0.f;
    for (int w = 0; w < kAttnWarpsFused; ++w) {
      const float mw = wm[w * 8 + head];
      const float c = mw == -INFINITY ? 0.f : expf(mw - M);
      fac[w * 6 + head] = c;
      Ls += wl[w * 8 + head] * c;
    }
    fac[24 + head] = M;
    fac[30 + head] = Ls;
  }
  abar();
  unsigned long long* part = p.attn_part + ((size_t)kvh * kMaxAttnSplits + s) * kAttnPartWords;
  for (int idx = ct; idx < 6 * kHeadDim; idx += 128) {
    const int head = idx / kHeadDim, d = idx % kHeadDim;
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarpsFused; ++w) O += wo[(w * 6 + head) * kHeadDim + d] * fac[w * 6 + head];
    st_tag32(part + idx, tag, O);
    if (d == 0) {
      st_tag32(part + 768 + head, tag, fac[24 + head]);
      st_tag32(part + 774 + head, tag, fac[30 + head]);
    }
  }
  abar();
  astamp(4);
  // ---- combine: this unit produces outputs [z0, z1) of its kv head.
  const uint32_t Z = (768 + S_eff - 1) / S_eff;
  const uint32_t z0 = min(768u, s * Z), z1 = min(768u, z0 + Z);
  if (z0 >= z1) return;
  const int h0 = z0 / kHeadDim, h1 = (z1 - 1) / kHeadDim;
  const uint32_t nh = h1 - h0 + 1;
  const uint32_t nz = z1 - z0;
  const uint32_t per_split = nz + 2 * nh;  // o slice, m[nh], l[nh]
  float* stage = reinterpret_cast<float*>(uni + kAVs);
  const uint32_t n_words = S_eff * per_split;
  // word w of the slice: split w / per_split, entry w % per_split; the
  // thread's words w0 + 128 j, their addresses computed once (128 = dq
  // splits + dr entries).
  const uint32_t dq = 128 / per_split, dr = 128 % per_split;
  const unsigned long long* kv_part = p.attn_part + (size_t)kvh * kMaxAttnSplits * kAttnPartWords;
  for (uint32_t w0 = ct; w0 < n_words; w0 += 128 * 8) {
    unsigned long long v[8];
    const unsigned long long* src[8];
    uint32_t pending = 0;
    {
      uint32_t sp = w0 / per_split, r = w0 % per_split;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t word = r < nz ? z0 + r : r < nz + nh ? 768 + h0 + (r - nz) : 774 + h0 + (r - nz - nh);
        src[j] = kv_part + (size_t)sp * kAttnPartWords + word;
        if (w0 + j * 128 < n_words) pending |= 1u << j;
        sp += dq;
        r += dr;
        if (r >= per_split) {
          r -= per_split;
          ++sp;
        }
      }
    }
    uint64_t t0 = 0;
    for (uint32_t it = 0; pending; ++it) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (pending & (1u << j)) v[j] = ld_tag64(src[j]);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if ((pending & (1u << j)) && (uint32_t)(v[j] >> 32) == tag) {
          stage[w0 + j * 128] = __uint_as_float((uint32_t)v[j]);
          pending &= ~(1u << j);
        }
      if (!pending) break;
      if (wait_check(it, t0, misc, p.err, kSiteCombine * 100 + layer)) break;
    }
  }
  abar();
  astamp(5);
  // Per (split, head of the slice) rescale factors and per-head totals, once.
  float* cfac = reinterpret_cast<float*>(uni + kACFac);  // [S_eff][nh] factors, then [nh] totals
  float* ctot = cfac + kMaxAttnSplits * 2;
  // A warp per head of the slice, a lane per split (fixed-order reductions).
  for (uint32_t hl = ct >> 5; hl < nh; hl += kAttnWarpsFused) {
    const uint32_t ln = ct & 31;
    float M = -INFINITY;
#pragma unroll 1
    for (uint32_t sp = ln; sp < S_eff; sp += 32) M = fmaxf(M, stage[sp * per_split + nz + hl]);
    M = warp_max(M);
    float Ls = 0.f;
#pragma unroll 1
    for (uint32_t sp = ln; sp < S_eff; sp += 32) {
      const float c = expf(stage[sp * per_split + nz + hl] - M);
      cfac[sp * nh + hl] = c;
      Ls += stage[sp * per_split + nz + nh + hl] * c;
    }
    Ls = warp_sum(Ls);
    if (ln == 0) ctot[hl] = Ls;
  }
  abar();
  for (uint32_t z = z0 + ct; z < z1; z += 128) {
    const uint32_t hl = z / kHeadDim - h0;
    float O = 0.f;
#pragma unroll 2
    for (uint32_t sp = 0; sp < S_eff; ++sp) O += stage[sp * per_split + (z - z0)] * cfac[sp * nh + hl];
    st_tag16(p.attn_ll + kvh * 768 + z, tag, f2h(O / ctot[hl]));
  }
  astamp(6);
}

// Issues item i into its ring slot: the slot's previous readers are done
// (their releases completed it), so after a proxy fence the bulk copy may
// overwrite it; slot_item tells waiters the slot now holds item i.
__device__ __noinline__ void issue_item(int i, const FusedItem* items, const FusedParams& p,
                                        int lm_phase, uint8_t* ring, uint64_t* full,
                                        volatile int* slot_item, volatile Misc* misc) {
  const int slot = i % kNS;
  const ItemFields it = unpack_item(items[i]);
  size_t off;
  uint32_t bytes;
  item_source(it, lm_phase, &off, &bytes);
  const uint8_t* src = (it.phase == lm_phase ? p.lm : p.q4) + off;
  fence_proxy_async();
  mbar_arrive_expect_tx(&full[slot], bytes);
  bulk_g2s_stream(ring + slot * kSlotBytes, src, bytes, &full[slot], policy_evict_first());
  __threadfence_block();
  slot_item[slot] = i;
  misc->issued[slot] = misc->issued[slot] + 1;
}

}  // namespace

// 256 threads = 8 warps, 2 per SM sub-partition: up to 255 registers a thread.
// kTrace: the phase trace's stamps are compiled in (a launch with
// FusedParams::trace set); without it the step carries none of their code.
template <bool kTrace>
__global__ void __launch_bounds__(kFusedThreads, 1) k_decode_fused(FusedParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* uni = smem + kOffUnion;
  __half* xloc = reinterpret_cast<__half*>(smem + kOffXloc);
  __half* xn = reinterpret_cast<__half*>(smem + kOffXn);
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* red2 = reinterpret_cast<float*>(smem + kOffRed2);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBars);
  // per slot: releases of the item in it so far, and the item issued into it
  uint32_t* rel_cnt = reinterpret_cast<uint32_t*>(full + kNS);
  volatile int* slot_item = reinterpret_cast<volatile int*>(rel_cnt + kNS);
  volatile Misc* misc = reinterpret_cast<volatile Misc*>(smem + kOffMisc);
  uint4* xf = reinterpret_cast<uint4*>(uni);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ib = p.item_begin[blockIdx.x];
  const int n_items = (int)(p.item_begin[blockIdx.x + 1] - ib);
  FusedItem* items = reinterpret_cast<FusedItem*>(smem + kOffItems);
  const uint16_t lm_phase = (uint16_t)(p.n_layers * kPhasesPerLayer);
  for (int i = threadIdx.x; i < n_items && i < kMaxItemsPerCta; i += blockDim.x) items[i] = p.items[ib + i];

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNS; ++i) {
      mbar_init(&full[i], 1);
      rel_cnt[i] = 0;
      slot_item[i] = -1;
      misc->issued[i] = 0;
    }
    misc->wait_ns = p.wait_ns;
    misc->abort = 0;
    misc->cphase = -1;
    for (int w = 0; w < 8; ++w) misc->last_rel[w] = -1;
    fence_mbar_init();
  }
  __syncthreads();

  unsigned long long* trace_out =
      kTrace && p.trace ? p.trace + (size_t)blockIdx.x * p.trace_stride : nullptr;
  unsigned long long* trace =
      trace_out ? reinterpret_cast<unsigned long long*>(smem + kOffTrace) : nullptr;
  if (trace)
    for (int i = threadIdx.x; i < p.trace_stride; i += blockDim.x) trace[i] = 0;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (trace) trace[0] = globaltimer();
    for (int i = 0; i < kNS && i < n_items; ++i) issue_item(i, items, p, lm_phase, ring, full, slot_item, misc);
  }
  {
    // ------------------------------------------------------------ consumers
    const int ct = threadIdx.x;
    const uint32_t L = p.seq_ctl[3];       // SeqCtl.seq_len
    const int token = (int)p.seq_ctl[4];   // SeqCtl.token
    const uint32_t epoch = *p.epoch;
    auto tagof = [&](uint32_t k) { return (uint32_t)((epoch << 8) + k) & 0xFFFFu; };
    const int g = lane >> 2, t = lane & 3;
    int cur = 0;
    // Lane 0 of a warp: this warp's share n of item i's kConsumerWarps
    // releases; the release that completes them refills the slot with item
    // i + kNS (none once the kernel is aborting).
    auto release = [&](int i, uint32_t n) {
      const int slot = i % kNS;
      __threadfence_block();   // this warp's reads of the slot before its release
      if (atomicAdd(&rel_cnt[slot], n) + n == (uint32_t)kConsumerWarps) {
        __threadfence_block();   // every warp's release before the refill
        rel_cnt[slot] = 0;
        // (the shared abort flag only: a global read here would sit on the
        // issuing warp's path at every refill)
        if (i + kNS < n_items && !misc->abort)
          issue_item(i + kNS, items, p, lm_phase, ring, full, slot_item, misc);
      }
      misc->last_rel[warp] = i;
    };
    auto phase_end = [&](uint16_t ph) {
      int e = cur;
      while (e < n_items && (int)(items[e] & 0xFF) == ph) ++e;
      return e;
    };
    // K-split processing of items [cur, e), each a whole 16-row tile: warp w
    // takes block pairs w, w+8, w+16; the tile's 16 sums meet in shared memory.
    // The warps release the item after the epilogue, off the path to it (the
    // release that completes the slot issues the next copy).
    auto timed_wait = [&](int i, int site) {
      return item_wait(i, full, slot_item, misc, p.err, site);
    };
    auto ksplit = [&](int e, auto&& epilogue) {
      for (int i = cur; i < e; ++i) {
        const ItemFields it = unpack_item(items[i]);
        float acc_g = 0.f, acc_g8 = 0.f;
        if (timed_wait(i, kSiteFull * 100 + it.phase % 100))
          q4_kslice3(ring + (i % kNS) * kSlotBytes, warp, xf, lane, acc_g, acc_g8);
        if (t == 0) {
          red[warp * 16 + g] = acc_g;
          red[warp * 16 + g + 8] = acc_g8;
        }
        cbar();
        if (ct < 16) {
          float sum = 0.f;
          for (int w = 0; w < kConsumerWarps; ++w) sum += red[w * 16 + ct];
          epilogue(it.tile, ct, sum);
        }
        cbar();
        if (lane == 0) release(i, 1);
      }
      cur = e;
    };
    const float* rope = p.rope_cs + (size_t)(L - 1) * 128;
    auto stamp = [&](int k) {
      if (trace && ct == 0) trace[k] = globaltimer();
    };
    auto lstamp = [&](int layer, int k) { stamp(3 + layer * kTraceStampsPerLayer + k); };
    stamp(2);

    for (int layer = 0; layer < p.n_layers; ++layer) {
      const uint16_t ph = (uint16_t)(layer * kPhasesPerLayer);
      if (ct == 0) misc->cphase = ph * 1000 + cur;
      lstamp(layer, kTsLayerStart);
      // Activation-independent inputs of this layer's QKV phase, fetched before
      // the wait for x: the input RMSNorm gamma, and for the first QKV tile the
      // rows' biases and the RoPE cos/sin of threads 0..15.
      const uint4 gamma_in = gamma_prefetch(p.norms + (size_t)(2 * layer) * kHidden, ct);
      const int e_qkv = phase_end(ph + kPhQKV);
      const int qtile = e_qkv > cur ? (int)unpack_item(items[cur]).tile : -1;
      float qbias = 0.f, qcos = 1.f, qsin = 0.f;
      if (qtile >= 0 && ct < 16) {
        const int head = qtile >> 3, j = qtile & 7, r = ct;
        const int row = head * 128 + (r < 8 ? 8 * j + r : 64 + 8 * j + (r - 8));
        qbias = h2f(p.qkv_bias[(size_t)layer * kQKVRows + row]);
        if (r < 8 && head < 14) {
          qcos = rope[2 * (8 * j + r)];
          qsin = rope[2 * (8 * j + r) + 1];
        }
      }
      // ---- x after the previous layer (or the embedding row, :57-60)
      if (layer == 0) {
        const uint4* src = reinterpret_cast<const uint4*>(p.embed + (size_t)token * kHidden);
        for (int u = ct; u < kHidden / 8; u += 256) reinterpret_cast<uint4*>(xloc)[u] = src[u];
      } else {
        poll_units<1>(p.x_ll, kHidden / 8, ct, 256, tagof(2 * layer), misc, p.err,
                      kSiteXIn * 100 + layer, [&](int u, const __half* v) {
                        reinterpret_cast<uint4*>(xloc)[u] = *reinterpret_cast<const uint4*>(v);
                      });
      }
      cbar();
      lstamp(layer, kTsXReady);
      // ---- P1: RMSNorm -> QKV -> bias -> RoPE -> q, KV cache
      {
        const int e = e_qkv;
        if (e > cur) {
          rmsnorm_out(xloc, gamma_in, red2, xf, nullptr, ct);
          const uint16_t tg = (uint16_t)tagof(layer);
          __half* kc = p.kc + (size_t)layer * p.kv_layer_stride + (size_t)(L - 1) * kKVDim;
          __half* vc = p.vc + (size_t)layer * p.kv_layer_stride + (size_t)(L - 1) * kKVDim;
          const __half* bias = p.qkv_bias + (size_t)layer * kQKVRows;
          // threads 0..15 hold the tile's 16 rows; rows r and r+8 form a RoPE pair
          ksplit(e, [&](int tile, int r, float sum) {
            const int head = tile >> 3, j = tile & 7;
            const int row = head * 128 + (r < 8 ? 8 * j + r : 64 + 8 * j + (r - 8));
            const bool pre = tile == qtile;  // prefetched bias / cos / sin
            red2[r] = h2f(f2h(sum + (pre ? qbias : h2f(bias[row]))));
            __syncwarp(0xffffu);
            if (r >= 8) return;
            const float x1 = red2[r], x2 = red2[r + 8];
            const int i = 8 * j + r;  // rotate-half pair index (rope.metal:17-22)
            __half o1, o2;
            if (head < 14) {
              const float c = pre ? qcos : rope[2 * i], sn = pre ? qsin : rope[2 * i + 1];
              o1 = f2h(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn)));
              o2 = f2h(__fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, c)));
            } else {
              o1 = f2h(x1);
              o2 = f2h(x2);
            }
            const int d1 = 8 * j + r, d2 = 64 + 8 * j + r;
            if (head < 12) {
              st_tag16(p.q_ll + head * 128 + d1, tg, o1);
              st_tag16(p.q_ll + head * 128 + d2, tg, o2);
            } else if (head < 14) {
              const int kh = head - 12;
              kc[kh * 128 + d1] = o1;
              kc[kh * 128 + d2] = o2;
              st_tag16(p.kv_ll + kh * 128 + d1, tg, o1);
              st_tag16(p.kv_ll + kh * 128 + d2, tg, o2);
            } else {
              const int vh = head - 14;
              vc[vh * 128 + d1] = o1;
              vc[vh * 128 + d2] = o2;
              st_tag16(p.kv_ll + 256 + vh * 128 + d1, tg, o1);
              st_tag16(p.kv_ll + 256 + vh * 128 + d2, tg, o2);
            }
          });
        }
      }
      lstamp(layer, kTsQKVDone);
      // ---- P2: attention units on the last CTAs
      {
        uint32_t S = (L + 63) / 64;
        const uint32_t cap = min((uint32_t)kMaxAttnSplits, gridDim.x / 2);
        S = max(1u, min(S, cap));
        uint32_t chunk = (L + S - 1) / S;
        chunk = (chunk + 15) / 16 * 16;
        const uint32_t S_eff = (L + chunk - 1) / chunk;
        const int u = (int)gridDim.x - 1 - (int)blockIdx.x;
        if (u < (int)(2 * S_eff) && warp < kAttnWarpsFused)
          attention_unit(p, layer, u & 1, u >> 1, S_eff, chunk, L, (uint16_t)tagof(layer), uni,
                         xn, misc, ct,
                         trace ? trace + 3 + p.n_layers * kTraceStampsPerLayer + 2 : nullptr);
      }
      cbar();
      lstamp(layer, kTsAttnDone);
      // ---- P3: O projection + bias + residual (attention.metal:58-65)
      {
        const int e = phase_end(ph + kPhO);
        if (e > cur) {
          const __half* ob = p.o_bias + (size_t)layer * kHidden;
          const int otile = (int)unpack_item(items[cur]).tile;
          const float obias = ct < 16 ? h2f(ob[16 * otile + ct]) : 0.f;
          poll_units<1>(p.attn_ll, kHidden / 8, ct, 256, tagof(layer), misc, p.err,
                        kSiteAttnOut * 100 + layer, [&](int u, const __half* v) {
                          __half tmp[8];
#pragma unroll
                          for (int q = 0; q < 8; ++q) tmp[q] = v[q];
                          xf[u] = make_xfrag(tmp);
                        });
          cbar();
          lstamp(layer, kTsOReady);
          const uint16_t tg = (uint16_t)tagof(2 * layer + 1);
          ksplit(e, [&](int tile, int r, float sum) {
            const int row = 16 * tile + r;
            const __half o = f2h(sum + (tile == otile ? obias : h2f(ob[row])));
            st_tag16(p.x_ll + row, tg, __hadd(xloc[row], o));
          });
        }
      }
      lstamp(layer, kTsODone);
      // ---- P4: x' -> RMSNorm -> gate|up -> SwiGLU -> h.  A CTA below
      // kMlpUnits owns MLP unit u = blockIdx.x: gate/up tiles 8u .. 8u+7, one
      // per warp (item cur + w has seq w), giving h[64u .. 64u+63].
      const uint4 gamma_post = gamma_prefetch(p.norms + (size_t)(2 * layer + 1) * kHidden, ct);
      poll_units<1>(p.x_ll, kHidden / 8, ct, 256, tagof(2 * layer + 1), misc, p.err,
                    kSiteXMid * 100 + layer, [&](int u, const __half* v) {
                      reinterpret_cast<uint4*>(xloc)[u] = *reinterpret_cast<const uint4*>(v);
                    });
      cbar();
      uint4* hf = reinterpret_cast<uint4*>(uni + kOffHFrag);
      {
        const int e = phase_end(ph + kPhGU);
        rmsnorm_out(xloc, gamma_post, red2, xf, nullptr, ct);
        lstamp(layer, kTsGUReady);
        const int i = cur + warp;
        if (i < e) {
          const ItemFields it = unpack_item(items[i]);
          const int slot = i % kNS;
          float acc_g = 0.f, acc_g8 = 0.f;
          if (timed_wait(i, kSiteFull * 100 + it.phase % 100))
            q4_chunk(ring + slot * kSlotBytes, it.k0, 0, it.nk, 1, xf, lane, acc_g, acc_g8);
          __syncwarp();
          if (lane == 0) release(i, kConsumerWarps);
          // gate and up with the zero bias of InferenceEngine.swift:82-85, then
          // half(silu(gate) * up) (activations.metal:14-26); every lane of
          // group g holds row g's sums (the MMA's 8 columns are equal).
          const __half gate = f2h(acc_g + 0.0f), up = f2h(acc_g8 + 0.0f);
          const __half h = f2h(silu_ref(h2f(gate)) * h2f(up));
          // h[8w .. 8w+7] of the unit is the down strip's x fragment for
          // block w / 4, lane quad w % 4 (make_xfrag order): hf[w].
          __half v[8];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            v[q] = __ushort_as_half((unsigned short)__shfl_sync(0xffffffffu, (unsigned)hbits(h), 4 * q));
          if (lane == 0) hf[warp] = make_xfrag(v);
        }
        cur = e;
      }
      cbar();
      lstamp(layer, kTsGUDone);
      // ---- P5: the unit's down strip: row tiles x block pair u, K-split
      // partial sums of all 1536 outputs over this unit's 64 k.  Warps 2j and
      // 2j+1 take item j (24 row tiles), 12 row tiles each, in two rounds of
      // six (a loop, not straight code: the instruction cache): one slot wait
      // and one release a warp.
      {
        const int e = phase_end(ph + kPhDown);
        if (e - cur == kDownItems) {
          const int i = cur + (warp >> 1);
          const int b0 = kDownRowTilesPerWarp * (warp & 1);
          const bool landed = timed_wait(i, kSiteFull * 100 + (int)(items[i] & 0xFF) % 100);
          const uint8_t* sb = ring + (i % kNS) * kSlotBytes + b0 * kBpBytes;
          // The warp's 12 row tiles are 192 consecutive rows of the unit's
          // partial vector, and every lane of group g holds rows g and g + 8 of
          // each tile: lane (g, t) stores row 8t + g of a pair of tiles, one
          // 256-byte store per pair.
          const uint16_t tg = (uint16_t)tagof(layer);
          const ItemFields it = unpack_item(items[i]);
          unsigned long long* part = p.mlp_part + (size_t)it.tile * kHidden + 16 * (it.k0 + b0) + 8 * t + g;
#pragma unroll 1
          for (int r = 0; r < kDownRowTilesPerWarp; r += kDownRound) {
            float acc[kDownRound][2];
#pragma unroll
            for (int j = 0; j < kDownRound; ++j) acc[j][0] = acc[j][1] = 0.f;
            if (landed) {
#pragma unroll
              for (int j = 0; j < kDownRound; j += 3) {
                q4_bp(sb + (r + j + 0) * kBpBytes, 0, 0, hf, lane, acc[j][0], acc[j][1]);
                q4_bp(sb + (r + j + 1) * kBpBytes, 0, 0, hf, lane, acc[j + 1][0], acc[j + 1][1]);
                q4_bp(sb + (r + j + 2) * kBpBytes, 0, 0, hf, lane, acc[j + 2][0], acc[j + 2][1]);
              }
            }
#pragma unroll
            for (int m = 0; m < kDownRound / 2; ++m)
              st_tag32(part + 16 * r + 32 * m, tg, t == 0 ? acc[2 * m][0] : t == 1 ? acc[2 * m][1]
                                                 : t == 2 ? acc[2 * m + 1][0] : acc[2 * m + 1][1]);
          }
          __syncwarp();
          if (lane == 0) release(i, kConsumerWarps / kWarpsPerDownItem);
        }
        cur = e;
      }
      // All warps done before any polls: a warp spinning on global loads
      // while others still stream their down items would queue its loads
      // ahead of their shared-memory traffic.
      cbar();
      lstamp(layer, kTsPartialsOut);
      // ---- P6: every CTA finishes rows [R0, R1) of the layer's output: the
      // 140 units' partial sums in unit order, + bias, rounded (matmul.metal:71),
      // + the residual x' (attention.metal:58-65).
      {
        const int R0 = (int)(blockIdx.x * kHidden / gridDim.x);
        const int R1 = (int)((blockIdx.x + 1) * kHidden / gridDim.x);
        const int n_rows = R1 - R0;
        float* stage = reinterpret_cast<float*>(uni + kOffMlpStage);
        // word w: unit w / kMaxReduceRows, row R0 + w % kMaxReduceRows (a
        // constant divisor; rows past n_rows are not polled).  A warp's words
        // are runs of consecutive rows of a unit: few L2 sectors a poll.
        auto word_src = [&](int w) {
          return p.mlp_part + (size_t)(w / kMaxReduceRows) * kHidden + R0 + w % kMaxReduceRows;
        };
        auto word_dst = [&](int w) { return (w % kMaxReduceRows) * kMlpUnits + w / kMaxReduceRows; };
        // (test hook: with stall_site == kSiteDownPart the poll expects a tag
        // nothing writes, so the wait runs out)
        const uint32_t ptag = p.stall_site == kSiteDownPart ? tagof(255) : tagof(layer);
        uint32_t pending = 0;
        unsigned long long v[kReducePerThread];
#pragma unroll
        for (int j = 0; j < kReducePerThread; ++j) {
          const int w = ct + j * kFusedThreads;
          if (w < kMaxReduceRows * kMlpUnits && w % kMaxReduceRows < n_rows) pending |= 1u << j;
        }
        uint64_t t0 = 0;
        for (uint32_t it = 0; pending; ++it) {
#pragma unroll
          for (int j = 0; j < kReducePerThread; ++j)
            if (pending & (1u << j)) v[j] = ld_tag64(word_src(ct + j * kFusedThreads));
#pragma unroll
          for (int j = 0; j < kReducePerThread; ++j)
            if ((pending & (1u << j)) && (uint32_t)(v[j] >> 32) == ptag) {
              stage[word_dst(ct + j * kFusedThreads)] = __uint_as_float((uint32_t)v[j]);
              pending &= ~(1u << j);
            }
          if (!pending) break;
          if (wait_check(it, t0, misc, p.err, kSiteDownPart * 100 + layer)) break;
        }
        cbar();
        const __half* db = p.down_bias + (size_t)layer * kHidden;
        const uint16_t tg = (uint16_t)tagof(2 * layer + 2);
        for (int r = warp; r < n_rows; r += kConsumerWarps) {
          float sum = 0.f;
          for (int u = lane; u < kMlpUnits; u += 32) sum += stage[r * kMlpUnits + u];
          sum = warp_sum(sum);
          if (lane == 0) {
            const int row = R0 + r;
            const __half d = f2h(sum + h2f(db[row]));
            st_tag16(p.x_ll + row, tg, __hadd(xloc[row], d));
          }
        }
      }
      cbar();
      lstamp(layer, kTsReduced);
    }
    // ---- final RMSNorm + LM head (each warp owns whole 16-row tiles)
    if (ct == 0) misc->cphase = lm_phase * 1000 + cur;
    stamp(3 + p.n_layers * kTraceStampsPerLayer);
    const uint4 gamma_final = gamma_prefetch(p.norms + (size_t)(2 * p.n_layers) * kHidden, ct);
    poll_units<1>(p.x_ll, kHidden / 8, ct, 256, tagof(2 * p.n_layers), misc, p.err,
                  kSiteXFinal * 100, [&](int u, const __half* v) {
                    reinterpret_cast<uint4*>(xloc)[u] = *reinterpret_cast<const uint4*>(v);
                  });
    cbar();
    rmsnorm_out(xloc, gamma_final, red2, nullptr, xn, ct);
    {
      const int e = phase_end(lm_phase);
      float d[4] = {0.f, 0.f, 0.f, 0.f}, d2[4] = {0.f, 0.f, 0.f, 0.f};
      for (int i = cur; i < e; ++i) {
        const ItemFields it = unpack_item(items[i]);
        if ((it.seq & (kConsumerWarps - 1)) != warp) continue;
        const int slot = i % kNS;
        if (item_wait(i, full, slot_item, misc, p.err, kSiteFull * 100 + it.phase % 100)) {
          const uint8_t* sb = ring + slot * kSlotBytes;
          int s = 0;
          for (; s + 1 < it.nk; s += 2) {
            const uint4 w = *reinterpret_cast<const uint4*>(sb + s * kLMStepBytes + lane * 16);
            const uint4 w2 = *reinterpret_cast<const uint4*>(sb + (s + 1) * kLMStepBytes + lane * 16);
            const uint2 b = *reinterpret_cast<const uint2*>(xn + 16 * (it.k0 + s) + 4 * t);
            const uint2 b2 = *reinterpret_cast<const uint2*>(xn + 16 * (it.k0 + s + 1) + 4 * t);
            const uint32_t a[4] = {w.x, w.z, w.y, w.w};
            const uint32_t a2[4] = {w2.x, w2.z, w2.y, w2.w};
            mma_16816(d, a, b.x, b.y, d);
            mma_16816(d2, a2, b2.x, b2.y, d2);
          }
          if (s < it.nk) {
            const uint4 w = *reinterpret_cast<const uint4*>(sb + s * kLMStepBytes + lane * 16);
            const uint2 b = *reinterpret_cast<const uint2*>(xn + 16 * (it.k0 + s) + 4 * t);
            const uint32_t a[4] = {w.x, w.z, w.y, w.w};
            mma_16816(d, a, b.x, b.y, d);
          }
        }
        __syncwarp();
        if (lane == 0) release(i, kConsumerWarps);
        if (it.last) {
          if (t == 0) {
            p.logits[16 * it.tile + g] = f2h(d[0] + d2[0]);
            p.logits[16 * it.tile + g + 8] = f2h(d[2] + d2[2]);
          }
          d[0] = d[1] = d[2] = d[3] = 0.f;
          d2[0] = d2[1] = d2[2] = d2[3] = 0.f;
        }
      }
      cur = e;
    }
    stamp(3 + p.n_layers * kTraceStampsPerLayer + 1);
  }
  __syncthreads();
  // Drain: every copy this CTA issued has landed before its shared memory goes
  // away.  A slot's n-th copy completes its barrier's phase n - 1, so the
  // wait is on the parity of the count of copies issued into it.
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer();
    for (int sl = 0; sl < kNS; ++sl) {
      const int n = misc->issued[sl];
      if (n == 0) continue;
      while (!mbar_try_wait(&full[sl], (uint32_t)(n - 1) & 1u))
        if (globaltimer() - t0 > kDrainNs) break;
    }
    if (trace) trace[1] = globaltimer();
  }
  if (trace) {
    __syncthreads();
    for (int i = threadIdx.x; i < p.trace_stride; i += blockDim.x) trace_out[i] = trace[i];
  }
}

// ------------------------------------------------------------------ host --
namespace {
struct FusedScratchLayout {
  size_t x_ll, q_ll, kv_ll, attn_part, attn_ll, mlp_part, total;
};
FusedScratchLayout fused_layout() {
  FusedScratchLayout l{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += (bytes + 255) / 256 * 256;
    return at;
  };
  l.x_ll = take(kHidden * 4);
  l.q_ll = take(kHidden * 4);
  l.kv_ll = take(512 * 4);
  l.attn_part = take((size_t)2 * kMaxAttnSplits * kAttnPartWords * 8);
  l.attn_ll = take(kHidden * 4);
  l.mlp_part = take((size_t)kHidden * kMlpUnits * 8);
  l.total = o;
  return l;
}
}  // namespace

int fused_scratch_bytes(int batch, int, int, size_t* bytes) {
  if (batch != 1)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "the fused decode step decodes one sequence");
  *bytes = fused_layout().total;
  return QWEN_OK;
}

int enqueue_fused_step(const FusedStepArgs& a, cudaStream_t st) {
  const QwenModel& m = *a.model;
  InferenceManager& s = *a.state;
  const FusedWeights& f = m.fused;
  if (!f.blob || !f.items) return set_error(QWEN_ERR_STATE, "fused weights not built");
  if (s.batch != 1)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "the fused decode step decodes one sequence");
  if (f.rope_ctx < s.max_ctx) return set_error(QWEN_ERR_STATE, "RoPE table shorter than max_ctx");
  static_assert(sizeof(SeqCtl) == 32, "SeqCtl layout read by the fused kernel");
  const FusedScratchLayout lay = fused_layout();
  uint8_t* sc = reinterpret_cast<uint8_t*>(s.fused_scratch);
  FusedParams p{};
  p.q4 = f.blob;
  p.lm = f.lm_tiles;
  p.embed = m.embed;
  p.norms = f.norms;
  p.qkv_bias = f.qkv_bias;
  p.o_bias = f.o_bias;
  p.down_bias = f.down_bias;
  p.rope_cs = f.rope_cs;
  p.items = f.items;
  p.item_begin = f.item_begin;
  p.seq_ctl = reinterpret_cast<const uint32_t*>(s.ctl);
  p.epoch = s.epoch;
  p.kc = s.kc;
  p.vc = s.vc;
  p.x_ll = reinterpret_cast<uint32_t*>(sc + lay.x_ll);
  p.q_ll = reinterpret_cast<uint32_t*>(sc + lay.q_ll);
  p.kv_ll = reinterpret_cast<uint32_t*>(sc + lay.kv_ll);
  p.attn_part = reinterpret_cast<unsigned long long*>(sc + lay.attn_part);
  p.attn_ll = reinterpret_cast<uint32_t*>(sc + lay.attn_ll);
  p.mlp_part = reinterpret_cast<unsigned long long*>(sc + lay.mlp_part);
  p.logits = s.logits;
  p.err = s.err;
  p.trace = s.trace;
  p.trace_stride = trace_stride_for(m.n_layers);
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  p.n_layers = m.n_layers;
  p.max_ctx = s.max_ctx;
  p.kv_layer_stride = (int)s.kv_layer_stride();
  p.wait_ns = a.wait_ns;
  p.stall_site = a.stall_site;
  void (*kern)(FusedParams) = p.trace ? k_decode_fused<true> : k_decode_fused<false>;
  if (int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kSmemBytes),
                           "cudaFuncSetAttribute(k_decode_fused)"))
    return rc;
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                       (int)cudaSharedmemCarveoutMaxShared);
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFusedThreads, kSmemBytes);
  if (per_sm < 1) {
    int dev = 0, smem_sm = 0, smem_optin = 0, smem_rsv = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&smem_rsv, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kern);
    return set_error(QWEN_ERR_CUDA,
                     "k_decode_fused does not fit on an SM (%d B dynamic + %zu B static shared memory, "
                     "%d threads x %d registers; SM: %d B shared, %d B per block opt-in, %d B reserved)",
                     kSmemBytes, fa.sharedSizeBytes, kFusedThreads, fa.numRegs, smem_sm, smem_optin,
                     smem_rsv);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(f.grid);
  cfg.blockDim = dim3(kFusedThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, p), "launch k_decode_fused");
}

}  // namespace qwen
