// sampler.cu -- on-device token sampler (extractNextTokenID,
// InferenceEngine.swift:273-368) as a radix select over a thread-block cluster.
//
// One cluster of C CTAs per sequence (C = 16, 8 or 4: the largest whose one
// wave of clusters holds the batch, else 4); CTA r owns ids [r*chunk, (r+1)*chunk) and keeps
// their fixed-point weights in shared memory.  The maximum and the
// final count go through distributed shared memory behind hardware cluster
// barriers; the radix passes' digit totals are pushed into every CTA's shared
// memory with st.async and awaited on a transaction-count mbarrier (a bounded
// wait that records kDevWaitTimeout in err when it gives up).
//
// Rule (the reference's steps with every order-dependent quantity exact):
//   greedy (T <= 0): first maximum over non-NaN logits; none -> 151645 (:277-294)
//   scaled = logit / T, NaN logits keep 0.0 (:297-309); max over non-NaN;
//   all NaN -> 151645 (:311-315)
//   E_i = trunc(sampler_exp(min(scaled_i - max, 0)) * 2^31)          (:317-326)
//   order (E desc, id asc) replaces the unstable sort (:337)
//   keep the shortest prefix with sum >= thr = floor(S * trunc(p*2^24) / 2^24) (:339-351)
//   R = floor(K * u24 / 2^24), K = kept sum; first kept id with running sum > R (:353-367)
// Both selections run as 4-pass weighted radix selects (8-bit digits) on E.
// The cutoff select's first pass is histogrammed while the weights are made
// (S is the sum of its totals); the draw's passes take their totals from the
// cutoff select's while the two prefixes agree, and scan only after they part.
#include <cooperative_groups.h>

#include "qwen_common.cuh"
#include "qwen_internal.h"

namespace cg = cooperative_groups;

namespace qwen {

constexpr int kSampThreads = 1024;

// exp for the sampler: Cody-Waite reduction with the two-part ln2 split of
// Cephes expf, degree-7 Taylor polynomial in Horner form with fused
// multiply-adds.  Identical operation sequence to the CPU oracle's.
__device__ __forceinline__ float sampler_exp(float x) {
  if (!(x <= 0.0f)) x = 0.0f;
  if (x < -100.0f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-n, 0.693359375f, x);
  r = __fmaf_rn(-n, -2.12194440e-4f, r);
  float p = 1.0f / 5040.0f;
  p = __fmaf_rn(p, r, 1.0f / 720.0f);
  p = __fmaf_rn(p, r, 1.0f / 120.0f);
  p = __fmaf_rn(p, r, 1.0f / 24.0f);
  p = __fmaf_rn(p, r, 1.0f / 6.0f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = (int)n;
  if (ni < -126) return 0.0f;
  return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

__device__ __forceinline__ unsigned long long mul_shift24(unsigned long long a, uint32_t b) {
  return (a >> 24) * b + (((a & 0xFFFFFFull) * b) >> 24);
}

constexpr int kSampWarps = kSampThreads / 32;

// Shared memory of one CTA of a C-CTA cluster (C = 4, 8 or 16).
template <int C>
struct SampShared {
  static constexpr int kC = C;
  static constexpr int kChunk = (kVocab + C - 1) / C;                           // 37984 / 18992 / 9496
  static constexpr int kPerThread = (kChunk + kSampThreads - 1) / kSampThreads;  // 38 / 19 / 10
  // The draw select runs beside the cutoff select: a pass then histograms
  // both member sets (disjoint once the draw's prefix has left the cutoff's),
  // the draw's in bins 256..511.
  static constexpr bool kSpec = true;
  static constexpr int kBins = kSpec ? 512 : 256;
  // One digit histogram per pair of warps; per four warps with 4 CTAs, whose
  // 38K weights take most of shared memory (the 64-sequence step: the draw
  // beside the cutoff there measured 2.081 -> 2.055 ms a step).
  static constexpr int kHist = C >= 8 ? kSampWarps / 2 : kSampWarps / 4;
  static constexpr int kWarpsPerHist = kSampWarps / kHist;
  uint32_t e[kChunk];                        // scaled floats, then fixed-point weights
  // Digit weights of the running pass as two exact halves (E & 0xFFFF, E >> 16):
  // a histogram sees at most 2 * 38 * 32 elements, so each half fits 32 bits.
  uint32_t whist[kHist][2][kBins];
  unsigned long long qsum[kSampThreads];     // partial merges of whist, [groups][bins]
  alignas(16) unsigned long long send[kBins];  // this rank's digit weights, copied to every rank
  alignas(16) unsigned long long inbox[C][kBins];  // each rank's digit weights of the last exchange
  uint64_t xbar;                             // inbox barrier (transaction bytes)
  unsigned long long tot[kBins];             // cluster totals of the running pass
  unsigned long long tot1[4][256];           // the cutoff select's totals per pass
  unsigned long long above1[4];              // its weight above the prefix after each pass
  float red_f[32];
  int red_i[32];
  unsigned long long red_u[32];
  uint32_t red_c[32];
  float cl_f[C];                             // per-CTA partials read by the cluster
  int cl_i;
  uint32_t sel;
  unsigned long long sel_above;
  // select state, written by warp 0 after each pass
  unsigned long long thr, an, ad, R;         // cutoff target, weight above the cutoff / draw prefix
  uint32_t pn, pd;                           // cutoff and draw prefixes
  int dmode, dfail, don, dhi;                // draw mode, pass it left the speculation, on e_star
                                             // then, its pass-3 weights in bins 256..511
};

static_assert(sizeof(SampShared<4>) <= 232448, "4-CTA sampler layout exceeds shared memory");

template <class SS>
__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v, SS& s) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) s.red_u[w] = v;
  __syncthreads();
  unsigned long long t = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += s.red_u[i];
  return t;
}

// Inclusive prefix sum of one value per thread over the block (thread order).
template <class SS>
__device__ __forceinline__ uint32_t block_incl_scan_u32(uint32_t v, SS& s) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) s.red_c[w] = v;
  __syncthreads();
  if (w == 0) {
    uint32_t t = s.red_c[lane], x = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t u = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += u;
    }
    s.red_c[lane] = x - t;   // exclusive offsets of the warps
  }
  __syncthreads();
  return v + s.red_c[w];
}

// Weighted radix selects over E (descending order), 4 passes of 8-bit digits.
// A pass histograms the members' weights by digit (per warp, two exact 32-bit
// halves), sums the histograms over the cluster, and picks the digit at which
// the running weight from the top first reaches the target.

// Zeroes bins [0, nb) of the digit histograms (warps share them: block barrier).
template <class SS>
__device__ __forceinline__ void hist_clear(SS& s, int nb) {
  const int lg = nb == 512 ? 9 : 8;
  uint32_t* h = &s.whist[0][0][0];
  for (int i = threadIdx.x; i < SS::kHist * 2 * nb; i += kSampThreads)
    h[(i >> lg) * SS::kBins + (i & (nb - 1))] = 0;
  __syncthreads();
}

// Adds weight e at digit d to this warp's histogram for each lane that is a
// member.  Zero weights change no sum, so callers pass them as non-members.
// The lanes of the first member's digit, and then those of digit 0, are
// summed across the warp (two 32-bit halves, exact) and added once; the other
// members add alone.  Digit 0 is where most weights of a flat distribution
// fall (every weight below 2^-7 of the largest in the first pass), and a
// warp's lanes all adding to one counter serialise: on random-init logits the
// 64-sequence weight pass took 36 us, 13 us with the sums (gating them on two
// or more lanes sharing the digit measured slower).  (Partitioning the
// warp by digit with match.any measured slower on flat distributions.)
template <class SS>
__device__ __forceinline__ void hist_add(SS& s, bool member, uint32_t e, uint32_t d) {
  const int lane = threadIdx.x & 31, wid = (threadIdx.x >> 5) / SS::kWarpsPerHist;
  uint32_t* hlo = s.whist[wid][0];
  uint32_t* hhi = s.whist[wid][1];
  const uint32_t mm = __ballot_sync(0xffffffffu, member);
  if (mm == 0u) return;
  const int first = __ffs(mm) - 1;
  const uint32_t d0 = __shfl_sync(0xffffffffu, d, first);
  {
    const bool in = member && d == d0;
    const uint32_t lo = __reduce_add_sync(0xffffffffu, in ? (e & 0xFFFFu) : 0u);
    const uint32_t hi = __reduce_add_sync(0xffffffffu, in ? (e >> 16) : 0u);
    if (lane == first) {
      atomicAdd(&hlo[d0], lo);
      atomicAdd(&hhi[d0], hi);
    }
    member = member && !in;
  }
  if (d0 != 0u) {
    const bool in = member && d == 0u;
    const uint32_t zm = __ballot_sync(0xffffffffu, in);
    if (zm != 0u) {
      const uint32_t lo = __reduce_add_sync(0xffffffffu, in ? (e & 0xFFFFu) : 0u);
      const uint32_t hi = __reduce_add_sync(0xffffffffu, in ? (e >> 16) : 0u);
      if (lane == __ffs(zm) - 1) {
        atomicAdd(&hlo[0], lo);
        atomicAdd(&hhi[0], hi);
      }
    }
    member = member && !in;
  }
  if (member) {
    atomicAdd(&hlo[d], e & 0xFFFFu);
    atomicAdd(&hhi[d], e >> 16);
  }
}

// Cluster totals of exchange n (bins [0, nb)) into s.tot.  Every CTA merges
// its histograms into s.send and copies it into inbox[its rank] of every CTA
// of the cluster (itself included) with one bulk shared-to-shared copy per
// rank, which completes transaction bytes on the receiver's xbar (one copy of
// nb * 8 bytes instead of nb remote 8-byte stores: the stores measured ~1.5 us
// per exchange of 256 bins on 16 ranks).  Each CTA then waits for the C ranks'
// bytes and sums them in rank order (so every CTA holds the same totals), and
// arrives on the cluster barrier once it has read its inbox.  A CTA waits on
// that barrier before it copies exchange n + 1, so one inbox suffices and the
// per-rank weights of the last exchange stay readable.  A copy may land before
// the receiver's expect_tx of that exchange; the phase cannot complete before
// the receiver's own arrival.  s.send is rewritten only after that barrier,
// when every copy that read it has landed.
template <class SS>
__device__ void hist_totals(SS& s, int rank, uint32_t n, int nb, int* err) {
  __syncthreads();
  {
    const int lg = nb == 512 ? 9 : 8;
    const int d = threadIdx.x & (nb - 1), q = threadIdx.x >> lg;
    const int per = SS::kHist >> (10 - lg);   // histograms per merge group
    uint32_t lo = 0, hi = 0;
    for (int w = 0; w < per; ++w) {
      lo += s.whist[q * per + w][0][d];
      hi += s.whist[q * per + w][1][d];
    }
    s.qsum[threadIdx.x] = ((unsigned long long)hi << 16) + lo;
  }
  __syncthreads();
  // every rank has read the previous exchange: its copies (which read s.send)
  // have all landed
  if (n > 0) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (threadIdx.x < nb) {
    unsigned long long h = 0;
    for (int q = threadIdx.x; q < kSampThreads; q += nb) h += s.qsum[q];
    s.send[threadIdx.x] = h;
    fence_proxy_async();   // the generic writes, visible to the bulk copies
  }
  __syncthreads();
  const uint32_t bar = smem_u32(&s.xbar);
  if (threadIdx.x == 0) mbar_arrive_expect_tx(&s.xbar, (uint32_t)(SS::kC * nb * sizeof(unsigned long long)));
  if (threadIdx.x < SS::kC) {
    const int r = threadIdx.x;
    uint32_t rdst, rbar;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rdst) : "r"(smem_u32(&s.inbox[rank][0])), "r"(r));
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(bar), "r"(r));
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(rdst), "r"(smem_u32(s.send)), "r"((uint32_t)(nb * sizeof(unsigned long long))), "r"(rbar)
        : "memory");
  }
  if (threadIdx.x < nb) {
    const int d = threadIdx.x;
    const uint32_t parity = n & 1;
    uint32_t ok = 0;
    for (uint32_t it = 0; it < (1u << 22) && !ok; ++it)
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(ok)
          : "r"(bar), "r"(parity)
          : "memory");
    if (!ok) raise_error(err, kDevWaitTimeout);
    unsigned long long sum = 0;
#pragma unroll
    for (int r = 0; r < SS::kC; ++r) sum += s.inbox[r][d];
    s.tot[d] = sum;
  }
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  __syncthreads();
}

// Warp-wide digit scan of 256 digit weights w (descending digits): lane l
// holds digits 255-8l .. 248-8l in v, their sum in mine and the inclusive sum
// over lanes 0..l in incl.
__device__ __forceinline__ void digit_scan(const unsigned long long* w, unsigned long long (&v)[8],
                                           unsigned long long& mine, unsigned long long& incl) {
  const int lane = threadIdx.x & 31;
  mine = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j] = w[255 - 8 * lane - j];
    mine += v[j];
  }
  incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
}

// The largest digit d with above + sum(w[d..255]) >= target (digit 0 when the
// total falls short) and above + sum(w[d+1..255]), in every lane.
__device__ __forceinline__ void digit_pick(const unsigned long long (&v)[8], unsigned long long mine,
                                           unsigned long long incl, unsigned long long above,
                                           unsigned long long target, uint32_t& sel,
                                           unsigned long long& sel_above) {
  const int lane = threadIdx.x & 31;
  const uint32_t hit = __ballot_sync(0xffffffffu, above + incl >= target);
  const int L = hit ? __ffs(hit) - 1 : 31;
  unsigned long long run = above + incl - mine;
  int j = 0;
  for (; j < 7; ++j) {
    if (run + v[j] >= target) break;
    run += v[j];
  }
  sel = (uint32_t)__shfl_sync(0xffffffffu, 255 - 8 * lane - j, L);
  sel_above = __shfl_sync(0xffffffffu, run, L);
}

// Selected digit of the pass: the largest d with above + sum(tot[d..255]) >=
// target (digit 0 when the total falls short) into s.sel, and the weight of
// the digits above it plus `above` into s.sel_above.  One warp: lane l holds
// digits 255-8l .. 248-8l in descending order.
template <class SS>
__device__ void pick_digit(SS& s, unsigned long long above, unsigned long long target) {
  const int lane = threadIdx.x & 31;
  if ((threadIdx.x >> 5) == 0) {
    unsigned long long v[8], mine = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = s.tot[255 - 8 * lane - j];
      mine += v[j];
    }
    unsigned long long incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const uint32_t hit = __ballot_sync(0xffffffffu, above + incl >= target);
    const int L = hit ? __ffs(hit) - 1 : 31;
    if (lane == L) {
      unsigned long long run = above + incl - mine;
      int j = 0;
      for (; j < 7; ++j) {
        if (run + v[j] >= target) break;
        run += v[j];
      }
      s.sel = (uint32_t)(255 - 8 * lane - j);
      s.sel_above = run;
    }
  }
  __syncthreads();
}

// The cutoff select (the value e_star where the weight from the top first
// reaches thr) with the draw select beside it, then the draw's exact
// remainder; shared by the cluster and grid kernels.  On entry s.tot holds the
// totals of pass 0 (built with the weights).  clear(nb) zeroes bins [0, nb) of
// the histograms; totals(nb) runs the next exchange of bins [0, nb) into
// s.tot.  Leaves the drawn value e2, the kept weight above it, R, e2's bin in
// the last exchange, and whether s.tot still holds that exchange's totals
// (else they are the cutoff's pass-3 totals, s.tot1[3]).
template <class SS, int kThreads, int kPer, class ClearF, class TotalsF>
__device__ __forceinline__ void select_draw(SS& s, int n_local, uint32_t p24, uint32_t u,
                                            ClearF&& clear, TotalsF&& totals, uint32_t& e2,
                                            unsigned long long& above, unsigned long long& R,
                                            uint32_t& bin3, bool& tot_real) {
  const int warp = threadIdx.x >> 5;

  // ---- the cutoff select (the value e_star where the weight from the top
  // first reaches thr) and, beside it, the draw select -----------------------
  // The draw wants the first kept id whose running weight exceeds
  // R = floor(kept * u / 2^24), kept = the cutoff's kept weight, which lies in
  // [thr, thr + e_star - 1]; after pass p the cutoff's prefix bounds e_star,
  // so R lies in a known range.  When both ends of the range pick the same
  // digit, that digit is the draw's (the pick is monotone in the target) and
  // the next pass histograms the draw's members too.  While the draw's prefix
  // equals the cutoff's ("on e_star") its digit weights follow from the
  // cutoff's histogram.  Pass 3 has the exact R.  When the ends part, the draw
  // resumes at that pass after the cutoff select, exactly as below.
  if (threadIdx.x == 0) {
    s.an = 0;
    s.ad = 0;
    s.pn = 0;
    s.pd = 0;
    s.dmode = SS::kSpec ? 0 : 2;   // 0 on e_star, 1 parted, 2 left the speculation
    s.dfail = 0;
    s.don = 1;
    s.dhi = 0;
  }
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t mask = pass == 0 ? 0u : 0xFFFFFFFFu << (shift + 8);
    if (pass > 0) {
      __syncthreads();
      const uint32_t pn = s.pn, pd = s.pd;
      const bool dact = SS::kSpec && s.dmode == 1;
      clear(dact ? 512 : 256);
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int i = k * kThreads + (int)threadIdx.x;
        const uint32_t e = i < n_local ? s.e[i] : 0u;
        const bool mn = e != 0u && (e & mask) == pn;
        const bool md = dact && (e & mask) == pd;   // members of the two never overlap
        hist_add(s, mn || md, e, ((e >> shift) & 255u) | (md ? 256u : 0u));
      }
      totals(dact ? 512 : 256);
    }
    if (threadIdx.x < 256) s.tot1[pass][threadIdx.x] = s.tot[threadIdx.x];
    if (warp == 0) {
      const int lane = threadIdx.x & 31;
      unsigned long long v[8], mine, incl;
      digit_scan(s.tot, v, mine, incl);
      if (pass == 0) {
        const unsigned long long S = __shfl_sync(0xffffffffu, incl, 31);
        unsigned long long t = mul_shift24(S, p24);
        if (t == 0) t = 1;
        if (lane == 0) s.thr = t;
      }
      __syncwarp();
      const unsigned long long thr = s.thr, an = s.an;
      uint32_t seln;
      unsigned long long aboven;
      digit_pick(v, mine, incl, an, thr, seln, aboven);
      const uint32_t pn = s.pn | (seln << shift);
      unsigned long long tl = 0, th = 0;
      if (pass == 3) {   // e_star = pn, exact kept and R
        const unsigned long long need = thr - aboven;
        const unsigned long long k_tie = (need + pn - 1) / pn;
        const unsigned long long R = mul_shift24(aboven + k_tie * pn, u);
        tl = th = R + 1;
        if (lane == 0) s.R = R;
      } else {
        const uint32_t e_hi = pn | ((1u << shift) - 1u);
        tl = mul_shift24(thr, u) + 1;
        th = mul_shift24(thr + e_hi - 1, u) + 1;
      }
      int dmode = s.dmode;
      uint32_t pd = s.pd;
      unsigned long long ad = s.ad;
      int dhi = 0;
      if (dmode == 0) {
        // on e_star: the draw stays there when its target lies below the
        // weight above the cutoff's digit, else picks among the digits above it
        if (tl > aboven) {
          pd = pn;
          ad = aboven;
        } else if (th <= aboven) {
          uint32_t sl, sh;
          unsigned long long al, ah;
          digit_pick(v, mine, incl, ad, tl, sl, al);
          digit_pick(v, mine, incl, ad, th, sh, ah);
          if (sl == sh) {
            dmode = 1;
            pd |= sl << shift;
            ad = al;
          } else {
            dmode = 2;
          }
        } else {
          dmode = 2;
        }
      } else if (dmode == 1) {
        unsigned long long w[8], dm, di;
        digit_scan(s.tot + (SS::kBins - 256), w, dm, di);
        uint32_t sl, sh;
        unsigned long long al, ah;
        digit_pick(w, dm, di, ad, tl, sl, al);
        digit_pick(w, dm, di, ad, th, sh, ah);
        if (sl == sh) {
          pd |= sl << shift;
          ad = al;
          dhi = 1;
        } else {
          dmode = 2;
        }
      }
      if (lane == 0) {
        s.an = aboven;
        s.above1[pass] = aboven;
        s.pn = pn;
        if (s.dmode != 2) {
          if (dmode == 2) {   // left at this pass: its state before the pass stays
            s.dfail = pass;
            s.don = s.dmode == 0;
          } else {
            s.pd = pd;
            s.ad = ad;
            s.dhi = dhi;
          }
          s.dmode = dmode;
        }
      }
    }
  }
  __syncthreads();
  const uint32_t e_star = s.pn;
  const unsigned long long above_star = s.an;   // weight of E > e_star
  R = s.R;
  if (s.dmode != 2) {
    e2 = s.pd;
    above = s.ad;
    bin3 = (e2 & 255u) | (s.dhi ? 256u : 0u);
    tot_real = true;
  } else {
    // ---- the draw from the pass at which it left the speculation: the same
    // select over the kept set (E > e_star, plus k_tie copies of e_star as one
    // weight at e_star) for R + 1 --------------------------------------------
    // While the draw's prefix equals e_star's, its digit totals follow from
    // the cutoff select's: above e_star's digit they are the same members; at
    // that digit they are the weight above e_star not yet counted above the
    // prefix, plus the tie weight; below it there are none.  Only passes after
    // the prefixes part scan the weights (and those members all exceed e_star).
    const unsigned long long thr = s.thr;
    const unsigned long long k_tie = (thr - above_star + e_star - 1) / e_star;  // e_star >= 1
    const int pf = s.dfail;
    uint32_t prefix = s.pd;
    above = s.ad;
    bool on_star = s.don != 0;
    tot_real = false;
    for (int pass = pf; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      const uint32_t mask = pass == 0 ? 0u : 0xFFFFFFFFu << (shift + 8);
      const uint32_t ds = (e_star >> shift) & 255u;
      if (on_star) {
        __syncthreads();
        if (threadIdx.x < 256) {
          const uint32_t d = threadIdx.x;
          s.tot[d] = d > ds ? s.tot1[pass][d]
                   : d == ds ? (above_star - s.above1[pass]) + k_tie * e_star : 0ull;
        }
        __syncthreads();
      } else {
        clear(256);
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const int i = k * kThreads + (int)threadIdx.x;
          const uint32_t e = i < n_local ? s.e[i] : 0u;
          hist_add(s, e > e_star && (e & mask) == prefix, e, (e >> shift) & 255u);
        }
        totals(256);
        tot_real = pass == 3;
      }
      pick_digit(s, above, R + 1);
      const uint32_t sel = s.sel;
      on_star = on_star && sel == ds;
      prefix |= sel << shift;
      above = s.sel_above;
    }
    e2 = prefix;
    bin3 = e2 & 255u;
  }
}

template <int C>
__global__ void __launch_bounds__(kSampThreads)
    k_sample(const __half* __restrict__ logits, int row_stride, int vocab, float temperature,
             float top_p, const uint32_t* __restrict__ u24, int32_t* __restrict__ out_ids,
             int* err) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  using SS = SampShared<C>;
  constexpr int kSampPerThread = SS::kPerThread;
  SS& s = *reinterpret_cast<SS*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int seq = blockIdx.y;
  const __half* lg = logits + (size_t)seq * row_stride;
  const int chunk = (vocab + C - 1) / C;
  const int lo = rank * chunk;
  const int n_local = max(0, min(vocab, lo + chunk) - lo);
  if (threadIdx.x == 0) {   // visible to the cluster after the first cluster.sync below
    mbar_init(&s.xbar, 1);
    fence_mbar_init();
  }

  // ---- greedy ---------------------------------------------------------
  if (!(temperature > 0.0f)) {
    float best = -INFINITY;
    int idx = 0x7fffffff;
    __half lv[kSampPerThread];   // all loads in flight before the first compare
#pragma unroll
    for (int k = 0; k < kSampPerThread; ++k) {
      const int i = k * kSampThreads + (int)threadIdx.x;
      lv[k] = i < n_local ? lg[lo + i] : __ushort_as_half((unsigned short)0x7e00u);
    }
#pragma unroll
    for (int k = 0; k < kSampPerThread; ++k) {   // increasing id: the first maximum is kept
      const int i = k * kSampThreads + (int)threadIdx.x;
      const float v = h2f(lv[k]);
      if (!isnan(v) && v > best) { best = v; idx = lo + i; }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    if ((threadIdx.x & 31) == 0) { s.red_f[threadIdx.x >> 5] = best; s.red_i[threadIdx.x >> 5] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (s.red_f[w] > best || (s.red_f[w] == best && s.red_i[w] < idx)) { best = s.red_f[w]; idx = s.red_i[w]; }
      s.cl_f[0] = best;
      s.cl_i = idx;
    }
    cluster.sync();
    if (rank == 0 && threadIdx.x == 0) {
      for (int r = 1; r < C; ++r) {
        SS* rs = cluster.map_shared_rank(&s, r);
        const float v = rs->cl_f[0];
        const int i = rs->cl_i;
        if (v > best || (v == best && i < idx)) { best = v; idx = i; }
      }
      out_ids[seq] = (best == -INFINITY) ? kStopToken : idx;
    }
    cluster.sync();
    return;
  }

  // ---- scale + max ---------------------------------------------------
  // The scaled logits stay in registers when a thread has few (C >= 8), else
  // they go through e (each thread reads back only what it wrote).
  constexpr bool kRegs = kSampPerThread <= 20;
  float sc[kRegs ? kSampPerThread : 1];
  float mx = -INFINITY;
  if constexpr (kRegs) {
#pragma unroll
    for (int k = 0; k < kSampPerThread; ++k) {
      const int i = k * kSampThreads + (int)threadIdx.x;
      sc[k] = i < n_local ? h2f(lg[lo + i]) : __int_as_float(0x7fc00000);
    }
#pragma unroll
    for (int k = 0; k < kSampPerThread; ++k) {
      float x = 0.0f;
      if (!isnan(sc[k])) {     // NaN logits keep 0.0 and stay out of the maximum
        x = __fdiv_rn(sc[k], temperature);
        mx = fmaxf(mx, x);
      }
      sc[k] = x;
    }
  } else {
    // every logit of the thread loaded before the first is used (the loads
    // are the pass's latency: four in flight at a time cost ~10 us)
    __half lv[kSampPerThread];
#pragma unroll
    for (int k = 0; k < kSampPerThread; ++k) {
      const int i = k * kSampThreads + (int)threadIdx.x;
      lv[k] = i < n_local ? lg[lo + i] : __ushort_as_half((unsigned short)0x7e00u);
    }
#pragma unroll
    for (int k = 0; k < kSampPerThread; ++k) {
      const int i = k * kSampThreads + (int)threadIdx.x;
      if (i < n_local) {
        const float v = h2f(lv[k]);
        float x = 0.0f;
        if (!isnan(v)) {
          x = __fdiv_rn(v, temperature);
          mx = fmaxf(mx, x);
        }
        s.e[i] = __float_as_uint(x);
      }
    }
  }
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) s.red_f[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, s.red_f[w]);
    s.cl_f[0] = m;
  }
  cluster.sync();
  __shared__ float s_M;
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int r = 0; r < C; ++r) m = fmaxf(m, cluster.map_shared_rank(&s, r)->cl_f[0]);
    s_M = m;
  }
  __syncthreads();
  const float M = s_M;
  if (M == -INFINITY) {
    if (rank == 0 && threadIdx.x == 0) out_ids[seq] = kStopToken;
    cluster.sync();
    return;
  }
  // ---- fixed-point weights, histogrammed by their first digit -----------
  // The first pass of the cutoff select needs every weight, so it is built
  // here; the total S is the sum of its cluster totals.
  hist_clear(s, 256);
#pragma unroll
  for (int k = 0; k < kSampPerThread; ++k) {
    const int i = k * kSampThreads + (int)threadIdx.x;
    uint32_t E = 0u;
    if (i < n_local) {
      float x;
      if constexpr (kRegs) x = sc[k];
      else x = __uint_as_float(s.e[i]);
      const float e = sampler_exp(__fsub_rn(x, M));
      E = __float2uint_rz(__fmul_rn(e, 2147483648.0f));
      s.e[i] = E;
    }
    hist_add(s, E != 0u, E, E >> 24);
  }
  uint32_t xn = 0;   // exchanges so far
  hist_totals(s, rank, xn++, 256, err);
  const float pc = fminf(fmaxf(top_p, 0.0f), 1.0f);
  const uint32_t p24 = (uint32_t)__float2uint_rz(__fmul_rn(pc, 16777216.0f));
  const uint32_t u = u24[seq] & 0xFFFFFFu;
  uint32_t e2, bin3;
  unsigned long long above, R;
  bool tot_real;
  select_draw<SS, kSampThreads, kSampPerThread>(
      s, n_local, p24, u, [&](int nb) { hist_clear(s, nb); },
      [&](int nb) { hist_totals(s, rank, xn++, nb, err); }, e2, above, R, bin3, tot_real);
  const unsigned long long j = (R - above) / e2;   // index inside the tie group (id order)

  // ---- j-th smallest id with E == e2 ---------------------------------------
  // The last exchange holds every rank's weight at e2's final digit, which is
  // that rank's count of E == e2 times e2: the ranks before this one hold
  // `before` of them, this one `cnt`.  Threads own contiguous id ranges so that
  // block order = id order.
  unsigned long long before = 0, cnt = 0;
  for (int r = 0; r < C; ++r) {
    const unsigned long long w = s.inbox[r][bin3];
    if (r < rank) before += w;
    if (r == rank) cnt = w;
  }
  before /= e2;
  cnt /= e2;
  if (j >= before && j < before + cnt) {
    const int per = (n_local + (int)blockDim.x - 1) / (int)blockDim.x;
    const int b0 = threadIdx.x * per, b1 = min(n_local, b0 + per);
    uint32_t c = 0;
    for (int i = b0; i < b1; ++i) c += (s.e[i] == e2);
    const uint32_t incl = block_incl_scan_u32(c, s), excl = incl - c;
    if (j >= before + excl && j < before + incl) {
      unsigned long long want = j - before - excl;
      for (int i = b0; i < b1; ++i) {
        if (s.e[i] == e2) {
          if (want == 0) { out_ids[seq] = lo + i; break; }
          --want;
        }
      }
    }
  }
  // pairs with the last exchange's arrival: no CTA leaves while a peer may
  // still read its shared memory
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}


// ---- one sequence over the whole GPU ----------------------------------------
// Batch-1 top-p: a 16-CTA cluster leaves 132 SMs idle while each of its CTAs
// histograms 9,496 ids a pass.  Here every SM takes ceil(vocab / grid) ids (at
// most 5 a thread), and the exchanges go through device memory: each CTA adds
// its nonzero digit sums into the exchange's totals with 64-bit reductions
// (integer sums: the order of the adds cannot change them), then passes a
// bounded grid barrier.  The launch is cooperative (every CTA resident).  The
// scratch is zero before the first launch and is left zero: exchange n-1's
// totals are cleared by one CTA after exchange n's barrier (every CTA has read
// them by then), the rest by the last CTA to finish.
constexpr int kGridThreads = 256;
constexpr int kGridPerThread = 5;
constexpr int kGridMaxIds = kGridThreads * kGridPerThread;   // 1,280: grids of >= 119 CTAs
constexpr int kGridMaxX = 8;                                 // 4 cutoff passes + at most 3 draw passes
constexpr int kGridMaxCtas = 1024;

struct GridScratch {
  unsigned long long tot[kGridMaxX][512];   // grid-wide digit totals per exchange
  uint32_t cnt[kGridMaxCtas];               // per-CTA counts of the drawn value (tie groups)
  uint32_t bar;                             // grid barrier arrivals
  uint32_t done;                            // CTAs finished
  uint32_t maxbits;                         // order-preserving bits of the largest scaled logit
  uint32_t pad;
};

struct GridShared {
  static constexpr bool kSpec = true;
  static constexpr int kBins = 512;
  static constexpr int kHist = kGridThreads / 32;   // one digit histogram per warp
  static constexpr int kWarpsPerHist = 1;
  uint32_t e[kGridMaxIds];
  uint32_t whist[kHist][2][kBins];
  unsigned long long tot[kBins];
  unsigned long long tot1[4][256];
  unsigned long long above1[4];
  float red_f[32];
  uint32_t red_c[32];
  unsigned long long red_u[32];
  uint32_t sel;
  unsigned long long sel_above;
  unsigned long long thr, an, ad, R;
  uint32_t pn, pd;
  int dmode, dfail, don, dhi;
  uint32_t cta_cnt;
  int last;
};

__device__ __forceinline__ uint32_t float_order(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float float_unorder(uint32_t m) {
  return __uint_as_float((m & 0x80000000u) ? (m & 0x7FFFFFFFu) : ~m);
}

// Limits of the grid kernel's barrier waits: wait_ns of %globaltimer; stall
// (test hook, the engine's test_stall): CTA 0 does not arrive at barrier
// kGridStallBarrier, so the others' waits run out.
struct GridWait {
  unsigned long long wait_ns;
  int stall;
  int* err;
};
constexpr int kGridWaitSite = 20;       // wait site reported in err[1] (x 100 + barrier)
constexpr int kGridStallBarrier = 1;    // the first exchange's barrier

__device__ __forceinline__ unsigned long long grid_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Thread 0's wait for `target` arrivals.  Every 64th poll looks at the error
// word (a CTA that gave up ends the others' waits) and the clock; a timeout
// records err[1] = site, err[2] = CTA (the first failure wins).
__device__ __noinline__ void grid_wait(const uint32_t* bar, uint32_t target, const GridWait& w,
                                       int site) {
  unsigned long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire_u32(bar) >= target) return;
    if ((it & 63) == 63) {
      if (w.err && *reinterpret_cast<volatile int*>(w.err) != 0) return;
      const unsigned long long now = grid_now();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > w.wait_ns) {
        if (w.err && atomicCAS(w.err, 0, kDevWaitTimeout) == 0) {
          w.err[1] = site;
          w.err[2] = blockIdx.x;
          w.err[3] = 0;
        }
        return;
      }
      __nanosleep(64);
    }
  }
}

// Every CTA arrives at barrier `index` (its target is index + 1 arrivals of
// every CTA), then waits.  The block barrier orders the CTA's writes before
// thread 0's release add, and its acquire load before the CTA's later reads
// (explicit fences around them measured 2 us slower a call).
__device__ __forceinline__ void grid_sync(GridScratch* g, uint32_t index, const GridWait& w) {
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!(w.stall && blockIdx.x == 0 && index == kGridStallBarrier)) red_release_add_u32(&g->bar, 1u);
    grid_wait(&g->bar, gridDim.x * (index + 1), w, kGridWaitSite * 100 + (int)index);
  }
  __syncthreads();
}

// Zeroes bins [0, nb) of the warps' histograms (once, before the weights pass:
// every merge then leaves the bins it read zero).
__device__ __forceinline__ void grid_hist_clear(GridShared& s, int nb) {
  const int lg = nb == 512 ? 9 : 8;
  uint32_t* h = &s.whist[0][0][0];
  for (int i = threadIdx.x; i < GridShared::kHist * 2 * nb; i += kGridThreads)
    h[(i >> lg) * GridShared::kBins + (i & (nb - 1))] = 0;
  __syncthreads();
}

// Exchange n of bins [0, nb): barrier n + 1 (barrier 0 is the maximum's).
__device__ void grid_totals(GridShared& s, GridScratch* g, uint32_t n, int nb, int nblk,
                            const GridWait& w) {
  __syncthreads();
  for (int b = threadIdx.x; b < nb; b += kGridThreads) {
    uint32_t lo = 0, hi = 0;   // at most 1,280 weights: each half fits 32 bits
#pragma unroll
    for (int w = 0; w < GridShared::kHist; ++w) {
      lo += s.whist[w][0][b];
      hi += s.whist[w][1][b];
      s.whist[w][0][b] = 0u;   // left zero for the next pass
      s.whist[w][1][b] = 0u;
    }
    const unsigned long long h = ((unsigned long long)hi << 16) + lo;
    if (h) atomicAdd(&g->tot[n][b], h);
  }
  grid_sync(g, n + 1, w);
  if (n > 0 && (int)blockIdx.x == (int)(n % (uint32_t)nblk))
    for (int b = threadIdx.x; b < 512; b += kGridThreads) g->tot[n - 1][b] = 0ull;
  for (int b = threadIdx.x; b < nb; b += kGridThreads) s.tot[b] = __ldcg(&g->tot[n][b]);
  __syncthreads();
}

__global__ void __launch_bounds__(kGridThreads, 1)
    k_sample_grid(const __half* __restrict__ logits, int vocab, float temperature, float top_p,
                  const uint32_t* __restrict__ u24, int32_t* __restrict__ out_ids,
                  GridScratch* __restrict__ g, int* err, unsigned long long wait_ns, int stall) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  GridShared& s = *reinterpret_cast<GridShared*>(smem_raw);
  const int nblk = gridDim.x, rank = blockIdx.x;
  const int chunk = (vocab + nblk - 1) / nblk;
  const int lo = rank * chunk;
  const int n_local = max(0, min(vocab, lo + chunk) - lo);
  const int tid = threadIdx.x, warp = tid >> 5;
  uint32_t xn = 0;   // exchanges so far
  const GridWait w{wait_ns, stall, err};

  // ---- scale + max (NaN logits keep 0.0 and stay out of the maximum) ----
  float sc[kGridPerThread];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < kGridPerThread; ++k) {
    const int i = k * kGridThreads + tid;
    sc[k] = i < n_local ? h2f(logits[lo + i]) : __int_as_float(0x7fc00000);
  }
#pragma unroll
  for (int k = 0; k < kGridPerThread; ++k) {
    float x = 0.0f;
    if (!isnan(sc[k])) {
      x = __fdiv_rn(sc[k], temperature);
      mx = fmaxf(mx, x);
    }
    sc[k] = x;
  }
  mx = warp_max(mx);
  if ((tid & 31) == 0) s.red_f[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = -INFINITY;
    for (int w = 0; w < kGridThreads / 32; ++w) m = fmaxf(m, s.red_f[w]);
    if (m != -INFINITY) atomicMax(&g->maxbits, float_order(m));
  }
  grid_sync(g, 0, w);
  const uint32_t mb = __ldcg(&g->maxbits);
  if (mb == 0u) {   // every logit NaN (InferenceEngine.swift:311-315)
    if (rank == 0 && tid == 0) out_ids[0] = kStopToken;
  } else {
    const float M = float_unorder(mb);
    // ---- fixed-point weights, histogrammed by their first digit ----------
    grid_hist_clear(s, 512);   // every later merge leaves the bins it read zero
#pragma unroll
    for (int k = 0; k < kGridPerThread; ++k) {
      const int i = k * kGridThreads + tid;
      uint32_t E = 0u;
      if (i < n_local) {
        const float e = sampler_exp(__fsub_rn(sc[k], M));
        E = __float2uint_rz(__fmul_rn(e, 2147483648.0f));
        s.e[i] = E;
      }
      hist_add(s, E != 0u, E, E >> 24);
    }
    grid_totals(s, g, xn++, 256, nblk, w);
    const float pc = fminf(fmaxf(top_p, 0.0f), 1.0f);
    const uint32_t p24 = (uint32_t)__float2uint_rz(__fmul_rn(pc, 16777216.0f));
    const uint32_t u = u24[0] & 0xFFFFFFu;
    uint32_t e2, bin3;
    unsigned long long above, R;
    bool tot_real;
    select_draw<GridShared, kGridThreads, kGridPerThread>(
        s, n_local, p24, u, [&](int) {},
        [&](int nb) { grid_totals(s, g, xn++, nb, nblk, w); }, e2, above, R, bin3, tot_real);
    const unsigned long long j = (R - above) / e2;   // index inside the tie group (id order)
    const unsigned long long total = (tot_real ? s.tot[bin3] : s.tot1[3][bin3]) / e2;

    // ---- j-th smallest id with E == e2: threads own contiguous id ranges so
    // that block order = id order; with more than one such id the CTAs'
    // counts go through device memory behind one more barrier ---------------
    const int per = (n_local + kGridThreads - 1) / kGridThreads;
    const int b0 = tid * per, b1 = min(n_local, b0 + per);
    uint32_t c = 0;
    for (int i = b0; i < b1; ++i) c += (s.e[i] == e2);
    const uint32_t incl = block_incl_scan_u32(c, s), excl = incl - c;
    if (tid == kGridThreads - 1) s.cta_cnt = incl;
    __syncthreads();
    unsigned long long before = 0;
    if (total > 1) {
      if (tid == 0) g->cnt[rank] = s.cta_cnt;
      grid_sync(g, xn + 1, w);
      unsigned long long part = 0;
      for (int r = tid; r < rank; r += kGridThreads) part += __ldcg(&g->cnt[r]);
      before = block_sum_u64(part, s);
    }
    if (j >= before + excl && j < before + incl) {
      unsigned long long want = j - before - excl;
      for (int i = b0; i < b1; ++i) {
        if (s.e[i] == e2) {
          if (want == 0) { out_ids[0] = lo + i; break; }
          --want;
        }
      }
    }
  }

  // ---- leave the scratch zero for the next launch ----
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s.last = atomicAdd(&g->done, 1u) == (uint32_t)(nblk - 1);
  }
  __syncthreads();
  if (s.last) {
    __threadfence();
    if (xn > 0)
      for (int b = tid; b < 512; b += kGridThreads) g->tot[xn - 1][b] = 0ull;
    for (int r = tid; r < nblk; r += kGridThreads) g->cnt[r] = 0u;
    if (tid == 0) {
      g->maxbits = 0u;
      g->bar = 0u;
      g->done = 0u;
    }
  }
}

size_t sampler_scratch_bytes(int n_seq) { return n_seq == 1 ? sizeof(GridScratch) : 0; }

// Cooperative launch over every SM; 1 when the grid path does not apply
// (a device with too few SMs for 1,280 ids a CTA).
static int launch_sample_grid(const __half* logits, int vocab, float temperature, float top_p,
                              const uint32_t* u24, int32_t* out_ids, void* scratch, int* err,
                              cudaStream_t st, unsigned long long wait_ns, int stall) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return -1;
  const int nblk = min(sms, kGridMaxCtas);
  if (nblk < 1 || (vocab + nblk - 1) / nblk > kGridMaxIds) return 1;
  const size_t smem = sizeof(GridShared);
  if (cudaFuncSetAttribute(k_sample_grid, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nblk);
  cfg.blockDim = dim3(kGridThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_sample_grid, logits, vocab, temperature, top_p, u24, out_ids,
                            reinterpret_cast<GridScratch*>(scratch), err, wait_ns, stall) == cudaSuccess
             ? 0
             : -1;
}

template <int C>
static int launch_sample_c(const __half* logits, int n_seq, int row_stride, int vocab,
                           float temperature, float top_p, const uint32_t* u24, int32_t* out_ids,
                           int* err, cudaStream_t st) {
  const size_t smem = sizeof(SampShared<C>);
  cudaFuncSetAttribute(k_sample<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (C > 8) cudaFuncSetAttribute(k_sample<C>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, n_seq);
  cfg.blockDim = dim3(kSampThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_sample<C>, logits, row_stride, vocab, temperature, top_p, u24,
                            out_ids, err) == cudaSuccess ? 0 : -1;
}

// How many C-CTA clusters of k_sample<C> fit on the device at once (0 when the
// occupancy calculator refuses the size).
template <int C>
static int active_clusters() {
  int n = 0;
  const size_t smem = sizeof(SampShared<C>);
  if (cudaFuncSetAttribute(k_sample<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return 0;
  if (C > 8 &&
      cudaFuncSetAttribute(k_sample<C>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, 1);
  cfg.blockDim = dim3(kSampThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaOccupancyMaxActiveClusters(&n, k_sample<C>, &cfg) != cudaSuccess) n = 0;
  return n;
}

// Cluster size per batch: a CTA's time barely depends on how many ids it owns
// (fixed per-pass costs dominate), so a batch takes as many rounds as it needs
// waves of clusters.  16-CTA clusters (the fewest ids per CTA) when the batch
// fits in one wave of them, 8 when it fits in one wave of those, else 4 (the
// most clusters at once).  16 is a non-portable size.  The counts are asked of
// the occupancy calculator once per device (sampler_prepare asks ahead of a
// stream capture).
static int sample_cluster_size(int dev, int n_seq) {
  static int fit16[64], fit8[64];
  static bool known[64];
  if (dev < 0 || dev >= 64) return 8;
  if (!known[dev]) {
    fit16[dev] = active_clusters<16>();
    fit8[dev] = active_clusters<8>();
    cudaGetLastError();   // a refused query leaves no error behind for the next launch check
    known[dev] = true;
  }
  if (n_seq <= fit16[dev]) return 16;
  if (n_seq <= fit8[dev]) return 8;
  return 4;
}

void sampler_prepare() {
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) sample_cluster_size(dev, 1);
}

int launch_sample(const __half* logits, int n_seq, int row_stride, int vocab, float temperature,
                  float top_p, const uint32_t* u24, int32_t* out_ids, void* scratch, int* err,
                  cudaStream_t st, unsigned long long wait_ns, int stall) {
  if (vocab <= 0 || vocab > kVocab || n_seq <= 0) return -1;
  if (scratch && n_seq == 1 && temperature > 0.0f) {
    const int rc = launch_sample_grid(logits, vocab, temperature, top_p, u24, out_ids, scratch, err,
                                      st, wait_ns, stall);
    if (rc <= 0) return rc;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  switch (sample_cluster_size(dev, n_seq)) {
    case 16:
      return launch_sample_c<16>(logits, n_seq, row_stride, vocab, temperature, top_p, u24, out_ids,
                                 err, st);
    case 8:
      return launch_sample_c<8>(logits, n_seq, row_stride, vocab, temperature, top_p, u24, out_ids,
                                err, st);
    default:
      return launch_sample_c<4>(logits, n_seq, row_stride, vocab, temperature, top_p, u24, out_ids,
                                err, st);
  }
}

}  // namespace qwen
