// sampler.cu -- on-device token sampler (extractNextTokenID,
// InferenceEngine.swift:273-368) as a radix select over a thread-block cluster.
//
// One cluster of 8 CTAs per sequence; CTA r owns ids [r*chunk, (r+1)*chunk)
// and keeps their fixed-point weights in shared memory.  Cluster-wide
// reductions go through distributed shared memory (hardware cluster barriers,
// no spin loops).
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
#include <cooperative_groups.h>

#include "qwen_common.cuh"
#include "qwen_internal.h"

namespace cg = cooperative_groups;

namespace qwen {

constexpr int kSampCluster = 8;
constexpr int kSampThreads = 1024;
constexpr int kSampMaxChunk = (kVocab + kSampCluster - 1) / kSampCluster;  // 18992

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

struct SampShared {
  uint32_t e[kSampMaxChunk];                 // scaled floats, then fixed-point weights
  unsigned long long hsum[2][256];
  uint32_t hcnt[2][256];
  float red_f[32];
  int red_i[32];
  unsigned long long red_u[32];
  float cl_f[kSampCluster];                  // per-CTA partials read by the cluster
  int cl_i;
  unsigned long long cl_u;
  uint32_t cl_cnt;
};

__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v, SampShared& s) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) s.red_u[w] = v;
  __syncthreads();
  unsigned long long t = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += s.red_u[i];
  return t;
}

// Weighted radix select over E (descending).  Elements are the CTA's E values
// with E > floor_excl... membership: E > e_star always, E == e_star counted with
// total weight tie_weight (handled via the tie term), E < e_star excluded --
// when e_star == 0 every element takes part.  Returns the selected value and
// the weight strictly above it; *cnt_eq receives the number of equal elements.
struct SelectResult {
  uint32_t value;
  unsigned long long above;
  uint32_t cnt_eq;
};

__device__ SelectResult radix_select(SampShared& s, cg::cluster_group& cluster, int n_local,
                                     unsigned long long target, bool restrict_kept,
                                     uint32_t e_star, unsigned long long tie_weight) {
  uint32_t prefix = 0, mask = 0;
  unsigned long long above = 0;
  uint32_t cnt_eq = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const int b = pass & 1;
    // Warp-aggregated histogram: lanes holding the same digit combine their
    // count and weight (as two 16-bit halves, exact) so that one lane per
    // distinct digit per warp touches shared memory.  Near-flat distributions
    // put most weights in a few digits; per-lane atomics would serialise.
    const int n_iter = (n_local + (int)blockDim.x - 1) / (int)blockDim.x;
    for (int k = 0; k < n_iter; ++k) {
      const int i = k * (int)blockDim.x + (int)threadIdx.x;
      uint32_t e = 0, d = 0xFFFFFFFFu;
      if (i < n_local) {
        e = s.e[i];
        const bool member = (e & mask) == prefix && !(restrict_kept && e <= e_star);
        if (member) d = (e >> shift) & 255u;
      }
      const uint32_t grp = __match_any_sync(0xffffffffu, d);
      const uint32_t lo = __reduce_add_sync(grp, d == 0xFFFFFFFFu ? 0u : (e & 0xFFFFu));
      const uint32_t hi = __reduce_add_sync(grp, d == 0xFFFFFFFFu ? 0u : (e >> 16));
      const int leader = __ffs(grp) - 1;
      if (d != 0xFFFFFFFFu && (int)(threadIdx.x & 31) == leader) {
        atomicAdd(&s.hsum[b][d], ((unsigned long long)hi << 16) + (unsigned long long)lo);
        atomicAdd(&s.hcnt[b][d], (uint32_t)__popc(grp));
      }
    }
    cluster.sync();
    // Totals per digit over the cluster (every CTA computes the same).
    __shared__ unsigned long long tot[256];
    __shared__ uint32_t totc[256];
    if (threadIdx.x < 256) {
      const int d = threadIdx.x;
      unsigned long long part[kSampCluster];
      uint32_t partc[kSampCluster];
#pragma unroll
      for (int r = 0; r < kSampCluster; ++r) {
        SampShared* rs = cluster.map_shared_rank(&s, r);
        part[r] = rs->hsum[b][d];
        partc[r] = rs->hcnt[b][d];
      }
      unsigned long long sum = 0;
      uint32_t c = 0;
#pragma unroll
      for (int r = 0; r < kSampCluster; ++r) {
        sum += part[r];
        c += partc[r];
      }
      if (restrict_kept && (e_star & mask) == prefix && (uint32_t)d == ((e_star >> shift) & 255u))
        sum += tie_weight;
      tot[d] = sum;
      totc[d] = c;
    }
    __syncthreads();
    // Zero the other buffer for the next pass (its last readers finished
    // before this pass's cluster barrier).
    for (int d = threadIdx.x; d < 256; d += blockDim.x) {
      s.hsum[b ^ 1][d] = 0;
      s.hcnt[b ^ 1][d] = 0;
    }
    // Selected digit: the largest d with above + sum(tot[d..255]) >= target.
    // Suffix sums by a block scan over the 256 digits (thread d holds digit 255-d).
    __shared__ unsigned long long suf[256];
    __shared__ uint32_t sel;
    __shared__ unsigned long long sel_above;
    if (threadIdx.x < 256) suf[threadIdx.x] = tot[255 - threadIdx.x];
    __syncthreads();
    for (int off = 1; off < 256; off <<= 1) {
      unsigned long long v = 0;
      if (threadIdx.x < 256 && threadIdx.x >= (unsigned)off) v = suf[threadIdx.x - off];
      __syncthreads();
      if (threadIdx.x < 256) suf[threadIdx.x] += v;
      __syncthreads();
    }
    if (threadIdx.x == 0) sel = 0, sel_above = above;
    __syncthreads();
    if (threadIdx.x < 256) {
      // suf[i] = sum of digits 255-i .. 255; digit d = 255 - i.
      const int i = threadIdx.x, d = 255 - i;
      const unsigned long long incl = above + suf[i];
      const unsigned long long excl = incl - tot[d];
      if ((incl >= target && excl < target) || (d == 0 && incl < target)) {
        sel = (uint32_t)d;
        sel_above = excl;
      }
    }
    __syncthreads();
    prefix |= sel << shift;
    mask |= 255u << shift;
    above = sel_above;
    cnt_eq = totc[sel];
    __syncthreads();
  }
  // Leave both buffers zero for a later select.
  cluster.sync();
  for (int d = threadIdx.x; d < 256; d += blockDim.x) {
    s.hsum[0][d] = s.hsum[1][d] = 0;
    s.hcnt[0][d] = s.hcnt[1][d] = 0;
  }
  __syncthreads();
  return SelectResult{prefix, above, cnt_eq};
}

__global__ void __cluster_dims__(kSampCluster, 1, 1) __launch_bounds__(kSampThreads)
    k_sample(const __half* __restrict__ logits, int row_stride, int vocab, float temperature,
             float top_p, const uint32_t* __restrict__ u24, int32_t* __restrict__ out_ids,
             int* err) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SampShared& s = *reinterpret_cast<SampShared*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int seq = blockIdx.y;
  const __half* lg = logits + (size_t)seq * row_stride;
  const int chunk = (vocab + kSampCluster - 1) / kSampCluster;
  const int lo = rank * chunk;
  const int n_local = max(0, min(vocab, lo + chunk) - lo);

  for (int d = threadIdx.x; d < 256; d += blockDim.x) {
    s.hsum[0][d] = s.hsum[1][d] = 0;
    s.hcnt[0][d] = s.hcnt[1][d] = 0;
  }

  // ---- greedy ---------------------------------------------------------
  if (!(temperature > 0.0f)) {
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < n_local; i += blockDim.x) {
      const float v = h2f(lg[lo + i]);
      if (isnan(v)) continue;
      if (v > best) { best = v; idx = lo + i; }   // increasing i: first max kept
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
      for (int r = 1; r < kSampCluster; ++r) {
        SampShared* rs = cluster.map_shared_rank(&s, r);
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
  float* sc = reinterpret_cast<float*>(s.e);
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n_local; i += blockDim.x) {
    const float v = h2f(lg[lo + i]);
    float x = 0.0f;
    if (!isnan(v)) {
      x = __fdiv_rn(v, temperature);
      mx = fmaxf(mx, x);
    }
    sc[i] = x;
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
    for (int r = 0; r < kSampCluster; ++r) m = fmaxf(m, cluster.map_shared_rank(&s, r)->cl_f[0]);
    s_M = m;
  }
  __syncthreads();
  const float M = s_M;
  if (M == -INFINITY) {
    if (rank == 0 && threadIdx.x == 0) out_ids[seq] = kStopToken;
    cluster.sync();
    return;
  }
  // ---- fixed-point weights + sum ---------------------------------------
  unsigned long long part = 0;
  for (int i = threadIdx.x; i < n_local; i += blockDim.x) {
    const float e = sampler_exp(__fsub_rn(sc[i], M));
    const uint32_t E = __float2uint_rz(__fmul_rn(e, 2147483648.0f));
    s.e[i] = E;
    part += E;
  }
  part = block_sum_u64(part, s);
  if (threadIdx.x == 0) s.cl_u = part;
  cluster.sync();
  __shared__ unsigned long long s_S;
  if (threadIdx.x == 0) {
    unsigned long long t = 0;
    for (int r = 0; r < kSampCluster; ++r) t += cluster.map_shared_rank(&s, r)->cl_u;
    s_S = t;
  }
  __syncthreads();
  const unsigned long long S = s_S;
  const float pc = fminf(fmaxf(top_p, 0.0f), 1.0f);
  const uint32_t p24 = (uint32_t)__float2uint_rz(__fmul_rn(pc, 16777216.0f));
  unsigned long long thr = mul_shift24(S, p24);
  if (thr == 0) thr = 1;

  // ---- nucleus cutoff ----------------------------------------------------
  const SelectResult c1 = radix_select(s, cluster, n_local, thr, false, 0, 0);
  const uint32_t e_star = c1.value;
  const unsigned long long need = thr - c1.above;
  const unsigned long long k_tie = (need + e_star - 1) / e_star;  // e_star >= 1
  const unsigned long long kept = c1.above + k_tie * e_star;

  // ---- draw ----------------------------------------------------------------
  const unsigned long long R = mul_shift24(kept, u24[seq] & 0xFFFFFFu);
  const SelectResult c2 = radix_select(s, cluster, n_local, R + 1, true, e_star, k_tie * e_star);
  const uint32_t e2 = c2.value;
  const unsigned long long j = (R - c2.above) / e2;   // index inside the tie group (id order)

  // ---- j-th smallest id with E == e2 ---------------------------------------
  // Threads own contiguous id ranges so that block order = id order.
  const int per = (n_local + (int)blockDim.x - 1) / (int)blockDim.x;
  const int b0 = threadIdx.x * per, b1 = min(n_local, b0 + per);
  uint32_t cnt = 0;
  for (int i = b0; i < b1; ++i) cnt += (s.e[i] == e2);
  // block exclusive scan of cnt
  __shared__ uint32_t scan[kSampThreads];
  scan[threadIdx.x] = cnt;
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {
    const uint32_t v = threadIdx.x >= (unsigned)off ? scan[threadIdx.x - off] : 0u;
    __syncthreads();
    scan[threadIdx.x] += v;
    __syncthreads();
  }
  const uint32_t incl = scan[threadIdx.x], excl = incl - cnt;
  if (threadIdx.x == blockDim.x - 1) s.cl_cnt = incl;
  cluster.sync();
  __shared__ unsigned long long s_before;
  if (threadIdx.x == 0) {
    unsigned long long t = 0;
    for (int r = 0; r < rank; ++r) t += cluster.map_shared_rank(&s, r)->cl_cnt;
    s_before = t;
  }
  __syncthreads();
  const unsigned long long before = s_before;
  if (j >= before + excl && j < before + incl) {
    unsigned long long want = j - before - excl;
    for (int i = b0; i < b1; ++i) {
      if (s.e[i] == e2) {
        if (want == 0) { out_ids[seq] = lo + i; break; }
        --want;
      }
    }
  }
  cluster.sync();
}

size_t sampler_scratch_bytes(int) { return 0; }

int launch_sample(const __half* logits, int n_seq, int row_stride, int vocab, float temperature,
                  float top_p, const uint32_t* u24, int32_t* out_ids, void*, int* err,
                  cudaStream_t st) {
  if (vocab <= 0 || vocab > kVocab || n_seq <= 0) return -1;
  const size_t smem = sizeof(SampShared);
  cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(kSampCluster, n_seq);
  k_sample<<<grid, kSampThreads, smem, st>>>(logits, row_stride, vocab, temperature, top_p, u24,
                                             out_ids, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace qwen
