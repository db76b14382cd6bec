// attention.cu -- split-K GQA decode attention (flash-decoding) for 12 query
// heads over 2 KV heads, head_dim 128, FP16 KV cache.
//
// Replaces attention_scores -> softmax -> attn_weighted_sum
// (attention.metal:9-56, activations.metal:29-55; InferenceEngine.swift:162-182):
//   s_t = 0.088388 * q_h . K_t,   p_t = exp(s_t - max) / sum,   o_h = sum_t p_t V_t
// evaluated as an online softmax over position chunks.
//
// Grid (splits, 2 kv heads, sequences).  A CTA owns one chunk of positions of
// one (sequence, kv head) and serves all 6 query heads of that group from a
// single read of K and V.  Each of its 4 warps walks 16-position sub-tiles:
//   S^T[16 pos x 8 heads] = K[16 x 128] . q^T   (8 m16n8k16 MMAs, K straight
//                                                from global, q in registers)
//   o^T[128 x 8]        += V^T[128 x 16] . P^T  (V staged in shared memory and
//                                                read with ldmatrix.trans; P is
//                                                split into fp16 hi + lo parts so
//                                                the product keeps ~22 bits)
// Warps merge in shared memory; chunks merge in a fixed order by the last CTA
// of the (sequence, kv head) to finish (an atomic ticket -- nothing waits), so
// results do not depend on scheduling.
#include "qwen_common.cuh"
#include "qwen_internal.h"

namespace qwen {

namespace {

constexpr int kAttnWarps = 4;
constexpr int kSub = 16;  // positions per warp sub-tile
constexpr int kMinSplitLen = kAttnWarps * kSub;  // 64 positions: one sub-tile per warp
constexpr int kMaxSplits = 32;                   // bounds the merge of one (sequence, kv head)
constexpr int kAttnCtaTarget = 148 * 8;          // ~8 resident CTAs per SM

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// Output element (seq, col): row-major out, or the activation tile layout
// ([col/64][row][128 B], 16-byte chunk j of row r at (j ^ (r & 7))).
__device__ __forceinline__ void store_out(const AttnParams& p, int seq, int col, float v) {
  if (p.act_out) {
    const int c = col >> 6, j = (col >> 3) & 7;
    const size_t off = ((size_t)c * p.act_nb + seq) * 128 + (((uint32_t)j ^ (uint32_t)(seq & 7)) << 4) +
                       (col & 7) * 2;
    *reinterpret_cast<__half*>(p.act_out + off) = f2h(v);
  } else {
    p.out[(size_t)seq * p.out_seq_stride + col] = f2h(v);
  }
}

}  // namespace

// V sub-tile rows are padded to 272 B so the 8 row addresses of each
// ldmatrix phase fall in distinct banks.
constexpr int kVRowBytes = 272;

__global__ void __launch_bounds__(128) k_attention_decode(AttnParams p) {
  __shared__ __align__(16) uint8_t vs[kAttnWarps][kSub * kVRowBytes];
  __shared__ __align__(16) uint16_t pt[kAttnWarps][2][kSub * 8];  // P^T hi/lo, [pos][head]
  __shared__ float wm[kAttnWarps][8], wl[kAttnWarps][8];
  __shared__ float wo[kAttnWarps][6][kHeadDim];
  __shared__ uint32_t s_ticket;

  // As a programmatic dependent: let the next kernel launch, then wait for the
  // previous one (no-ops in a plain launch).
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();
  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const uint32_t L = p.seq_len[(size_t)seq * p.seq_len_stride];
  if (L == 0 || L > p.max_ctx) {
    if (threadIdx.x == 0 && split == 0 && kvh == 0) raise_error(p.err, kDevBadArgument);
    return;
  }
  // Chunking: S = min(gridDim.x, ceil(L/64)) splits of a 16-multiple length
  // (at least one 16-position sub-tile per warp).
  const uint32_t max_s = gridDim.x;
  uint32_t S = (L + kMinSplitLen - 1) / kMinSplitLen;
  if (S > max_s) S = max_s;
  uint32_t chunk = (L + S - 1) / S;
  chunk = (chunk + kSub - 1) / kSub * kSub;
  const uint32_t S_eff = (L + chunk - 1) / chunk;
  if ((uint32_t)split >= S_eff) return;
  const uint32_t p0 = split * chunk;
  const uint32_t p1 = min(L, p0 + chunk);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const __half* kbase = p.k + (size_t)seq * p.kv_seq_stride + (size_t)kvh * p.kv_head_stride;
  const __half* vbase = p.v + (size_t)seq * p.kv_seq_stride + (size_t)kvh * p.kv_head_stride;

  // q fragments: lane (g,t) holds q[head 6*kvh + g][32t .. 32t+31] (zero for g >= 6).
  uint32_t qf[16];
  {
    const bool hv = g < 6;
    const uint4* qp = reinterpret_cast<const uint4*>(p.q + (size_t)seq * p.q_seq_stride +
                                                     (size_t)(6 * kvh + (hv ? g : 0)) * kHeadDim +
                                                     32 * t);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 v = hv ? qp[j] : make_uint4(0, 0, 0, 0);
      qf[4 * j + 0] = v.x;
      qf[4 * j + 1] = v.y;
      qf[4 * j + 2] = v.z;
      qf[4 * j + 3] = v.w;
    }
  }

  // Running state for heads 2t, 2t+1 (replicated over g).
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  for (uint32_t base = p0 + warp * kSub; base < p1; base += kAttnWarps * kSub) {
    // ---- stage V rows [base, base+16) into shared memory (zero past p1).
    {
      const int r = lane >> 1, half_sel = lane & 1;
      const uint32_t pos = base + r;
      uint8_t* dst = vs[warp] + r * kVRowBytes + half_sel * 128;
      if (pos < p1) {
        const uint4* src = reinterpret_cast<const uint4*>(vbase + (size_t)pos * p.kv_pos_stride) +
                           half_sel * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j) reinterpret_cast<uint4*>(dst)[j] = src[j];
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) reinterpret_cast<uint4*>(dst)[j] = make_uint4(0, 0, 0, 0);
      }
    }
    // ---- S^T = K q^T: lane reads K[pos g][32t..32t+31] and K[pos g+8][..].
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const uint32_t pg = base + g, pg8 = base + g + 8;
      uint32_t kg[16], kg8[16];
      const uint4* srcg = reinterpret_cast<const uint4*>(kbase + (size_t)min(pg, p1 - 1) * p.kv_pos_stride + 32 * t);
      const uint4* srcg8 = reinterpret_cast<const uint4*>(kbase + (size_t)min(pg8, p1 - 1) * p.kv_pos_stride + 32 * t);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 a = srcg[j], b = srcg8[j];
        kg[4 * j] = a.x; kg[4 * j + 1] = a.y; kg[4 * j + 2] = a.z; kg[4 * j + 3] = a.w;
        kg8[4 * j] = b.x; kg8[4 * j + 1] = b.y; kg8[4 * j + 2] = b.z; kg8[4 * j + 3] = b.w;
      }
#pragma unroll
      for (int st = 0; st < 8; ++st) {
        // mma-k (2t,2t+1) <-> d = 32t+4st, +1 ; (2t+8, 2t+9) <-> d = 32t+4st+2, +3
        const uint32_t a[4] = {kg[2 * st], kg8[2 * st], kg[2 * st + 1], kg8[2 * st + 1]};
        mma_16816(s, a, qf[2 * st], qf[2 * st + 1], s);
      }
      // s[0]: (pos g, head 2t)  s[1]: (pos g, head 2t+1)
      // s[2]: (pos g+8, head 2t) s[3]: (pos g+8, head 2t+1)
      const bool vg = pg < p1, vg8 = pg8 < p1;
#pragma unroll
      for (int j = 0; j < 4; ++j) s[j] *= kAttnScale;
      if (!vg) s[0] = s[1] = -INFINITY;
      if (!vg8) s[2] = s[3] = -INFINITY;
    }
    // ---- online softmax for heads 2t and 2t+1.
    float pr[4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float mx = fmaxf(s[hh], s[2 + hh]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float m_new = fmaxf(m_run[hh], mx);
      const float corr = m_run[hh] == -INFINITY ? 0.f : expf(m_run[hh] - m_new);
      const float e0 = expf(s[hh] - m_new), e1 = expf(s[2 + hh] - m_new);
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
    // ---- P^T to shared memory as fp16 hi/lo: pt[pos][head].
    {
      uint16_t* hi = pt[warp][0];
      uint16_t* lo = pt[warp][1];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int pos = g + (j >= 2 ? 8 : 0), head = 2 * t + (j & 1);
        const __half h = f2h(pr[j]);
        const __half l = f2h(pr[j] - h2f(h));
        hi[pos * 8 + head] = hbits(h);
        lo[pos * 8 + head] = hbits(l);
      }
    }
    __syncwarp();
    // B fragments (k = pos, n = head): lane (g,t): (pos 2t, 2t+1 ; head g), (pos 2t+8, 2t+9 ; head g)
    uint32_t bh0, bh1, bl0, bl1;
    {
      const uint16_t* hi = pt[warp][0];
      const uint16_t* lo = pt[warp][1];
      bh0 = (uint32_t)hi[(2 * t) * 8 + g] | ((uint32_t)hi[(2 * t + 1) * 8 + g] << 16);
      bh1 = (uint32_t)hi[(2 * t + 8) * 8 + g] | ((uint32_t)hi[(2 * t + 9) * 8 + g] << 16);
      bl0 = (uint32_t)lo[(2 * t) * 8 + g] | ((uint32_t)lo[(2 * t + 1) * 8 + g] << 16);
      bl1 = (uint32_t)lo[(2 * t + 8) * 8 + g] | ((uint32_t)lo[(2 * t + 9) * 8 + g] << 16);
    }
    // ---- o^T += V^T P^T over the 8 d-tiles.  A = V^T[16 d x 16 pos] via
    // ldmatrix.trans of V rows: matrices (pos 0-7, d 0-7), (pos 0-7, d 8-15),
    // (pos 8-15, d 0-7), (pos 8-15, d 8-15) -> a0..a3 after transposition
    // are (d g, pos 2t..), (d g+8, pos 2t..), (d g, pos 2t+8..), (d g+8, pos 2t+8..).
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int prow = ri + ((mi >> 1) << 3);   // position row of this address
      const int dcol = (mi & 1) << 3;           // d offset within the tile
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t a[4];
        ldmatrix_x4_trans(a, vs[warp] + prow * kVRowBytes + (16 * i + dcol) * 2);
        mma_16816(o[i], a, bh0, bh1, o[i]);
        mma_16816(o[i], a, bl0, bl1, o[i]);
      }
    }
    __syncwarp();
  }

  // ---- merge the 4 warps.  o[i][0]: (d 16i+g, head 2t) o[i][1]: (d 16i+g, head 2t+1)
  //                          o[i][2]: (d 16i+g+8, head 2t) o[i][3]: (d 16i+g+8, head 2t+1)
  if (g == 0) {
    wm[warp][2 * t] = m_run[0];
    wm[warp][2 * t + 1] = m_run[1];
    wl[warp][2 * t] = l_run[0];
    wl[warp][2 * t + 1] = l_run[1];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int head = 2 * t + (j & 1), d = 16 * i + g + (j >= 2 ? 8 : 0);
      if (head < 6) wo[warp][head][d] = o[i][j];
    }
  __syncthreads();

  const size_t unit = ((size_t)seq * kKVHeads + kvh);
  float* part_o = p.part_o + (unit * max_s + split) * (6 * kHeadDim);
  float* part_ml = p.part_ml + (unit * max_s + split) * 12;
  for (int idx = threadIdx.x; idx < 6 * kHeadDim; idx += blockDim.x) {
    const int head = idx / kHeadDim, d = idx % kHeadDim;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][head]);
    float Lsum = 0.f, O = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) {
      if (wm[w][head] == -INFINITY) continue;
      const float c = expf(wm[w][head] - M);
      Lsum += wl[w][head] * c;
      O += wo[w][head][d] * c;
    }
    if (S_eff == 1) {
      store_out(p, seq, (6 * kvh + head) * kHeadDim + d, O / Lsum);
    } else {
      part_o[idx] = O;
      if (d == 0) {
        part_ml[2 * head] = M;
        part_ml[2 * head + 1] = Lsum;
      }
    }
  }
  if (S_eff == 1) return;

  // ---- ticket: the last CTA of this (seq, kv head) merges all chunks in order.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_ticket = atomicAdd(&p.counters[unit], 1u);
  __syncthreads();
  if (s_ticket != S_eff - 1) return;
  __threadfence();
  const float* all_o = p.part_o + unit * max_s * (6 * kHeadDim);
  const float* all_ml = p.part_ml + unit * max_s * 12;
  // Per head: the maximum over splits, each split's rescale factor and the
  // total weight, staged once in shared memory (wo/wm are free by now).
  float* sc = &wo[0][0][0];             // [S_eff][6] factors
  float* hsum = &wo[1][0][0];           // [6] totals
  if (threadIdx.x < 6) {
    const int head = threadIdx.x;
    float M = -INFINITY;
    for (uint32_t sp = 0; sp < S_eff; ++sp) M = fmaxf(M, __ldcg(all_ml + sp * 12 + 2 * head));
    float Lsum = 0.f;
    for (uint32_t sp = 0; sp < S_eff; ++sp) {
      const float m = __ldcg(all_ml + sp * 12 + 2 * head);
      const float c = m == -INFINITY ? 0.f : expf(m - M);
      sc[sp * 6 + head] = c;
      Lsum += __ldcg(all_ml + sp * 12 + 2 * head + 1) * c;
    }
    hsum[head] = Lsum;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 6 * kHeadDim; idx += blockDim.x) {
    const int head = idx / kHeadDim;
    float part[kMaxSplits];
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; ++sp)
      part[sp] = (uint32_t)sp < S_eff ? __ldcg(all_o + sp * (6 * kHeadDim) + idx) : 0.f;
    float O = 0.f;
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; ++sp)
      if ((uint32_t)sp < S_eff) O += part[sp] * sc[sp * 6 + head];
    store_out(p, seq, (6 * kvh) * kHeadDim + idx, O / hsum[head]);
  }
  if (threadIdx.x == 0) p.counters[unit] = 0;  // re-arm for the next launch
}

// Splits for a launch: enough CTAs for ~8 per SM over the batch, at least 64
// positions per split, at most 32 splits (the merge reads them all).
int attn_max_splits(int max_ctx, int n_seq) {
  int s = (max_ctx + kMinSplitLen - 1) / kMinSplitLen;
  const int target = kAttnCtaTarget / (kKVHeads * (n_seq > 0 ? n_seq : 1));
  const int cap = target < 1 ? 1 : (target > kMaxSplits ? kMaxSplits : target);
  return s < cap ? s : cap;
}

// Scratch layout: the merge tickets first, at a fixed offset, so that calls
// with different split counts find them where the last call left them (zero);
// then the per-split (m, l) pairs and the per-split partial outputs.
static size_t attn_ticket_bytes(int n_seq) {
  return ((size_t)n_seq * kKVHeads * sizeof(uint32_t) + 255) / 256 * 256;
}

size_t attn_scratch_bytes(int max_splits, int n_seq) {
  const size_t units = (size_t)n_seq * kKVHeads;
  return attn_ticket_bytes(n_seq) + units * max_splits * (6 * kHeadDim + 12) * sizeof(float);
}

void attn_bind_scratch(AttnParams& p, void* scratch, int max_splits, int n_seq) {
  const size_t units = (size_t)n_seq * kKVHeads;
  uint8_t* base = reinterpret_cast<uint8_t*>(scratch);
  p.counters = reinterpret_cast<uint32_t*>(base);
  p.part_ml = reinterpret_cast<float*>(base + attn_ticket_bytes(n_seq));
  p.part_o = p.part_ml + units * max_splits * 12;
}

void launch_attention_decode(const AttnParams& p, int max_splits, int n_seq, cudaStream_t st,
                             bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(max_splits, kKVHeads, n_seq);
  cfg.blockDim = dim3(128);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, k_attention_decode, p);
}

}  // namespace qwen
