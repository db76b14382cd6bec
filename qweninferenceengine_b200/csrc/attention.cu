// attention.cu -- split-K GQA decode attention (flash-decoding) for 12 query
// heads over 2 KV heads, head_dim 128, FP16 KV cache, any number of sequences.
//
// Replaces attention_scores -> softmax -> attn_weighted_sum
// (attention.metal:9-56, activations.metal:29-55; InferenceEngine.swift:162-182):
//   s_t = 0.088388 * q_h . K_t,   p_t = exp(s_t - max) / sum,   o_h = sum_t p_t V_t
// evaluated as an online softmax over position chunks.
//
// Persistent grid (one CTA per SM) over work units = (sequence, kv head,
// split): a split is a run of 128-position tiles of one sequence and one kv
// head (query heads 6h .. 6h+5).  The batch's sequences times the two kv heads
// usually fill the machine with one split each, and a unit then holds a whole
// head: no merge across CTAs.
//   warp 8      producer: per tile, one lane issues 4 TMA tile loads from 2-D
//               tensor maps over the K and V caches (rows = positions, 256
//               fp16 per row): the unit's head's two 64-element halves, boxes
//               of 128 positions x 64 elements with the 128-byte swizzle, so
//               the K fragment loads and the V ldmatrix.trans reads hit
//               distinct banks; a 3-stage ring (192 KB in flight per SM);
//               the ring runs on across units, so loads of the next unit
//               overlap the merge of this one
//   warps 0..7  warp w takes positions 16w .. 16w+15 of every tile:
//                 S^T[16 pos x 8 heads] = K[16 x 128] . q^T   (8 m16n8k16 MMAs)
//                 o^T[128 x 8]        += V^T[128 x 16] . P^T  (V by
//                     ldmatrix.trans; P split into fp16 hi + lo parts so the
//                     product keeps ~22 bits)
// The 8 warps merge in shared memory; where a head has several splits they
// merge in a fixed order by the last CTA of the (sequence, head) to finish (an
// atomic ticket -- nothing waits), so results do not depend on scheduling.
// Waits are bounded (2 s).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "qwen_common.cuh"
#include "qwen_internal.h"

namespace qwen {

namespace {

constexpr int kTilePos = 128;                       // positions per ring stage
constexpr int kSub = 16;                            // positions per warp sub-tile
constexpr int kConsumerWarps = 8;
constexpr int kAttnThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 3;
constexpr int kBoxBytes = kTilePos * 128;          // 128 positions x 64 fp16, swizzled
constexpr int kBoxes = 2;                           // the unit's head: 2 x 64 fp16 per position
static_assert(kConsumerWarps * kSub == kTilePos, "a tile is one sub-tile per consumer warp");
constexpr int kMaxSplits = 32;                      // bounds the merge of a sequence
constexpr int kUnitsPerSm = 1;                      // work units per SM to aim for (each costs a merge)
constexpr unsigned long long kAttnWaitNs = 2000000000ull;

struct AttnSmem {
  uint8_t k[kStages][kBoxes][kBoxBytes];            // 1024-byte aligned (swizzle atoms)
  uint8_t v[kStages][kBoxes][kBoxBytes];
  uint16_t pt[kConsumerWarps][2][kSub * 8];        // P^T hi/lo, [pos][head]
  float wm[kConsumerWarps][8], wl[kConsumerWarps][8];
  float wo[kConsumerWarps][6][kHeadDim];
  float sc[2][kMaxSplits][8];                      // split merge factors [head group][split][head]
  float hsum[2][8];
  uint64_t full[kStages], empty[kStages];
  uint32_t ticket;
  int abort;
  int unit_abort;   // abort as seen by the merge of the running unit (uniform)
};

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
// 2-D TMA tile load (box of the tensor map at element x, row y) into shared
// memory, completion as transaction bytes on bar.  x is a multiple of 64
// elements (128 B).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], "
      "[%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// Byte offset of 16-byte chunk `chunk` of row `row` in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)row * 128u + ((uint32_t)(chunk ^ (row & 7)) << 4);
}
// Barrier of the 8 consumer warps (the producer warp does not take part).
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded parity wait; on timeout records kDevWaitTimeout and sets abort.
__device__ bool attn_wait(uint64_t* bar, uint32_t parity, AttnSmem& s, int* err,
                          bool honour_abort = true) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = gtime();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (honour_abort && *((volatile int*)&s.abort)) return false;
      if (gtime() - t0 > kAttnWaitNs) {
        *((volatile int*)&s.abort) = 1;
        raise_error(err, kDevWaitTimeout);
        return false;
      }
    }
  }
}

// Output element (seq, col): row-major out, or the activation tile layout
// ([col/64][row][128 B], 16-byte chunk j of row r at (j ^ (r & 7))).
__device__ __forceinline__ void store_out(const AttnParams& p, int seq, int col, float v) {
  if (p.act_out) {
    const int c = col >> 6, j = (col >> 3) & 7;
    const size_t off = ((size_t)c * p.act_nb + seq) * 128 +
                       (((uint32_t)j ^ (uint32_t)(seq & 7)) << 4) + (col & 7) * 2;
    *reinterpret_cast<__half*>(p.act_out + off) = f2h(v);
  } else {
    p.out[(size_t)seq * p.out_seq_stride + col] = f2h(v);
  }
}

struct Unit {
  int seq, kvh, split;
  uint32_t p0, p1, s_eff;
};

// q of the unit's six query heads (qs, 6 x 128) and the step's new k | v rows
// of its kv head (kvn: 128 k, then 128 v) of sequence `seq` from the QKV
// partials, as the batched QKV finish forms them: sum of the splits in split
// order, + bias, rounded to fp16, RoPE on the q / k heads at position pos
// (rope.metal:12-39), the v row rounded after the bias.  256 consumer threads:
// RoPE pairs ctid and ctid + 256 (pairs 0..383 the q heads, 384..447 the k
// head), v element ctid < 128; every split's loads issued together.
__device__ __forceinline__ void form_qkv(const AttnParams& p, int seq, int kvh, uint32_t pos,
                                         __half* qs, __half* kvn, int ctid) {
  constexpr int kQPairs = 6 * 64, kPairs = kQPairs + 64;   // 448
  constexpr int kJobs = (kPairs + 255) / 256;               // 2
  const size_t stride = (size_t)p.qkv_rows * kQKVRows;
  const float* part = p.qkv_part + (size_t)seq * kQKVRows;
  const float* cs = p.rope_cs + (size_t)pos * 128;
  int i1[kJobs];
  float s1[kJobs], s2[kJobs];
  __half b1[kJobs], b2[kJobs];
  float2 rot[kJobs];   // (cos, sin) of the pair
#pragma unroll
  for (int j = 0; j < kJobs; ++j) {   // biases and RoPE factors loaded with the partials
    const int pr = ctid + 256 * j;
    const int pc = pr < kPairs ? pr : 0;
    i1[j] = pc < kQPairs ? (6 * kvh + (pc >> 6)) * 128 + (pc & 63)
                         : kHidden + kvh * 128 + (pc - kQPairs);
    s1[j] = s2[j] = 0.f;
    b1[j] = p.qkv_bias[i1[j]];
    b2[j] = p.qkv_bias[i1[j] + 64];
    rot[j] = reinterpret_cast<const float2*>(cs)[pc & 63];
  }
  const int iv = kHidden + kKVDim + kvh * 128 + (ctid & 127);   // v element (ctid < 128)
  const __half bvh = p.qkv_bias[iv];
  float sv = 0.f;
#pragma unroll 4
  for (int sp = 0; sp < p.qkv_splits; ++sp) {
    const float* ps = part + (size_t)sp * stride;
    float a[kJobs], b[kJobs];
#pragma unroll
    for (int j = 0; j < kJobs; ++j) {
      a[j] = __ldcg(ps + i1[j]);
      b[j] = __ldcg(ps + i1[j] + 64);
    }
    const float c = __ldcg(ps + iv);
#pragma unroll
    for (int j = 0; j < kJobs; ++j) {
      s1[j] += a[j];
      s2[j] += b[j];
    }
    sv += c;
  }
#pragma unroll
  for (int j = 0; j < kJobs; ++j) {
    const int pr = ctid + 256 * j;
    if (pr >= kPairs) break;
    const float x1 = h2f(f2h(s1[j] + h2f(b1[j])));
    const float x2 = h2f(f2h(s2[j] + h2f(b2[j])));
    const float c = rot[j].x, sn = rot[j].y;
    const __half r1 = f2h(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn)));
    const __half r2 = f2h(__fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, c)));
    __half* dst = pr < kQPairs ? qs + (pr >> 6) * 128 + (pr & 63) : kvn + (pr - kQPairs);
    dst[0] = r1;
    dst[64] = r2;
  }
  if (ctid < 128) kvn[128 + ctid] = f2h(sv + h2f(bvh));
}
// Unit u = (sequence u / (2 max_s), kv head (u / max_s) % 2, split u % max_s):
// n_tiles = ceil(L/128) tiles in S = min(max_s, n_tiles) near-equal runs;
// false if the split is empty.
__device__ __forceinline__ bool unit_of(const AttnParams& p, int u, int max_s, Unit& w) {
  w.seq = u / (2 * max_s);
  w.kvh = (u / max_s) & 1;
  w.split = u % max_s;
  const uint32_t L = p.seq_len[(size_t)w.seq * p.seq_len_stride];
  if (L == 0 || L > p.max_ctx) return false;
  const uint32_t n_tiles = (L + kTilePos - 1) / kTilePos;
  const uint32_t S = n_tiles < (uint32_t)max_s ? n_tiles : (uint32_t)max_s;
  const uint32_t tps = (n_tiles + S - 1) / S;
  w.s_eff = (n_tiles + tps - 1) / tps;
  if ((uint32_t)w.split >= w.s_eff) return false;
  w.p0 = (uint32_t)w.split * tps * kTilePos;
  w.p1 = min(L, w.p0 + tps * kTilePos);
  return true;
}

}  // namespace

// kFusedQkv: q and the new k / v rows formed from the QKV partials
// (AttnParams::qkv_part set, the batched decode step); each launch runs the
// instantiation of its mode, without the other's code.
template <bool kFusedQkv>
__global__ void __launch_bounds__(kAttnThreads, 1)
    k_attention_decode(AttnParams p, int max_s, int n_units, int rows_per_seq,
                       const __grid_constant__ CUtensorMap tmk,
                       const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ uint8_t attn_smem_raw[];
  AttnSmem& s = *reinterpret_cast<AttnSmem*>(
      attn_smem_raw + ((1024u - (smem_u32(attn_smem_raw) & 1023u)) & 1023u));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kConsumerWarps);
    }
    s.abort = 0;
    fence_mbar_init();
  }
  // As a programmatic dependent: let the next kernel launch, then wait for the
  // previous one (no-ops in a plain launch).
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer --
    uint32_t it = 0;
    if (lane == 0) {
      for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        Unit w;
        if (!unit_of(p, u, max_s, w)) continue;
        const int row0 = (p.row_seq ? p.row_seq[w.seq] : w.seq) * rows_per_seq;
        for (uint32_t base = w.p0; base < w.p1; base += kTilePos, ++it) {
          const int st = it % kStages;
          if (it >= kStages && !attn_wait(&s.empty[st], ((it / kStages) - 1) & 1, s, p.err))
            continue;  // aborting: keep the tile count, issue nothing
          mbar_arrive_expect_tx(&s.full[st], 2 * kBoxes * kBoxBytes);
#pragma unroll
          for (int b = 0; b < kBoxes; ++b) {   // the unit's head: elements 128 kvh + 64 b ..
            tma_load_2d(s.k[st][b], &tmk, kHeadDim * w.kvh + 64 * b, row0 + (int)base, &s.full[st]);
            tma_load_2d(s.v[st][b], &tmv, kHeadDim * w.kvh + 64 * b, row0 + (int)base, &s.full[st]);
          }
        }
      }
      // Every issued copy lands before the CTA may exit.
      for (uint32_t j = it > kStages ? it - kStages : 0; j < it; ++j)
        attn_wait(&s.full[j % kStages], (j / kStages) & 1, s, p.err, false);
    }
    __syncwarp();
    return;
  }

  // -------------------------------------------------------------- consumers --
  const int slice = warp;                        // 16-row slice of a tile
  const int g = lane >> 2, t = lane & 3;
  const int ctid = threadIdx.x;                  // 0..255
  uint32_t it = 0;
  for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
    Unit w;
    if (!unit_of(p, u, max_s, w)) {
      if (ctid == 0 && u % (2 * max_s) == 0) {
        const uint32_t L = p.seq_len[(size_t)(u / (2 * max_s)) * p.seq_len_stride];
        if (L == 0 || L > p.max_ctx) raise_error(p.err, kDevBadArgument);
      }
      continue;
    }
    const int h = w.kvh;
    // q (and in a decode step's fused mode the new k / v rows) in shared
    // memory of the merge: q in wo (read into registers before the first tile;
    // the merge writes wo after the last), the rows in sc (used by the last
    // tile's patch; sc is written only after the merge's barriers).
    const uint32_t pos = p.seq_len[(size_t)w.seq * p.seq_len_stride] - 1;
    __half* qs = reinterpret_cast<__half*>(&s.wo[0][0][0]);
    __half* kvn = reinterpret_cast<__half*>(&s.sc[0][0][0]);
    static_assert(sizeof(s.sc) >= 2 * kHeadDim * sizeof(__half), "new k / v rows exceed sc");
    static_assert(sizeof(s.wo) >= 6 * kHeadDim * sizeof(__half), "q exceeds wo");
    constexpr bool fused_qkv = kFusedQkv;
    const bool owns_pos = fused_qkv && pos >= w.p0 && pos < w.p1;
    if (fused_qkv) {
      form_qkv(p, w.seq, h, pos, qs, kvn, ctid);
      consumers_sync();
      if (owns_pos && ctid < 32) {
        // this head's new rows into the caches, for the steps after this one
        const int kvs = p.row_seq ? p.row_seq[w.seq] : w.seq;
        const size_t off = (size_t)kvs * p.kv_seq_stride + (size_t)pos * p.kv_pos_stride +
                           (size_t)h * p.kv_head_stride;
        __half* dst = const_cast<__half*>(ctid < 16 ? p.k : p.v) + off;
        reinterpret_cast<uint4*>(dst)[ctid & 15] = reinterpret_cast<const uint4*>(kvn)[ctid];
      }
    }
    // q fragments: lane (g,t) holds q[head 6h + g][32t .. 32t+31] (zero for g >= 6).
    uint32_t qf[16];
    {
      const bool hv = g < 6;
      const uint4* qp = reinterpret_cast<const uint4*>(
          (fused_qkv ? qs + (size_t)(hv ? g : 0) * kHeadDim
                     : p.q + (size_t)w.seq * p.q_seq_stride + (size_t)(6 * h + (hv ? g : 0)) * kHeadDim) +
          32 * t);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 v = hv ? qp[j] : make_uint4(0, 0, 0, 0);
        qf[4 * j + 0] = v.x;
        qf[4 * j + 1] = v.y;
        qf[4 * j + 2] = v.z;
        qf[4 * j + 3] = v.w;
      }
    }
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    for (uint32_t tb = w.p0; tb < w.p1; tb += kTilePos, ++it) {
      const int st = it % kStages;
      bool ok = true;
      if (lane == 0) ok = attn_wait(&s.full[st], (it / kStages) & 1, s, p.err);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      const uint32_t base = tb + 16 * slice;
      const int r0 = 16 * slice;  // first row of this warp in the boxes
      bool zeroed = false;
      if (ok && owns_pos && pos >= base && pos < base + 16) {
        // The new position's k / v rows of this warp's head into the stage
        // (the cache may not hold them yet): lane -> (k|v, 64-element box,
        // 16-byte chunk), swizzled as the tensor map lays the box out.
        const int r = (int)(pos - tb), kv = lane >> 4, half = (lane >> 3) & 1, ch = lane & 7;
        uint8_t* box = kv ? s.v[st][half] : s.k[st][half];
        *reinterpret_cast<uint4*>(box + swz(r, ch)) =
            *reinterpret_cast<const uint4*>(kvn + kv * kHeadDim + half * 64 + ch * 8);
        zeroed = true;   // generic stores into the stage: proxy fence before its release
        __syncwarp();
      }
      if (ok && base < w.p1) {
        // ---- S^T = K q^T: lane reads K[row g][32t..32t+31] and K[row g+8][..].
        float sv[4] = {0.f, 0.f, 0.f, 0.f};
        {
          uint32_t kg[16], kg8[16];
          // d = 32t + 8j: box t/2, chunk 4(t&1) + j of rows r0+g, r0+g+8.
          const uint8_t* kbox = s.k[st][t >> 1];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 a = *reinterpret_cast<const uint4*>(kbox + swz(r0 + g, 4 * (t & 1) + j));
            const uint4 b = *reinterpret_cast<const uint4*>(kbox + swz(r0 + g + 8, 4 * (t & 1) + j));
            kg[4 * j] = a.x; kg[4 * j + 1] = a.y; kg[4 * j + 2] = a.z; kg[4 * j + 3] = a.w;
            kg8[4 * j] = b.x; kg8[4 * j + 1] = b.y; kg8[4 * j + 2] = b.z; kg8[4 * j + 3] = b.w;
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            // mma-k (2t,2t+1) <-> d = 32t+4q, +1 ; (2t+8, 2t+9) <-> d = 32t+4q+2, +3
            const uint32_t a[4] = {kg[2 * q], kg8[2 * q], kg[2 * q + 1], kg8[2 * q + 1]};
            mma_16816(sv, a, qf[2 * q], qf[2 * q + 1], sv);
          }
          // sv[0]: (pos g, head 2t) sv[1]: (pos g, head 2t+1)
          // sv[2]: (pos g+8, head 2t) sv[3]: (pos g+8, head 2t+1)
#pragma unroll
          for (int j = 0; j < 4; ++j) sv[j] *= kAttnScale;
          if (base + g >= w.p1) sv[0] = sv[1] = -INFINITY;
          if (base + g + 8 >= w.p1) sv[2] = sv[3] = -INFINITY;
        }
        // ---- online softmax for heads 2t and 2t+1.
        float pr[4];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float mx = fmaxf(sv[hh], sv[2 + hh]);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float m_new = fmaxf(m_run[hh], mx);
          const float corr = m_run[hh] == -INFINITY ? 0.f : expf(m_run[hh] - m_new);
          const float e0 = expf(sv[hh] - m_new), e1 = expf(sv[2 + hh] - m_new);
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
          uint16_t* hi = s.pt[warp][0];
          uint16_t* lo = s.pt[warp][1];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int pos = g + (j >= 2 ? 8 : 0), head = 2 * t + (j & 1);
            const __half hv = f2h(pr[j]);
            const __half lv = f2h(pr[j] - h2f(hv));
            hi[pos * 8 + head] = hbits(hv);
            lo[pos * 8 + head] = hbits(lv);
          }
        }
        // Rows past the end hold stale data: zero this head's half (P is 0
        // there, but 0 * NaN would not be).
        if (base + 16 > w.p1) {
          for (int r = (int)(w.p1 - base); r < 16; ++r)
            if (lane < 16)  // both boxes of this head, whole 128-byte rows
              *reinterpret_cast<uint4*>(s.v[st][lane >> 3] + (r0 + r) * 128 +
                                        (lane & 7) * 16) = make_uint4(0, 0, 0, 0);
          zeroed = true;
        }
        __syncwarp();
        // B fragments (k = pos, n = head): lane (g,t): (pos 2t, 2t+1 ; head g), (pos 2t+8, 2t+9 ; head g)
        uint32_t bh0, bh1, bl0, bl1;
        {
          const uint16_t* hi = s.pt[warp][0];
          const uint16_t* lo = s.pt[warp][1];
          bh0 = (uint32_t)hi[(2 * t) * 8 + g] | ((uint32_t)hi[(2 * t + 1) * 8 + g] << 16);
          bh1 = (uint32_t)hi[(2 * t + 8) * 8 + g] | ((uint32_t)hi[(2 * t + 9) * 8 + g] << 16);
          bl0 = (uint32_t)lo[(2 * t) * 8 + g] | ((uint32_t)lo[(2 * t + 1) * 8 + g] << 16);
          bl1 = (uint32_t)lo[(2 * t + 8) * 8 + g] | ((uint32_t)lo[(2 * t + 9) * 8 + g] << 16);
        }
        // ---- o^T += V^T P^T over the 8 d-tiles: A = V^T[16 d x 16 pos] by
        // ldmatrix.trans of V rows: matrices (pos 0-7, d 0-7), (pos 0-7, d 8-15),
        // (pos 8-15, d 0-7), (pos 8-15, d 8-15).
        {
          const int mi = lane >> 3, ri = lane & 7;
          const int prow = ri + ((mi >> 1) << 3);
          const int dcol = (mi & 1) << 3;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            // d = 16i + dcol: box 2h + i/4, chunk 2(i&3) + dcol/8.
            uint32_t a[4];
            ldmatrix_x4_trans(a, s.v[st][i >> 2] + swz(r0 + prow, 2 * (i & 3) + (dcol >> 3)));
            mma_16816(o[i], a, bh0, bh1, o[i]);
            mma_16816(o[i], a, bl0, bl1, o[i]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        if (zeroed) fence_proxy_async();  // generic stores before the next TMA write
        mbar_arrive(&s.empty[st]);
      }
    }

    // ---- merge the 8 warps (all on the unit's head group).  o[i][0]: (d 16i+g, head 2t)
    // o[i][1]: (d 16i+g, head 2t+1) o[i][2]: (d 16i+g+8, head 2t) o[i][3]: (d 16i+g+8, head 2t+1)
    if (g == 0) {
      s.wm[warp][2 * t] = m_run[0];
      s.wm[warp][2 * t + 1] = m_run[1];
      s.wl[warp][2 * t] = l_run[0];
      s.wl[warp][2 * t + 1] = l_run[1];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int head = 2 * t + (j & 1), d = 16 * i + g + (j >= 2 ? 8 : 0);
        if (head < 6) s.wo[warp][head][d] = o[i][j];
      }
    // One snapshot of the abort flag, so every consumer thread takes the same
    // barriers below.
    if (ctid == 0) s.unit_abort = *((volatile int*)&s.abort);
    consumers_sync();
    const bool aborting = s.unit_abort != 0;
    // partials of split (seq, split) of head group h at [seq][split][h]
    const size_t pidx = ((size_t)w.seq * max_s + w.split) * 2 + h;
    float* part_o = p.part_o + pidx * (6 * kHeadDim);
    float* part_ml = p.part_ml + pidx * 12;
    for (int idx = ctid; idx < 6 * kHeadDim && !aborting; idx += 256) {
      const int head = idx / kHeadDim, d = idx % kHeadDim;
      float M = -INFINITY;
#pragma unroll
      for (int ww = 0; ww < kConsumerWarps; ++ww) M = fmaxf(M, s.wm[ww][head]);
      float Lsum = 0.f, O = 0.f;
#pragma unroll
      for (int ww = 0; ww < kConsumerWarps; ++ww) {
        const float m = s.wm[ww][head];
        if (m == -INFINITY) continue;
        const float c = expf(m - M);
        Lsum += s.wl[ww][head] * c;
        O += s.wo[ww][head][d] * c;
      }
      if (w.s_eff == 1) {
        store_out(p, w.seq, (6 * h + head) * kHeadDim + d, O / Lsum);
      } else {
        part_o[idx] = O;
        if (d == 0) {
          part_ml[2 * head] = M;
          part_ml[2 * head + 1] = Lsum;
        }
      }
    }
    if (w.s_eff > 1 && !aborting) {
      // ---- ticket: the last CTA of this (sequence, head) merges its splits
      // in order.
      __threadfence();
      consumers_sync();
      if (ctid == 0) s.ticket = atomicAdd(&p.counters[w.seq * 2 + h], 1u);
      consumers_sync();
      if (s.ticket == w.s_eff - 1) {
        __threadfence();
        const float* all_ml = p.part_ml + (size_t)w.seq * max_s * 2 * 12;
        const float* all_o = p.part_o + (size_t)w.seq * max_s * 2 * (6 * kHeadDim);
        if (warp == 0) {  // lane = split
          const int hg = h;
          const bool have = (uint32_t)lane < w.s_eff;
          // the split's 6 (m, l) pairs in one go (48 bytes, 16-byte aligned)
          float ml[12];
#pragma unroll
          for (int q = 0; q < 3; ++q) {
            const float4 v = have ? __ldcg(reinterpret_cast<const float4*>(
                                        all_ml + ((size_t)lane * 2 + hg) * 12) + q)
                                  : make_float4(-INFINITY, 0.f, -INFINITY, 0.f);
            ml[4 * q] = v.x;
            ml[4 * q + 1] = v.y;
            ml[4 * q + 2] = v.z;
            ml[4 * q + 3] = v.w;
          }
#pragma unroll
          for (int head = 0; head < 6; ++head) {
            const float m = ml[2 * head];
            const float l = ml[2 * head + 1];
            float M = m;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
            const float c = m == -INFINITY ? 0.f : expf(m - M);
            s.sc[0][lane][head] = c;
            // fixed-order tree sum over splits (lane order) for determinism
            float L = l * c;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
              const float o2 = __shfl_down_sync(0xffffffffu, L, off);
              if ((lane & (2 * off - 1)) == 0) L += o2;
            }
            if (lane == 0) s.hsum[0][head] = L;
          }
        }
        consumers_sync();
        {
          // The thread's three outputs (idx = ctid + 256 j), summed over the
          // splits in split order; each split's partials are loaded together,
          // so the merge waits one L2 round trip per split rather than one per
          // output.
          constexpr int kPer = 6 * kHeadDim / 256;
          static_assert(kPer * 256 == 6 * kHeadDim, "merge outputs per thread");
          float O[kPer];
#pragma unroll
          for (int j = 0; j < kPer; ++j) O[j] = 0.f;
#pragma unroll 2
          for (uint32_t sp = 0; sp < w.s_eff; ++sp) {
            float v[kPer];
#pragma unroll
            for (int j = 0; j < kPer; ++j)
              v[j] = __ldcg(all_o + ((size_t)sp * 2 + h) * (6 * kHeadDim) + ctid + 256 * j);
#pragma unroll
            for (int j = 0; j < kPer; ++j) O[j] += v[j] * s.sc[0][sp][(ctid + 256 * j) / kHeadDim];
          }
#pragma unroll
          for (int j = 0; j < kPer; ++j) {
            const int r = ctid + 256 * j;
            store_out(p, w.seq, 6 * h * kHeadDim + r, O[j] / s.hsum[0][r / kHeadDim]);
          }
        }
        if (ctid == 0) p.counters[w.seq * 2 + h] = 0;  // re-arm for the next launch
      }
    }
    consumers_sync();  // wo / wm / sc are reused by the next unit
  }
}

// Splits per (sequence, kv head) for a launch: ~1 work unit per SM over the
// batch's 2 n_seq heads, at most one per 128-position tile, at most 32 (the
// merge reads them all).
int attn_max_splits(int max_ctx, int n_seq) {
  const int tiles = (max_ctx + kTilePos - 1) / kTilePos;
  int target = (148 * kUnitsPerSm) / (2 * (n_seq > 0 ? n_seq : 1));   // units per (sequence, kv head)
  if (target < 1) target = 1;
  const int s = tiles < target ? tiles : target;
  return s < kMaxSplits ? s : kMaxSplits;
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

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// rows x 256 fp16 (512-byte rows), boxes of 128 rows x 64 elements, 128-byte
// swizzle, zero fill past the last row.
bool encode_kv_map(CUtensorMap* map, const __half* base, uint64_t rows) {
  auto enc = tensor_map_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)kKVDim, rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kKVDim * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kTilePos};
  const cuuint32_t elem[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box,
             elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int launch_attention_decode(const AttnParams& p, int max_splits, int n_seq, cudaStream_t st,
                            bool pdl) {
  // The tensor maps see each cache as rows of 256 fp16 (both kv heads of a position).
  if (p.kv_pos_stride != kKVDim || p.kv_head_stride != kHeadDim || p.kv_seq_stride % kKVDim ||
      max_splits < 1 || max_splits > kMaxSplits || n_seq < 1 || p.max_ctx < 1)
    return -1;
  const int rows_per_seq = (int)(p.kv_seq_stride / kKVDim);
  const int kv_seqs = p.kv_n_seq > 0 ? p.kv_n_seq : n_seq;
  if (kv_seqs > 1 && rows_per_seq < (int)p.max_ctx) return -1;
  const uint64_t rows = (uint64_t)(kv_seqs - 1) * rows_per_seq + p.max_ctx;
  CUtensorMap tmk, tmv;
  if (!encode_kv_map(&tmk, p.k, rows) || !encode_kv_map(&tmv, p.v, rows)) return -1;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return -1;
  const int n_units = n_seq * kKVHeads * max_splits;
  const size_t smem = sizeof(AttnSmem) + 1024;
  void (*kern)(AttnParams, int, int, int, const CUtensorMap, const CUtensorMap) =
      p.qkv_part ? k_attention_decode<true> : k_attention_decode<false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_units < sms ? n_units : sms);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p, max_splits, n_units, rows_per_seq, tmk,
                            tmv) == cudaSuccess
             ? 0
             : -1;
}

}  // namespace qwen
