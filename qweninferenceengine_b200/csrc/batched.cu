// batched.cu -- the decode step for a batch of independent sequences on the
// tcgen05 tensor cores (QWEN_KERNELS_TC): the reference's forward
// (InferenceEngine.swift:54-271) for every sequence at once, each projection
// one tensor-core GEMM over all sequences (tc_gemm.cu), attention per
// sequence with its own length (attention.cu), fp16 rounding points as in
// the reference.
//
// Per layer (B sequences, nb = B padded to 16 activation rows):
//   act_h <- rmsnorm(x)                     (previous layer's finish kernel)
//   part  <- W_qkv . act_h                  tensor cores, K split
//   q, K/V cache <- rope(half(part + b))    k_qkv_finish (rope.metal:12-39,
//                                           attention.metal:67-84)
//   act_h <- attention(q, cache)            split-K GQA decode attention, written
//                                           straight into the activation tiles
//   part  <- W_o . act_h
//   x     <- half(x + half(part + b_o)); act_h <- rmsnorm(x)   k_resid_norm_finish
//   act_i <- half(silu(g) * u)              W_gu . act_h, tiles of 64 gate + 64 up
//                                           rows, SwiGLU in the GEMM epilogue
//                                           (activations.metal:9-27)
//   part  <- W_down . act_i
//   x     <- half(x + half(part + b_down)); act_h <- rmsnorm_next(x)
// then logits = LM . act_h (fp16 out, no split).
#include <cooperative_groups.h>

#include <cmath>
#include <vector>

#include "engine.h"
#include "qwen_common.cuh"
#include "status.h"
#include "tc_gemm.h"

namespace qwen {

namespace {

constexpr int kQKVTiles = kQKVRows / kTcM;          // 16
constexpr int kOTiles = kHidden / kTcM;             // 12
constexpr int kGUTiles = 2 * kInter / kTcM;         // 140
constexpr int kDownTiles = kHidden / kTcM;          // 12
constexpr int kChunks1536 = kHidden / kTcChunkK;    // 24
constexpr int kChunks8960 = kInter / kTcChunkK;     // 140
constexpr size_t kTcQKVBytes = (size_t)kQKVTiles * kChunks1536 * kQ4TcChunkBytes;
constexpr size_t kTcOBytes = (size_t)kOTiles * kChunks1536 * kQ4TcChunkBytes;
constexpr size_t kTcGUBytes = (size_t)kGUTiles * kChunks1536 * kQ4TcChunkBytes;
constexpr size_t kTcDownBytes = (size_t)kDownTiles * kChunks8960 * kQ4TcChunkBytes;
constexpr size_t kTcLayerBytes = kTcQKVBytes + kTcOBytes + kTcGUBytes + kTcDownBytes;

// Byte offset of element i of activation row b in the tile layout of nb rows.
__device__ __forceinline__ size_t act_off(int b, int i, int nb) {
  const int c = i >> 6, j = (i >> 3) & 7;
  return ((size_t)c * nb + b) * 128 + (((uint32_t)j ^ (uint32_t)(b & 7)) << 4) + (i & 7) * 2;
}

// Programmatic dependent launch: let the next kernel of the step launch (its
// prologue overlaps this kernel), then wait until the previous kernel has
// completed and its writes are visible.
__device__ __forceinline__ void pdl_prologue() {
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();
}

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...), "launch");
}

// Same, launched as clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, unsigned cluster_x,
                       cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...), "launch");
}

constexpr int kTcMaxSplits = 24;  // split counts the plan may pick (checked on the host)

// 1/sqrt(mean(x^2) + eps) of one 1536 row held by NT threads, PER values each
// (rmsnorm.metal:9-46; fp32 sum of squares).
template <int NT, int PER>
__device__ __forceinline__ float rms_scale_row(const float (&vals)[PER], float* red) {
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) acc += vals[j] * vals[j];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) tot += red[w];
  return 1.0f / sqrtf(tot / 1536.0f + kRmsEps);
}

// act row b <- half(half(x * s) * gamma).
__global__ void __launch_bounds__(512) k_rms_to_act(const __half* __restrict__ x,
                                                    const __half* __restrict__ gamma,
                                                    uint8_t* __restrict__ act, int nb) {
  pdl_prologue();
  __shared__ float red[16];
  const int b = blockIdx.x;
  const __half* xr = x + (size_t)b * kHidden;
  float v[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) v[j] = h2f(xr[threadIdx.x + 512 * j]);
  const float s = rms_scale_row<512, 3>(v, red);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int i = threadIdx.x + 512 * j;
    *reinterpret_cast<__half*>(act + act_off(b, i, nb)) = __hmul(f2h(v[j] * s), gamma[i]);
  }
}

// sum_sp part[sp][b][i] in split order; every load issued before the sum.
__device__ __forceinline__ float sum_splits(const float* __restrict__ part, int splits, int nbv,
                                            int n, int b, int i) {
  const size_t stride = (size_t)nbv * n, idx = (size_t)b * n + i;
  float v[kTcMaxSplits];
#pragma unroll
  for (int sp = 0; sp < kTcMaxSplits; ++sp) v[sp] = sp < splits ? __ldcg(part + sp * stride + idx) : 0.f;
  float s = 0.f;
#pragma unroll
  for (int sp = 0; sp < kTcMaxSplits; ++sp)
    if (sp < splits) s += v[sp];
  return s;
}

// QKV epilogue, one CTA per (sequence, head): biases, fp16 rounding, RoPE at
// position seq_len - 1 on the 12 q heads and 2 k heads (blockIdx.y < 14), K/V
// appended to the cache (blockIdx.y 12..14).
__global__ void __launch_bounds__(64) k_qkv_finish(const float* __restrict__ part, int splits, int nbv,
                                                   const __half* __restrict__ bias,
                                                   const float* __restrict__ rope_cs,
                                                   const uint32_t* __restrict__ seq_len,
                                                   int seq_len_stride,
                                                   const int32_t* __restrict__ row_seq, int max_ctx,
                                                   __half* __restrict__ q, __half* __restrict__ kc,
                                                   __half* __restrict__ vc, size_t kv_seq_stride) {
  pdl_prologue();
  const int b = blockIdx.x, head = blockIdx.y, t = threadIdx.x;
  const uint32_t L = seq_len[(size_t)b * seq_len_stride];
  const int kvs = row_seq ? row_seq[b] : b;  // the row's KV sequence
  const uint32_t pos = L - 1;
  if (L == 0 || pos >= (uint32_t)max_ctx) return;  // step_begin clamps; never taken
  if (head < kHeads + kKVHeads) {
    const int i0 = head * 128 + t;  // q heads, then the k heads at 1536
    const float x1 = h2f(f2h(sum_splits(part, splits, nbv, kQKVRows, b, i0) + h2f(bias[i0])));
    const float x2 =
        h2f(f2h(sum_splits(part, splits, nbv, kQKVRows, b, i0 + 64) + h2f(bias[i0 + 64])));
    const float* cs = rope_cs + (size_t)pos * 128;
    const float c = cs[2 * t], s = cs[2 * t + 1];
    const __half r1 = f2h(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
    const __half r2 = f2h(__fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c)));
    if (head < kHeads) {
      q[(size_t)b * kHidden + i0] = r1;
      q[(size_t)b * kHidden + i0 + 64] = r2;
    } else {
      __half* kr = kc + (size_t)kvs * kv_seq_stride + (size_t)pos * kKVDim;
      kr[i0 - kHidden] = r1;
      kr[i0 - kHidden + 64] = r2;
    }
  } else {
    __half* vr = vc + (size_t)kvs * kv_seq_stride + (size_t)pos * kKVDim;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = kHidden + kKVDim + t + 64 * e;
      vr[i - kHidden - kKVDim] = f2h(sum_splits(part, splits, nbv, kQKVRows, b, i) + h2f(bias[i]));
    }
  }
}

// x <- half(x + half(sum + bias)); act_h row <- rmsnorm(x) with gamma.  A
// cluster of kFinCtas CTAs per row, one column per thread, so every thread
// issues all its split loads at once (one CTA per row kept 84 of 148 SMs idle
// and walked three columns per thread); the row's sum of squares meets in
// distributed shared memory (each rank pushes its partial to every rank), added in rank order.
constexpr int kFinCtas = 4;
constexpr int kFinThreads = kHidden / kFinCtas;  // 384
__global__ void __launch_bounds__(kFinThreads) k_resid_norm_finish(
    const float* __restrict__ part, int splits, int nbv, const __half* __restrict__ bias,
    __half* __restrict__ x, const __half* __restrict__ gamma, uint8_t* __restrict__ act, int nb) {
  pdl_prologue();
  namespace cg = cooperative_groups;
  __shared__ float red[kFinThreads / 32];
  __shared__ float ss_in[kFinCtas];  // every rank's sum of squares, written by that rank
  cg::cluster_group cluster = cg::this_cluster();
  const int b = blockIdx.y;
  const int rank = (int)cluster.block_rank();
  const int i = rank * kFinThreads + (int)threadIdx.x;
  __half* xr = x + (size_t)b * kHidden;
  const __half y = f2h(sum_splits(part, splits, nbv, kHidden, b, i) + h2f(bias[i]));
  const __half xn = __hadd(xr[i], y);
  xr[i] = xn;
  const float v = h2f(xn);
  const float acc = warp_sum(v * v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kFinThreads / 32; ++w) t += red[w];
#pragma unroll
    for (int r = 0; r < kFinCtas; ++r) *cluster.map_shared_rank(&ss_in[rank], r) = t;
  }
  // the pushes land before the barrier and the sums are then read locally, so
  // no CTA touches another's shared memory after it (no second barrier before
  // exit)
  cluster.sync();
  float tot = 0.f;
#pragma unroll
  for (int r = 0; r < kFinCtas; ++r) tot += ss_in[r];
  const float sc = 1.0f / sqrtf(tot / 1536.0f + kRmsEps);
  *reinterpret_cast<__half*>(act + act_off(b, i, nb)) = __hmul(f2h(v * sc), gamma[i]);
}

// Row r = position p0 + r of sequence 0: x[r] = embedding of its prompt id,
// len[r] = p0 + r + 1 (InferenceEngine.swift:57-60 per position).
// Rows of one chunk of a prefill: row r = b * n_pos + j is position p0 + j of
// sequence b -- the embedding of its prompt id, its length and its KV sequence.
__global__ void __launch_bounds__(192) k_prefill_rows(const int32_t* __restrict__ prompt,
                                                      int prompt_stride, int p0, int n_pos,
                                                      const __half* __restrict__ embed,
                                                      __half* __restrict__ x,
                                                      uint32_t* __restrict__ len,
                                                      int32_t* __restrict__ row_seq) {
  const int r = blockIdx.x, b = r / n_pos, j = r % n_pos;
  const int32_t tok = prompt[(size_t)b * prompt_stride + p0 + j];
  if (threadIdx.x == 0) {
    len[r] = (uint32_t)(p0 + j + 1);
    row_seq[r] = b;
  }
  reinterpret_cast<uint4*>(x + (size_t)r * kHidden)[threadIdx.x] =
      reinterpret_cast<const uint4*>(embed + (size_t)tok * kHidden)[threadIdx.x];
}

struct TcPlan {
  int qkv, o, down;  // K splits (gate/up runs unsplit: its epilogue needs whole sums)
};

TcPlan plan_for(int sm_count) {
  return TcPlan{tc_choose_splits(kQKVTiles, kChunks1536, sm_count),
                tc_choose_splits(kOTiles, kChunks1536, sm_count),
                tc_choose_splits(kDownTiles, kChunks8960, sm_count)};
}

int gemm(const uint8_t* blob, bool q4, const uint8_t* act, const InferenceManager& s, int rows,
         int n_rows, int k, int splits, float* part, __half* out, long long ld_out, cudaStream_t st,
         uint8_t* swiglu_act = nullptr) {
  TcGemmArgs a;
  a.w = blob;
  a.q4 = q4;
  a.act = act;
  a.nb = act_rows(rows);
  a.act_stride_rows = s.tc_nb;
  a.nb_valid = rows;
  a.n_rows = n_rows;
  a.k = k;
  a.splits = splits;
  a.part = part;
  a.out = out;
  a.ld_out = ld_out;
  a.swiglu_act = swiglu_act;
  a.swiglu_nb = s.tc_nb;
  a.err = s.err;
  a.pdl = true;
  if (launch_tc_gemm(a, st) != 0) return launch_status("tensor-core projection");
  return QWEN_OK;
}

}  // namespace

// Decode steps: 7 kernels a layer (the attention forms q and the new k / v
// rows from the QKV partials itself); a chunked prefill launches the QKV
// finish too (8 a layer).
int tc_kernels_per_step(int n_layers) { return 1 + 7 * n_layers + 1; }

int build_tc_weights(QwenModel& m, int max_ctx, cudaStream_t st) {
  TcWeights& t = m.tc;
  t.layer_bytes = kTcLayerBytes;
  if (!t.blob) QWEN_CUDA(cudaMalloc(&t.blob, kTcLayerBytes * m.n_layers), "cudaMalloc(tc weights)");
  if (!t.lm) QWEN_CUDA(cudaMalloc(&t.lm, f16_tc_blob_bytes(kVocab, kHidden)), "cudaMalloc(tc lm)");
  auto rq = [&](const Q4Linear& w, uint8_t* dst) {
    return launch_repack_q4_tc(w.packed, w.scales, w.rows, w.k, dst, st) == 0
               ? QWEN_OK
               : launch_status("repack q4 (tensor-core layout)");
  };
  for (int l = 0; l < m.n_layers; ++l) {
    const QwenLayer& L = m.layers[l];
    uint8_t* base = t.blob + kTcLayerBytes * l;
    uint8_t* qkv = base;
    uint8_t* o = qkv + kTcQKVBytes;
    uint8_t* gu = o + kTcOBytes;
    uint8_t* down = gu + kTcGUBytes;
    // Concatenating rows = concatenating whole tiles of the blob.
    QWEN_TRY(rq(L.q, qkv));
    QWEN_TRY(rq(L.k, qkv + (size_t)(kHidden / kTcM) * kChunks1536 * kQ4TcChunkBytes));
    QWEN_TRY(rq(L.v, qkv + (size_t)((kHidden + kKVDim) / kTcM) * kChunks1536 * kQ4TcChunkBytes));
    QWEN_TRY(rq(L.o, o));
    // Gate/up pairing: tile t = gate rows 64t .. 64t+63, then up rows 64t .. 64t+63.
    if (launch_repack_q4_tc_rows(L.gate.packed, L.gate.scales, kInter, kHidden, gu, 64, 0, st) ||
        launch_repack_q4_tc_rows(L.up.packed, L.up.scales, kInter, kHidden, gu, 64, 64, st))
      return launch_status("repack gate/up (tensor-core layout)");
    QWEN_TRY(rq(L.down, down));
  }
  if (launch_repack_f16_tc(m.embed, kVocab, kHidden, t.lm, st) != 0)
    return launch_status("repack lm head");
  QWEN_TRY(upload_rope_table(&t.rope_cs, &t.rope_ctx, max_ctx, st));
  QWEN_CUDA(cudaStreamSynchronize(st), "sync");
  return QWEN_OK;
}

int tc_state_allocate(InferenceManager& s, int sm_count) {
  if (s.act_h) return QWEN_OK;
  if (s.batch > kTcMaxNb)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "tensor-core step: batch %d > %d", s.batch, kTcMaxNb);
  // Prefills run in chunks of rows, kTcPrefillRows positions of a batch-1
  // engine or kTcMaxNb (sequence, position) rows of a larger batch.
  s.tc_rows = s.batch == 1 ? kTcPrefillRows : kTcMaxNb;
  s.tc_nb = act_rows(s.tc_rows);
  const TcPlan p = plan_for(sm_count);
  const size_t part = std::max((size_t)p.qkv * kQKVRows,
                               std::max((size_t)p.o * kHidden, (size_t)p.down * kHidden)) *
                      s.tc_rows;
  QWEN_TRY(s.alloc_tracked(act_bytes(s.tc_nb, kHidden), (void**)&s.act_h));
  QWEN_TRY(s.alloc_tracked(act_bytes(s.tc_nb, kInter), (void**)&s.act_i));
  QWEN_TRY(s.alloc_tracked(part * sizeof(float), (void**)&s.tc_part));
  {
    const size_t R = (size_t)s.tc_rows;
    QWEN_TRY(s.alloc_tracked(R * kHidden * 2, (void**)&s.tc_px));
    QWEN_TRY(s.alloc_tracked(R * kHidden * 2, (void**)&s.tc_pq));
    QWEN_TRY(s.alloc_tracked(R * kVocab * 2, (void**)&s.tc_plogits));
    QWEN_TRY(s.alloc_tracked(R * sizeof(uint32_t), (void**)&s.tc_row_len));
    QWEN_TRY(s.alloc_tracked(R * sizeof(int32_t), (void**)&s.tc_row_seq));
    s.tc_psplits = attn_max_splits(s.max_ctx, s.tc_rows);
    QWEN_TRY(s.alloc_tracked(attn_scratch_bytes(s.tc_psplits, s.tc_rows), &s.tc_pattn));
  }
  return QWEN_OK;
}

TcRows tc_decode_rows(InferenceManager& s) {
  return TcRows{s.batch,        s.x,           s.q,
                &s.ctl[0].seq_len, (int)(sizeof(SeqCtl) / sizeof(uint32_t)), nullptr,
                s.attn_scratch, s.attn_splits, s.logits};
}

int launch_prefill_rows(InferenceManager& s, const __half* embed, int p0, int n_pos,
                        cudaStream_t st) {
  const int rows = s.batch * n_pos;
  if (!s.tc_px || n_pos < 1 || rows > s.tc_rows || p0 < 0 || p0 + n_pos > s.max_ctx)
    return set_error(QWEN_ERR_STATE, "chunked prefill: bad rows");
  k_prefill_rows<<<rows, kHidden / 8, 0, st>>>(s.prompt, s.max_ctx, p0, n_pos, embed, s.tc_px,
                                               s.tc_row_len, s.tc_row_seq);
  return launch_status("prefill rows");
}

int enqueue_tc_model(QwenModel& m, InferenceManager& s, const TcRows& v, int sm_count,
                     cudaStream_t st, cudaEvent_t* marks, int* n_marks) {
  // Optional per-launch timeline: an event after every kernel.
  auto mark = [&]() {
    if (marks) cudaEventRecord(marks[(*n_marks)++], st);
  };
  const TcWeights& t = m.tc;
  if (!t.blob || !s.act_h) return set_error(QWEN_ERR_STATE, "tensor-core step not prepared");
  if (t.rope_ctx < s.max_ctx) return set_error(QWEN_ERR_STATE, "RoPE table shorter than max_ctx");
  if (v.rows < 1 || v.rows > s.tc_rows) return set_error(QWEN_ERR_STATE, "tensor-core step: %d rows", v.rows);
  const TcPlan p = plan_for(sm_count);
  if (std::max(p.qkv, std::max(p.o, p.down)) > kTcMaxSplits)
    return set_error(QWEN_ERR_STATE, "tensor-core step: split plan exceeds %d", kTcMaxSplits);
  const int B = v.rows, nb = s.tc_nb;
  AttnParams ap{};
  ap.q = v.q;
  ap.q_seq_stride = kHidden;
  ap.kv_seq_stride = (long long)s.kv_seq_stride();
  ap.kv_pos_stride = kKVDim;
  ap.kv_head_stride = kHeadDim;
  ap.seq_len = v.seq_len;
  ap.seq_len_stride = v.seq_len_stride;
  ap.max_ctx = (uint32_t)s.max_ctx;
  ap.out = s.attn_out;
  ap.out_seq_stride = kHidden;
  ap.act_out = s.act_h;  // the O projection's input tiles, written directly
  ap.act_nb = nb;
  ap.row_seq = v.row_seq;
  ap.kv_n_seq = s.batch;
  ap.err = s.err;
  // Decode rows: the attention forms q and the step's new k / v rows from the
  // QKV partials (no finish kernel).  A chunked prefill's rows attend to each
  // other's new rows, which must all be in the caches first: it keeps the
  // QKV finish.
  const bool fused_qkv = v.row_seq == nullptr;
  if (fused_qkv) {
    ap.qkv_part = s.tc_part;
    ap.qkv_splits = p.qkv;
    ap.qkv_rows = B;
    ap.rope_cs = t.rope_cs;
  }
  attn_bind_scratch(ap, v.attn_scratch, v.attn_splits, B);

  QWEN_TRY(launch_pdl(k_rms_to_act, dim3(B), dim3(512), st, v.x, m.layers[0].input_norm, s.act_h, nb));
  mark();
  for (int l = 0; l < m.n_layers; ++l) {
    const QwenLayer& L = m.layers[l];
    const uint8_t* qkv = t.blob + t.layer_bytes * l;
    const uint8_t* o = qkv + kTcQKVBytes;
    const uint8_t* gu = o + kTcOBytes;
    const uint8_t* down = gu + kTcGUBytes;
    __half* kc = s.kc + (size_t)l * s.kv_layer_stride();
    __half* vc = s.vc + (size_t)l * s.kv_layer_stride();

    QWEN_TRY(gemm(qkv, true, s.act_h, s, B, kQKVRows, kHidden, p.qkv, s.tc_part, nullptr, 0, st));
    mark();
    if (fused_qkv) {
      ap.qkv_bias = L.qkv_bias;
    } else {
      QWEN_TRY(launch_pdl(k_qkv_finish, dim3(B, kHeads + kKVHeads + 1), dim3(64), st, s.tc_part,
                          p.qkv, B, L.qkv_bias, t.rope_cs, v.seq_len, v.seq_len_stride, v.row_seq,
                          s.max_ctx, v.q, kc, vc, s.kv_seq_stride()));
      mark();
    }
    ap.k = kc;
    ap.v = vc;
    if (launch_attention_decode(ap, v.attn_splits, B, st, true) != 0)
      return set_error(QWEN_ERR_CUDA, "attention launch failed (%s)", cudaGetErrorString(cudaGetLastError()));
    mark();
    QWEN_TRY(gemm(o, true, s.act_h, s, B, kHidden, kHidden, p.o, s.tc_part, nullptr, 0, st));
    mark();
    QWEN_TRY(launch_pdl_cluster(k_resid_norm_finish, dim3(kFinCtas, B), dim3(kFinThreads), kFinCtas,
                                st, s.tc_part, p.o, B, L.o_bias, v.x, L.post_attn_norm, s.act_h,
                                nb));
    mark();
    QWEN_TRY(gemm(gu, true, s.act_h, s, B, 2 * kInter, kHidden, 1, nullptr, nullptr, 0, st, s.act_i));
    mark();
    QWEN_TRY(gemm(down, true, s.act_i, s, B, kHidden, kInter, p.down, s.tc_part, nullptr, 0, st));
    mark();
    const __half* next_norm = l + 1 < m.n_layers ? m.layers[l + 1].input_norm : m.final_norm;
    QWEN_TRY(launch_pdl_cluster(k_resid_norm_finish, dim3(kFinCtas, B), dim3(kFinThreads), kFinCtas,
                                st, s.tc_part, p.down, B, L.down_bias, v.x, next_norm, s.act_h,
                                nb));
    mark();
  }
  if (v.logits) {
    QWEN_TRY(gemm(t.lm, false, s.act_h, s, B, kVocab, kHidden, 1, nullptr, v.logits, kVocab, st));
    mark();
  }
  return launch_status("tensor-core model step");
}

}  // namespace qwen
