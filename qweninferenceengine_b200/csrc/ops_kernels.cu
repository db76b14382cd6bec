// ops_kernels.cu -- one CUDA kernel per reference Metal pipeline, taking the
// reference's own buffer layouts (the operator-level drop-in boundary).
//
//   gemv_q4_0        matmul.metal:9-73       -> k_gemv_q4_rowmajor
//   gemv_fp16        matmul.metal:75-113     -> k_gemv_fp16_rowmajor
//   rms_norm_q4      rmsnorm.metal:9-46      -> k_rms_norm
//   apply_rope_q4    rope.metal:12-39        -> k_rope
//   write_kv_cache   attention.metal:67-84   -> k_write_kv_cache
//   attention_scores attention.metal:9-32    -> k_attention_scores
//   softmax          activations.metal:29-55 -> k_softmax
//   attn_weighted_sum attention.metal:34-56  -> k_attn_weighted_sum
//   residual_add     attention.metal:58-65   -> k_residual_add
//   swiglu           activations.metal:9-27  -> k_swiglu
//
// The fused decode step (decode_step.cu) does not use these; they exist so a
// caller can replace the reference's dispatches one by one.
#include "qwen_common.cuh"
#include "qwen_internal.h"

namespace qwen {

__constant__ float c_inv_freq[64];  // 1e6^(-2i/128), computed on the host with libm powf

// ------------------------------------------------------------ Q4 GEMV ----
// One CTA (4 warps) per 16-row tile; warp w takes blocks b = w, w+4, ...
// x fragments are staged in shared memory once per CTA.
__global__ void __launch_bounds__(128) k_gemv_q4_rowmajor(const uint8_t* __restrict__ packed,
                                                          const __half* __restrict__ scales,
                                                          const __half* __restrict__ x,
                                                          __half* __restrict__ y,
                                                          const __half* __restrict__ bias,
                                                          int n_rows, int k) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint4* xf = reinterpret_cast<uint4*>(smem);  // [k/32][4] fragments
  __shared__ float red[4][16];
  const int nblk = k / 32;
  for (int i = threadIdx.x; i < nblk * 4; i += blockDim.x) {
    const int b = i >> 2, t = i & 3;
    const uint4 raw = *reinterpret_cast<const uint4*>(x + 32 * b + 8 * t);
    __half v[8];
    *reinterpret_cast<uint4*>(v) = raw;
    xf[i] = make_xfrag(v);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * 16;
  const int rg = row0 + g, rg8 = row0 + g + 8;
  const bool vg = rg < n_rows, vg8 = rg8 < n_rows;
  const uint8_t* wg_row = packed + (size_t)(vg ? rg : 0) * (k / 2) + 4 * t;
  const uint8_t* wg8_row = packed + (size_t)(vg8 ? rg8 : 0) * (k / 2) + 4 * t;
  const __half* sg_row = scales + (size_t)(vg ? rg : 0) * nblk;
  const __half* sg8_row = scales + (size_t)(vg8 ? rg8 : 0) * nblk;
  float acc_g = 0.f, acc_g8 = 0.f;
  for (int b = warp; b < nblk; b += 4) {
    const uint32_t wg = vg ? __ldg(reinterpret_cast<const uint32_t*>(wg_row + 16 * b)) : 0x88888888u;
    const uint32_t wg8 = vg8 ? __ldg(reinterpret_cast<const uint32_t*>(wg8_row + 16 * b)) : 0x88888888u;
    float d[4];
    q4_block_mma(wg, wg8, xf[b * 4 + t], d);
    acc_g += __half2float(sg_row[b]) * d[0];
    acc_g8 += __half2float(sg8_row[b]) * d[2];
  }
  if (t == 0) {
    red[warp][g] = acc_g;
    red[warp][g + 8] = acc_g8;
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int r = row0 + threadIdx.x;
    if (r < n_rows) {
      float s = red[0][threadIdx.x] + red[1][threadIdx.x] + red[2][threadIdx.x] + red[3][threadIdx.x];
      if (bias) s += __half2float(bias[r]);
      y[r] = f2h(s);
    }
  }
}

// Same product for K up to kGemvTileMaxK, with the CTA's whole 16-row tile in
// flight at once: every thread issues 16-byte cp.async copies of the tile's
// packed rows into shared memory (rows padded by 16 bytes, so the fragment
// reads of rows g and g + 8 hit distinct banks), then 8 warps take blocks
// b = w, w + 8, ... from shared memory.  One kernel of ~560 CTAs keeps ~50 KB
// of weights in flight per SM, where the per-block 4-byte loads of
// k_gemv_q4_rowmajor kept one block per warp.  Launched as a programmatic
// dependent: the weights and scales (which no earlier kernel writes) are
// fetched before griddepcontrol.wait, x (which the previous kernel may have
// produced) and y after it, so back-to-back projections overlap a kernel's
// weight fetch with the previous one's tail.
constexpr int kGemvTileMaxK = 3072;
constexpr int kGemvTileThreads = 256;
__host__ __device__ inline int gemv_tile_row_stride(int k) { return k / 2 + 16; }
__host__ __device__ inline int gemv_tile_smem(int k) {
  const int nblk = k / 32;
  return 16 * gemv_tile_row_stride(k) + ((16 * nblk * 2 + 15) / 16) * 16 + nblk * 4 * 16;
}

__global__ void __launch_bounds__(kGemvTileThreads) k_gemv_q4_tile(const uint8_t* __restrict__ packed,
                                                                  const __half* __restrict__ scales,
                                                                  const __half* __restrict__ x,
                                                                  __half* __restrict__ y,
                                                                  const __half* __restrict__ bias,
                                                                  int n_rows, int k) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[kGemvTileThreads / 32][16];
  const int rb = k / 2, rs = gemv_tile_row_stride(k), nblk = k / 32;
  uint8_t* wt = smem;                                                 // [16][rs]
  __half* sc = reinterpret_cast<__half*>(smem + 16 * rs);              // [16][nblk]
  uint4* xf = reinterpret_cast<uint4*>(smem + 16 * rs + ((16 * nblk * 2 + 15) / 16) * 16);  // [nblk][4]
  const int row0 = blockIdx.x * 16;
  const int rows = min(16, n_rows - row0);
  const int chunks = rb / 16;
  if (threadIdx.x == 0) pdl_launch_dependents();
  for (int c = threadIdx.x; c < rows * chunks; c += kGemvTileThreads) {
    const int r = c / chunks, j = c - r * chunks;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(wt + r * rs + 16 * j)),
                 "l"(packed + (size_t)(row0 + r) * rb + 16 * j)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  // scales (contiguous for the tile's rows) and the x fragments, meanwhile
  for (int i = threadIdx.x; i < rows * nblk; i += kGemvTileThreads) sc[i] = scales[(size_t)row0 * nblk + i];
  pdl_wait();
  for (int i = threadIdx.x; i < nblk * 4; i += kGemvTileThreads) {
    const int b = i >> 2, t = i & 3;
    __half v[8];
    *reinterpret_cast<uint4*>(v) = *reinterpret_cast<const uint4*>(x + 32 * b + 8 * t);
    xf[i] = make_xfrag(v);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  // rows past n_rows hold stale shared memory: their sums are never stored
  const uint8_t* wg_row = wt + g * rs + 4 * t;
  const uint8_t* wg8_row = wt + (g + 8) * rs + 4 * t;
  float acc_g = 0.f, acc_g8 = 0.f;
  for (int b = warp; b < nblk; b += kGemvTileThreads / 32) {
    const uint32_t wg = *reinterpret_cast<const uint32_t*>(wg_row + 16 * b);
    const uint32_t wg8 = *reinterpret_cast<const uint32_t*>(wg8_row + 16 * b);
    float d[4];
    q4_block_mma(wg, wg8, xf[b * 4 + t], d);
    acc_g += __half2float(sc[g * nblk + b]) * d[0];
    acc_g8 += __half2float(sc[(g + 8) * nblk + b]) * d[2];
  }
  if (t == 0) {
    red[warp][g] = acc_g;
    red[warp][g + 8] = acc_g8;
  }
  __syncthreads();
  if (threadIdx.x < rows) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kGemvTileThreads / 32; ++w) s += red[w][threadIdx.x];
    const int r = row0 + threadIdx.x;
    if (bias) s += __half2float(bias[r]);
    y[r] = f2h(s);
  }
}

// ----------------------------------------------------------- fp16 GEMV ----
// One CTA (4 warps) per 16-row tile, warp w takes k16 steps s = w, w+4, ...
// Lane (g,t) feeds W[g][16s+4t..+3] and W[g+8][..] as its A fragment and
// x[16s+4t..+3] as its B fragment (the k order inside a step is free).
__global__ void __launch_bounds__(128) k_gemv_fp16_rowmajor(const __half* __restrict__ w,
                                                            const __half* __restrict__ x,
                                                            __half* __restrict__ y, int n_rows,
                                                            int k) {
  __shared__ float red[4][16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * 16;
  const int rg = row0 + g, rg8 = row0 + g + 8;
  const bool vg = rg < n_rows, vg8 = rg8 < n_rows;
  const __half* wg = w + (size_t)(vg ? rg : 0) * k + 4 * t;
  const __half* wg8 = w + (size_t)(vg8 ? rg8 : 0) * k + 4 * t;
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  const int nsteps = k / 16;
  for (int s = warp; s < nsteps; s += 4) {
    uint2 a0 = vg ? __ldg(reinterpret_cast<const uint2*>(wg + 16 * s)) : make_uint2(0, 0);
    uint2 a1 = vg8 ? __ldg(reinterpret_cast<const uint2*>(wg8 + 16 * s)) : make_uint2(0, 0);
    const uint2 bx = __ldg(reinterpret_cast<const uint2*>(x + 16 * s + 4 * t));
    const uint32_t a[4] = {a0.x, a1.x, a0.y, a1.y};
    mma_16816(d, a, bx.x, bx.y, d);
  }
  if (t == 0) {
    red[warp][g] = d[0];
    red[warp][g + 8] = d[2];
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int r = row0 + threadIdx.x;
    if (r < n_rows)
      y[r] = f2h(red[0][threadIdx.x] + red[1][threadIdx.x] + red[2][threadIdx.x] +
                 red[3][threadIdx.x]);
  }
}

// ------------------------------------------------------------ RMSNorm -----
// out = half(half(x * s) * gamma), s = 1/sqrt(sum(x^2)/1536 + 1e-6).
__global__ void __launch_bounds__(256) k_rms_norm(const __half* __restrict__ x,
                                                  const __half* __restrict__ gamma,
                                                  __half* __restrict__ out) {
  __shared__ float part[8];
  __shared__ float scale;
  float acc = 0.f;
  for (int i = threadIdx.x; i < kHidden; i += 256) {
    const float v = h2f(x[i]);
    acc += v * v;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < 8; ++i) tot += part[i];
    scale = 1.0f / sqrtf(tot / 1536.0f + kRmsEps);
  }
  __syncthreads();
  const float s = scale;
  for (int i = threadIdx.x; i < kHidden; i += 256)
    out[i] = __hmul(f2h(h2f(x[i]) * s), gamma[i]);
}

// --------------------------------------------------------------- RoPE -----
__global__ void k_rope(__half* __restrict__ vec, int n_heads, const uint32_t* __restrict__ seq_len) {
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= n_heads * 64) return;
  const int head = tid / 64, pair = tid % 64;
  const int i0 = head * 128 + pair, i1 = i0 + 64;
  const float m = (float)(seq_len[0] - 1);
  const float theta = m * c_inv_freq[pair];
  float s, c;
  sincosf(theta, &s, &c);
  const float x1 = h2f(vec[i0]), x2 = h2f(vec[i1]);
  vec[i0] = f2h(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
  vec[i1] = f2h(__fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c)));
}

// ----------------------------------------------------------- KV write -----
__global__ void k_write_kv_cache(const __half* __restrict__ k, const __half* __restrict__ v,
                                 __half* __restrict__ kc, __half* __restrict__ vc,
                                 const uint32_t* __restrict__ seq_len, uint32_t max_ctx) {
  const int tid = threadIdx.x;
  if (tid >= kKVDim) return;
  const uint32_t pos = seq_len[0] - 1;
  if (pos >= max_ctx) return;
  kc[(size_t)pos * kKVDim + tid] = k[tid];
  vc[(size_t)pos * kKVDim + tid] = v[tid];
}

// ----------------------------------------------- attention, three passes --
// scores[h][t] = 0.088388 * q_h . K[t, (h/6)*128 : +128]; one warp per (h, t).
__global__ void k_attention_scores(const __half* __restrict__ q, const __half* __restrict__ kc,
                                   float* __restrict__ scores, const uint32_t* __restrict__ seq_len) {
  const uint32_t L = seq_len[0];
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int h = warp % kHeads;
  const uint32_t t = warp / kHeads;
  if (t >= L) return;
  const __half* qp = q + h * kHeadDim + lane * 4;
  const __half* kp = kc + (size_t)t * kKVDim + (h / 6) * kHeadDim + lane * 4;
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) acc += h2f(qp[j]) * h2f(kp[j]);
  acc = warp_sum(acc);
  if (lane == 0) scores[(size_t)h * L + t] = acc * kAttnScale;
}

// Per head: max (initial -1e9), e = exp(s - max), sum (0 -> 1e-9), divide.
__global__ void __launch_bounds__(256) k_softmax(float* __restrict__ scores,
                                                 const uint32_t* __restrict__ seq_len) {
  const uint32_t L = seq_len[0];
  float* s = scores + (size_t)blockIdx.x * L;
  __shared__ float part[8];
  __shared__ float bcast;
  float mx = -1e9f;
  for (uint32_t i = threadIdx.x; i < L; i += 256) mx = fmaxf(mx, s[i]);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = part[0];
    for (int i = 1; i < 8; ++i) m = fmaxf(m, part[i]);
    bcast = m;
  }
  __syncthreads();
  mx = bcast;
  float sum = 0.f;
  for (uint32_t i = threadIdx.x; i < L; i += 256) {
    const float e = expf(s[i] - mx);
    s[i] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < 8; ++i) tot += part[i];
    bcast = tot == 0.f ? 1e-9f : tot;
  }
  __syncthreads();
  const float inv_den = bcast;
  for (uint32_t i = threadIdx.x; i < L; i += 256) s[i] = s[i] / inv_den;
}

// out[h*128+d] = half(sum_t P[h][t] * V[t][(h/6)*128 + d]).
__global__ void k_attn_weighted_sum(const float* __restrict__ scores, const __half* __restrict__ vc,
                                    __half* __restrict__ out, const uint32_t* __restrict__ seq_len) {
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= kHidden) return;
  const uint32_t L = seq_len[0];
  const int h = tid / 128, d = tid % 128, vh = h / 6;
  const float* p = scores + (size_t)h * L;
  const __half* vp = vc + vh * kHeadDim + d;
  float acc = 0.f;
  for (uint32_t t = 0; t < L; ++t) acc += p[t] * h2f(vp[(size_t)t * kKVDim]);
  out[tid] = f2h(acc);
}

// ---------------------------------------------------------- elementwise ---
__global__ void k_residual_add(const __half* __restrict__ a, const __half* __restrict__ b,
                               __half* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __hadd(a[i], b[i]);
}


__global__ void k_swiglu(__half* __restrict__ gate, const __half* __restrict__ up, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) gate[i] = f2h(silu_ref(h2f(gate[i])) * h2f(up[i]));
}

// ------------------------------------------------------------- dequant ----
__global__ void k_dequant_q4(const uint8_t* __restrict__ packed, const __half* __restrict__ scales,
                             size_t n_weights, float* __restrict__ out) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_weights / 8) return;
  // Decode 8 weights through the same word dequantiser the GEMV kernels use.
  const uint32_t w = reinterpret_cast<const uint32_t*>(packed)[i];
  uint32_t h[4];
  dequant_word(w, h);
  const float s = h2f(scales[(i * 8) / 32]);
  const __half2* hp = reinterpret_cast<const __half2*>(h);
  // h[0] = (k0,k4), h[1] = (k1,k5), h[2] = (k2,k6), h[3] = (k3,k7)
  float q[8];
  for (int j = 0; j < 4; ++j) {
    q[j] = __low2float(hp[j]);
    q[j + 4] = __high2float(hp[j]);
  }
  for (int j = 0; j < 8; ++j) out[i * 8 + j] = q[j] * s;
}

// ---------------------------------------------------------- host side -----
static inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int launch_gemv_q4_rowmajor(const uint8_t* packed, const __half* scales, const __half* x,
                            __half* y, const __half* bias, int n_rows, int k, void* stream) {
  // The tile kernel wants 16-byte aligned rows (k a multiple of 32 makes each
  // row 16-byte sized) and an aligned x for its 16-byte fragment loads.
  if (k <= kGemvTileMaxK && (reinterpret_cast<uintptr_t>(packed) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((n_rows + 15) / 16);
    cfg.blockDim = dim3(kGemvTileThreads);
    cfg.dynamicSmemBytes = gemv_tile_smem(k);
    cfg.stream = S(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_gemv_q4_tile, packed, scales, x, y, bias, n_rows, k) == cudaSuccess ? 0 : -1;
  }
  const int smem = (k / 32) * 64;
  if (smem > 48 * 1024) {
    static bool attr_set = false;
    if (!attr_set) {
      cudaFuncSetAttribute(k_gemv_q4_rowmajor, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           200 * 1024);
      attr_set = true;
    }
  }
  k_gemv_q4_rowmajor<<<(n_rows + 15) / 16, 128, smem, S(stream)>>>(packed, scales, x, y, bias,
                                                                    n_rows, k);
  return 0;
}

int launch_gemv_fp16_rowmajor(const __half* w, const __half* x, __half* y, int n_rows, int k,
                              void* stream) {
  k_gemv_fp16_rowmajor<<<(n_rows + 15) / 16, 128, 0, S(stream)>>>(w, x, y, n_rows, k);
  return 0;
}

int launch_rms_norm(const __half* x, const __half* gamma, __half* out, void* stream) {
  k_rms_norm<<<1, 256, 0, S(stream)>>>(x, gamma, out);
  return 0;
}

int set_rope_inv_freq(const float* inv_freq64) {
  return cudaMemcpyToSymbol(c_inv_freq, inv_freq64, 64 * sizeof(float)) == cudaSuccess ? 0 : -1;
}

int launch_rope(__half* vec, int n_heads, const uint32_t* seq_len, void* stream) {
  const int n = n_heads * 64;
  k_rope<<<(n + 255) / 256, 256, 0, S(stream)>>>(vec, n_heads, seq_len);
  return 0;
}

int launch_write_kv_cache(const __half* k, const __half* v, __half* kc, __half* vc,
                          const uint32_t* seq_len, uint32_t max_ctx, void* stream) {
  k_write_kv_cache<<<1, 256, 0, S(stream)>>>(k, v, kc, vc, seq_len, max_ctx);
  return 0;
}

int launch_attention_scores(const __half* q, const __half* kc, float* scores,
                            const uint32_t* seq_len, uint32_t max_seq, void* stream) {
  const size_t warps = (size_t)max_seq * kHeads;
  k_attention_scores<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, S(stream)>>>(q, kc, scores,
                                                                               seq_len);
  return 0;
}

int launch_softmax(float* scores, const uint32_t* seq_len, void* stream) {
  k_softmax<<<kHeads, 256, 0, S(stream)>>>(scores, seq_len);
  return 0;
}

int launch_attn_weighted_sum(const float* scores, const __half* vc, __half* out,
                             const uint32_t* seq_len, void* stream) {
  k_attn_weighted_sum<<<kHidden / 128, 128, 0, S(stream)>>>(scores, vc, out, seq_len);
  return 0;
}

int launch_residual_add(const __half* a, const __half* b, __half* out, int n, void* stream) {
  k_residual_add<<<(n + 255) / 256, 256, 0, S(stream)>>>(a, b, out, n);
  return 0;
}

int launch_swiglu(__half* gate, const __half* up, int n, void* stream) {
  k_swiglu<<<(n + 255) / 256, 256, 0, S(stream)>>>(gate, up, n);
  return 0;
}

int launch_dequant_q4(const uint8_t* packed, const __half* scales, size_t n_weights, float* out,
                      void* stream) {
  const size_t words = n_weights / 8;
  k_dequant_q4<<<(unsigned)((words + 255) / 256), 256, 0, S(stream)>>>(packed, scales, n_weights,
                                                                       out);
  return 0;
}

}  // namespace qwen
