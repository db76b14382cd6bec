// weights.cu -- device-side weight preparation: the packAndSave4Bit quantiser
// (QwenPipelines.swift:97-145), a counter-based normal generator for
// random-init models, and fp32 -> fp16 conversion.
#include "qwen_common.cuh"
#include "qwen_internal.h"

#include <cmath>

namespace qwen {

// One thread per 32-weight block of the flattened tensor:
//   scale = maxAbs / 7 (fp32, stored fp16), inv = 1/scale (0 if scale == 0),
//   q = clamp(round_half_away(w * inv), -8, 7) + 8, byte = qLow | qHigh << 4.
__global__ void k_quantize_q4(const float* __restrict__ w, size_t n, uint8_t* __restrict__ packed,
                              __half* __restrict__ scales) {
  const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t nb = (n + 31) / 32;
  if (b >= nb) return;
  const size_t start = b * 32;
  float v[32];
  float max_abs = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = start + i < n ? w[start + i] : 0.0f;
    max_abs = fmaxf(max_abs, fabsf(v[i]));
  }
  const float scale = __fdiv_rn(max_abs, 7.0f);
  const float inv = scale != 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
  scales[b] = f2h(scale);
  uint32_t words[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float rl = roundf(__fmul_rn(v[i], inv)), rh = roundf(__fmul_rn(v[i + 1], inv));
    int ql = (int)fminf(fmaxf(rl, -8.0f), 7.0f) + 8;
    int qh = (int)fminf(fmaxf(rh, -8.0f), 7.0f) + 8;
    const uint32_t byte = (uint32_t)(ql | (qh << 4));
    words[i / 8] |= byte << (8 * ((i / 2) & 3));
  }
  uint4* dst = reinterpret_cast<uint4*>(packed + b * 16);
  *dst = make_uint4(words[0], words[1], words[2], words[3]);
}

__device__ __forceinline__ uint64_t dev_splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Box-Muller on two 24-bit uniforms from SplitMix64 of (seed, stream, pair index).
__global__ void k_fill_normal(float* __restrict__ out, size_t n, uint64_t seed, uint64_t stream_id,
                              float mean, float stddev) {
  const size_t pair = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (2 * pair >= n) return;
  const uint64_t key = dev_splitmix64(seed ^ dev_splitmix64(stream_id * 0x100000001B3ull + 0x51ull));
  const uint64_t r = dev_splitmix64(key + pair);
  const float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
  const float u2 = (float)((r >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
  const float rad = sqrtf(-2.0f * logf(u1));
  float sn, cs;
  sincospif(2.0f * u2, &sn, &cs);
  out[2 * pair] = mean + stddev * rad * cs;
  if (2 * pair + 1 < n) out[2 * pair + 1] = mean + stddev * rad * sn;
}

__global__ void k_f32_to_f16(const float* __restrict__ in, __half* __restrict__ out, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = f2h(in[i]);
}

int launch_quantize_q4(const float* w, size_t n, uint8_t* packed, __half* scales,
                       cudaStream_t st) {
  const size_t nb = (n + 31) / 32;
  k_quantize_q4<<<(unsigned)((nb + 255) / 256), 256, 0, st>>>(w, n, packed, scales);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_fill_normal(float* out, size_t n, uint64_t seed, uint64_t stream_id, float mean,
                       float stddev, cudaStream_t st) {
  const size_t pairs = (n + 1) / 2;
  k_fill_normal<<<(unsigned)((pairs + 255) / 256), 256, 0, st>>>(out, n, seed, stream_id, mean,
                                                                 stddev);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_f32_to_f16(const float* in, __half* out, size_t n, cudaStream_t st) {
  k_f32_to_f16<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(in, out, n);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ------------------------------------------------------------ host side --
uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// 24-bit uniform for (seed, sequence, step).
uint32_t uniform24(uint64_t seed, uint64_t sequence, uint64_t step) {
  const uint64_t key = splitmix64((sequence << 32) ^ step);
  return (uint32_t)(splitmix64(seed ^ key) >> 40);
}

// 1e6^(-2i/128) in fp32 with libm powf, as rope.metal:29 evaluates it.
void rope_inv_freq(float* inv_freq64) {
  for (int i = 0; i < 64; ++i)
    inv_freq64[i] = std::pow(1000000.0f, -((float)(i * 2) / 128.0f));
}

}  // namespace qwen
