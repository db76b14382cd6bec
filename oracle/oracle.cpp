// oracle.cpp -- CPU oracle (test infrastructure; see oracle.h).
//
// Scalar restatement of the reference engine's arithmetic.  Every function
// cites the reference file:line it follows.  Compile with -ffp-contract=off so
// that a*b+c stays two rounded operations, as written in the reference source.
//
// Conventions taken where Metal leaves the order open (the same choices are
// made by oracle/metal_shim, so the compiled reference and this restatement
// agree bit for bit):
//   * simd_sum adds the 32 lanes in lane order, starting from lane 0.
//   * exp / pow / rsqrt / sin / cos are the accurate libm functions
//     (rsqrt(x) = 1/sqrt(x)); the Apple compiler's fast-math versions are not
//     available off Apple hardware.
#include "oracle.h"

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace {

constexpr int kHidden = 1536;
constexpr int kInter = 8960;
constexpr int kHeads = 12;
constexpr int kKVDim = 256;
constexpr int kHeadDim = 128;
constexpr int kVocab = 151936;
constexpr int kGemvThreads = 768;   // QwenConfig.swift:21
constexpr int kNormThreads = 256;   // InferenceEngine.swift:93

inline float h2f(uint16_t h) {
  _Float16 v;
  std::memcpy(&v, &h, 2);
  return (float)v;
}
inline uint16_t f2h(float f) {
  _Float16 v = (_Float16)f;
  uint16_t h;
  std::memcpy(&h, &v, 2);
  return h;
}
// half*half and half+half of the Metal source: exact in fp32, rounded once.
inline uint16_t hmul(uint16_t a, uint16_t b) { return f2h(h2f(a) * h2f(b)); }
inline uint16_t hadd(uint16_t a, uint16_t b) { return f2h(h2f(a) + h2f(b)); }

// simd_sum over one 32-lane group, lane order.
inline float simd_sum32(const float* lanes) {
  float acc = lanes[0];
  for (int i = 1; i < 32; ++i) acc += lanes[i];
  return acc;
}

// One threadgroup of gemv_q4_0 (matmul.metal:9-73): returns final_row_sum
// before the fp16 store.
float gemv_q4_row(const uint8_t* row_w, const uint16_t* row_s, const uint16_t* x, int k,
                  int threads, const uint16_t* bias_elem) {
  const int bytes_per_row = k / 2;
  const int stride = (bytes_per_row + threads - 1) / threads;
  const int simd_groups = threads / 32;
  float lanes[32];
  float shared_sums[32];
  for (int sg = 0; sg < simd_groups; ++sg) {
    for (int lane = 0; lane < 32; ++lane) {
      const int tid = sg * 32 + lane;
      float thread_sum = 0.0f;
      for (int i = 0; i < stride; ++i) {
        const int byte_idx = tid + i * threads;
        if (byte_idx >= bytes_per_row) break;
        const uint8_t packed = row_w[byte_idx];
        const float w_low = (float)((packed & 0x0f) - 8);
        const float w_high = (float)((packed >> 4) - 8);
        const float scale = h2f(row_s[byte_idx / 16]);
        const float a = w_low * scale * h2f(x[byte_idx * 2]);
        const float b = w_high * scale * h2f(x[byte_idx * 2 + 1]);
        thread_sum += a + b;
      }
      lanes[lane] = thread_sum;
    }
    shared_sums[sg] = simd_sum32(lanes);
  }
  float final_row_sum = 0.0f;
  for (int i = 0; i < simd_groups; ++i) final_row_sum += shared_sums[i];
  if (bias_elem) final_row_sum += h2f(*bias_elem);
  return final_row_sum;
}

}  // namespace

extern "C" {

// matmul.metal:9-73 -- one threadgroup per row, `threads` threads per group.
void oracle_gemv_q4_0(const uint8_t* packed, const uint16_t* scales, const uint16_t* x,
                      uint16_t* y, const uint16_t* bias, int n_rows, int k, int threads) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < n_rows; ++r) {
    const float s = gemv_q4_row(packed + (size_t)r * (k / 2), scales + (size_t)r * (k / 32), x,
                                k, threads, bias ? bias + r : nullptr);
    y[r] = f2h(s);
  }
}

// matmul.metal:75-113.
void oracle_gemv_fp16(const uint16_t* w, const uint16_t* x, uint16_t* y, int n_rows, int k,
                      int threads) {
  const int stride = (k + threads - 1) / threads;
  const int simd_groups = threads / 32;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < n_rows; ++r) {
    const uint16_t* row = w + (size_t)r * k;
    float lanes[32], shared_sums[32];
    for (int sg = 0; sg < simd_groups; ++sg) {
      for (int lane = 0; lane < 32; ++lane) {
        const int tid = sg * 32 + lane;
        float thread_sum = 0.0f;
        for (int i = 0; i < stride; ++i) {
          const int idx = tid + i * threads;
          if (idx < k) thread_sum += h2f(row[idx]) * h2f(x[idx]);
        }
        lanes[lane] = thread_sum;
      }
      shared_sums[sg] = simd_sum32(lanes);
    }
    float final_sum = 0.0f;
    for (int i = 0; i < simd_groups; ++i) final_sum += shared_sums[i];
    y[r] = f2h(final_sum);
  }
}

// rmsnorm.metal:9-46 (one threadgroup of `threads` threads, dim 1536).
void oracle_rms_norm(const uint16_t* x, const uint16_t* gamma, uint16_t* out, int threads) {
  const int num_simd = (threads + 31) / 32;
  float shared_sums[32];
  for (int sg = 0; sg < num_simd; ++sg) {
    float lanes[32];
    for (int lane = 0; lane < 32; ++lane) {
      const int tid = sg * 32 + lane;
      float acc = 0.0f;
      if (tid < threads)
        for (int i = tid; i < kHidden; i += threads) {
          const float v = h2f(x[i]);
          acc += v * v;
        }
      lanes[lane] = acc;
    }
    shared_sums[sg] = simd_sum32(lanes);
  }
  float total = 0.0f;
  for (int i = 0; i < num_simd; ++i) total += shared_sums[i];
  const float scale = 1.0f / std::sqrt(total / 1536.0f + 1e-6f);
  for (int i = 0; i < kHidden; ++i) out[i] = hmul(f2h(h2f(x[i]) * scale), gamma[i]);
}

// rope.metal:12-39: rotate-half pairs (i, i+64) of each 128-wide head,
// position m = seq_len - 1, theta base 1e6.
void oracle_rope(uint16_t* vec, int n_heads, uint32_t seq_len) {
  const float m = (float)(seq_len - 1);
  for (int tid = 0; tid < n_heads * 64; ++tid) {
    const int head = tid / 64, pair = tid % 64;
    const int i0 = head * 128 + pair, i1 = i0 + 64;
    const float theta = m * std::pow(1000000.0f, -((float)(pair * 2) / 128.0f));
    const float c = std::cos(theta), s = std::sin(theta);
    const float x1 = h2f(vec[i0]), x2 = h2f(vec[i1]);
    vec[i0] = f2h(x1 * c - x2 * s);
    vec[i1] = f2h(x1 * s + x2 * c);
  }
}

// attention.metal:67-84 (the 1024-slot guard is the reference's fixed cache
// size; here the caller sizes the cache).
void oracle_write_kv_cache(const uint16_t* k, const uint16_t* v, uint16_t* k_cache,
                           uint16_t* v_cache, uint32_t seq_len) {
  const uint32_t pos = seq_len - 1;
  for (int t = 0; t < kKVDim; ++t) {
    k_cache[(size_t)pos * kKVDim + t] = k[t];
    v_cache[(size_t)pos * kKVDim + t] = v[t];
  }
}

// attention.metal:9-32, activations.metal:29-55, attention.metal:34-56.
void oracle_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                      uint16_t* out, uint32_t seq_len, float* scores) {
  const uint32_t L = seq_len;
  for (int h = 0; h < kHeads; ++h) {  // attention_scores
    const int kh = h / 6;
    const uint16_t* qp = q + h * kHeadDim;
    for (uint32_t i = 0; i < L; ++i) {
      const uint16_t* kp = k_cache + (size_t)i * kKVDim + kh * kHeadDim;
      float dot = 0.0f;
      for (int d = 0; d < kHeadDim; ++d) dot += h2f(qp[d]) * h2f(kp[d]);
      scores[(size_t)h * L + i] = dot * 0.088388f;
    }
  }
  for (int h = 0; h < kHeads; ++h) {  // softmax
    float* s = scores + (size_t)h * L;
    float mx = -1e9f;
    for (uint32_t i = 0; i < L; ++i) mx = std::max(mx, s[i]);
    float sum = 0.0f;
    for (uint32_t i = 0; i < L; ++i) {
      const float e = std::exp(s[i] - mx);
      s[i] = e;
      sum += e;
    }
    if (sum == 0.0f) sum = 1e-9f;
    for (uint32_t i = 0; i < L; ++i) s[i] /= sum;
  }
  for (int tid = 0; tid < kHidden; ++tid) {  // attn_weighted_sum
    const int h = tid / 128, d = tid % 128, vh = h / 6;
    float acc = 0.0f;
    for (uint32_t i = 0; i < L; ++i)
      acc += scores[(size_t)h * L + i] * h2f(v_cache[(size_t)i * kKVDim + vh * kHeadDim + d]);
    out[tid] = f2h(acc);
  }
}

// attention.metal:58-65.
void oracle_residual_add(const uint16_t* x, const uint16_t* y, uint16_t* out, int n) {
  for (int i = 0; i < n; ++i) out[i] = hadd(x[i], y[i]);
}

// activations.metal:9-27.
void oracle_swiglu(uint16_t* gate, const uint16_t* up, int n) {
  for (int i = 0; i < n; ++i) {
    const float x = h2f(gate[i]);
    float silu;
    if (x > 15.0f) silu = x;
    else if (x < -15.0f) silu = 0.0f;
    else silu = x / (1.0f + std::exp(-x));
    gate[i] = f2h(silu * h2f(up[i]));
  }
}

// QwenPipelines.swift:97-145: symmetric block-32 quantizer over the flattened
// tensor.  scale = maxAbs/7 (stored fp16), q = clamp(round(w/scale), -8, 7)+8,
// Swift round() = half away from zero = roundf; byte = qLow | qHigh << 4.
void oracle_quantize_q4(const float* w, size_t n, uint8_t* packed, uint16_t* scales) {
  const size_t nb = (n + 31) / 32;
#pragma omp parallel for schedule(static)
  for (long long bl = 0; bl < (long long)nb; ++bl) {
    const size_t b = (size_t)bl, start = b * 32;
    float max_abs = 0.0f;
    for (int i = 0; i < 32; ++i)
      if (start + i < n) max_abs = std::max(max_abs, std::fabs(w[start + i]));
    const float scale = max_abs / 7.0f;
    const float inv = scale != 0.0f ? 1.0f / scale : 0.0f;
    scales[b] = f2h(scale);
    for (int i = 0; i < 32; i += 2) {
      const float wl = start + i < n ? w[start + i] : 0.0f;
      const float wh = start + i + 1 < n ? w[start + i + 1] : 0.0f;
      auto q = [&](float v) {
        float r = std::round(v * inv);
        r = std::min(std::max(r, -128.0f), 127.0f);  // Int8(clamping:)
        int qi = (int)r;
        qi = std::min(std::max(qi, -8), 7);
        return (uint8_t)(qi + 8);
      };
      packed[b * 16 + i / 2] = (uint8_t)(q(wl) | (q(wh) << 4));
    }
  }
}

void oracle_dequant_q4(const uint8_t* packed, const uint16_t* scales, size_t n_weights,
                       float* out) {
  for (size_t i = 0; i < n_weights; ++i) {
    const uint8_t b = packed[i / 2];
    const int q = (i & 1) ? (b >> 4) : (b & 0x0f);
    out[i] = (float)(q - 8) * h2f(scales[i / 32]);
  }
}

// ---------------------------------------------------------------------------
// Sampler.
//
// InferenceEngine.swift:273-368 samples with an unseeded RNG and an unstable
// sort, so the reference itself is not reproducible.  The deterministic rule
// used by both this oracle and the GPU sampler keeps the reference's steps and
// makes every order-dependent quantity exact:
//   scaled_i = logit_i / T (fp32 division); NaN logits keep 0.0 (:297,:302)
//   m = max over non-NaN scaled; all-NaN (m = -inf) -> 151645 (:311-315)
//   x_i = scaled_i - m, clamped to <= 0 (NaN -> 0)
//   e_i = sampler_exp(x_i); E_i = trunc(e_i * 2^31)  (fixed point, uint32)
//   S = sum E_i (exact integer); thr = floor(S * P24 / 2^24), P24 = trunc(top_p * 2^24)
//   order by (E desc, id asc); keep the shortest prefix with cum >= thr (:339-351)
//   R = floor(K * U24 / 2^24) with K the kept sum; return the first kept token
//   with cum > R (:353-367).
// ---------------------------------------------------------------------------

// exp(x) for the sampler: Cody-Waite range reduction (Cody & Waite, "Software
// Manual for the Elementary Functions", 1980) with the two-part ln2 split used
// by Cephes expf, then the degree-7 Taylor polynomial of e^r on |r| <= ln2/2
// (truncation error < 6e-9), Horner form with explicit fused multiply-adds.
float oracle_sampler_exp(float x) {
  if (!(x <= 0.0f)) x = 0.0f;
  if (x < -100.0f) return 0.0f;
  const float n = std::nearbyint(x * 1.44269504088896341f);
  float r = std::fma(-n, 0.693359375f, x);
  r = std::fma(-n, -2.12194440e-4f, r);
  float p = 1.0f / 5040.0f;
  p = std::fma(p, r, 1.0f / 720.0f);
  p = std::fma(p, r, 1.0f / 120.0f);
  p = std::fma(p, r, 1.0f / 24.0f);
  p = std::fma(p, r, 1.0f / 6.0f);
  p = std::fma(p, r, 0.5f);
  p = std::fma(p, r, 1.0f);
  p = std::fma(p, r, 1.0f);
  const int ni = (int)n;
  if (ni < -126) return 0.0f;
  uint32_t bits = (uint32_t)(ni + 127) << 23;
  float scale;
  std::memcpy(&scale, &bits, 4);
  return p * scale;
}

static uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint32_t oracle_uniform24(uint64_t seed, uint64_t sequence, uint64_t step) {
  const uint64_t key = splitmix64((sequence << 32) ^ step);
  return (uint32_t)(splitmix64(seed ^ key) >> 40);
}

// InferenceEngine.swift:277-294.
int oracle_sample_greedy(const uint16_t* logits, int vocab) {
  float best = -INFINITY;
  int idx = 0;
  for (int i = 0; i < vocab; ++i) {
    const float v = h2f(logits[i]);
    if (std::isnan(v)) continue;
    if (v > best) {
      best = v;
      idx = i;
    }
  }
  if (best == -INFINITY) return 151645;
  return idx;
}

static uint64_t mul_shift24(uint64_t a, uint32_t b) {
  // floor(a * b / 2^24) for a < 2^49, b <= 2^24, exactly.
  return (a >> 24) * b + (((a & 0xFFFFFFull) * b) >> 24);
}

int oracle_sample_top_p(const uint16_t* logits, int vocab, float temperature, float top_p,
                        uint32_t u24) {
  if (temperature <= 0.0f) return oracle_sample_greedy(logits, vocab);
  std::vector<float> scaled(vocab, 0.0f);
  float mx = -INFINITY;
  for (int i = 0; i < vocab; ++i) {
    const float v = h2f(logits[i]);
    if (std::isnan(v)) continue;
    scaled[i] = v / temperature;
    if (scaled[i] > mx) mx = scaled[i];
  }
  if (mx == -INFINITY) return 151645;
  std::vector<uint32_t> E(vocab);
  uint64_t S = 0;
  for (int i = 0; i < vocab; ++i) {
    const float e = oracle_sampler_exp(scaled[i] - mx);
    E[i] = (uint32_t)(e * 2147483648.0f);
    S += E[i];
  }
  const uint32_t p24 = (uint32_t)(std::min(std::max(top_p, 0.0f), 1.0f) * 16777216.0f);
  const uint64_t thr = mul_shift24(S, p24);
  std::vector<int> order(vocab);
  for (int i = 0; i < vocab; ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](int a, int b) {
    if (E[a] != E[b]) return E[a] > E[b];
    return a < b;
  });
  uint64_t cum = 0;
  int cut = vocab - 1;
  for (int i = 0; i < vocab; ++i) {
    cum += E[order[i]];
    if (cum >= thr) {
      cut = i;
      break;
    }
  }
  const uint64_t kept = cum;
  const uint64_t R = mul_shift24(kept, u24);
  uint64_t run = 0;
  for (int i = 0; i <= cut; ++i) {
    run += E[order[i]];
    if (run > R) return order[i];
  }
  return order[cut];
}

// InferenceEngine.swift:296-367 in fp32, with r = u * newSum.
int oracle_sample_reference_float(const uint16_t* logits, int vocab, float temperature,
                                  float top_p, float u) {
  if (temperature <= 0.0f) return oracle_sample_greedy(logits, vocab);
  std::vector<float> l(vocab, 0.0f);
  float mx = -INFINITY;
  for (int i = 0; i < vocab; ++i) {
    const float v = h2f(logits[i]);
    if (std::isnan(v)) continue;
    l[i] = v / temperature;
    if (l[i] > mx) mx = l[i];
  }
  if (mx == -INFINITY) return 151645;
  float sum = 0.0f;
  for (int i = 0; i < vocab; ++i) {
    l[i] = std::exp(l[i] - mx);
    sum += l[i];
  }
  for (int i = 0; i < vocab; ++i) l[i] /= sum;
  std::vector<int> order(vocab);
  for (int i = 0; i < vocab; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return l[a] > l[b]; });
  float cum = 0.0f;
  int cutoff = 0;
  for (int i = 0; i < vocab; ++i) {
    cum += l[order[i]];
    if (cum >= top_p) {
      cutoff = i;
      break;
    }
  }
  cutoff = std::max(1, cutoff + 1);
  float new_sum = 0.0f;
  for (int i = 0; i < cutoff; ++i) new_sum += l[order[i]];
  const float r = u * new_sum;
  float run = 0.0f;
  for (int i = 0; i < cutoff; ++i) {
    run += l[order[i]];
    if (r <= run) return order[i];
  }
  return order[cutoff - 1];
}

// ---------------------------------------------------------------------------
// Whole model (reference weight directory layout).
// ---------------------------------------------------------------------------
}  // extern "C"

struct OracleLayer {
  std::vector<uint16_t> in_norm, post_norm, qkv_bias, o_bias, down_bias;
  std::vector<uint8_t> q, k, v, o, gate, up, down;
  std::vector<uint16_t> qs, ks, vs, os, gs, us, ds;
};

struct oracle_model {
  int n_layers = 0;
  std::vector<uint16_t> embed, final_norm;
  std::vector<OracleLayer> layers;
};

struct oracle_state {
  int max_ctx = 0;
  std::vector<uint16_t> x, residual, q, k, v, attn_out, gate, up, mlp_out;
  std::vector<float> scores;
  std::vector<std::vector<uint16_t>> kc, vc;
};

template <class T>
static bool read_file(const std::string& path, std::vector<T>& out, size_t expect_elems) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) {
    std::fprintf(stderr, "oracle: cannot open %s\n", path.c_str());
    return false;
  }
  std::fseek(f, 0, SEEK_END);
  const long sz = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  if (sz < 0 || (size_t)sz != expect_elems * sizeof(T)) {
    std::fprintf(stderr, "oracle: %s has %ld bytes, expected %zu\n", path.c_str(), sz,
                 expect_elems * sizeof(T));
    std::fclose(f);
    return false;
  }
  out.resize(expect_elems);
  const size_t got = std::fread(out.data(), sizeof(T), expect_elems, f);
  std::fclose(f);
  return got == expect_elems;
}

extern "C" {

oracle_model* oracle_model_load(const char* dir, int n_layers) {
  auto* m = new oracle_model();
  m->n_layers = n_layers;
  const std::string d(dir);
  bool ok = read_file(d + "/global/embed_tokens.bin", m->embed, (size_t)kVocab * kHidden) &&
            read_file(d + "/global/final_norm.bin", m->final_norm, kHidden);
  m->layers.resize(n_layers);
  for (int i = 0; ok && i < n_layers; ++i) {
    const std::string p = d + "/layer" + std::to_string(i) + "/";
    OracleLayer& L = m->layers[i];
    const size_t hh = (size_t)kHidden * kHidden, kh = (size_t)kKVDim * kHidden,
                 ih = (size_t)kInter * kHidden;
    ok = read_file(p + "layer" + std::to_string(i) + "_norm.bin", L.in_norm, kHidden) &&
         read_file(p + "layer" + std::to_string(i) + "_post_attn_norm.bin", L.post_norm,
                   kHidden) &&
         read_file(p + "q_proj_4bit.bin", L.q, hh / 2) &&
         read_file(p + "q_proj_scales.bin", L.qs, hh / 32) &&
         read_file(p + "k_proj_4bit.bin", L.k, kh / 2) &&
         read_file(p + "k_proj_scales.bin", L.ks, kh / 32) &&
         read_file(p + "v_proj_4bit.bin", L.v, kh / 2) &&
         read_file(p + "v_proj_scales.bin", L.vs, kh / 32) &&
         read_file(p + "o_proj_4bit.bin", L.o, hh / 2) &&
         read_file(p + "o_proj_scales.bin", L.os, hh / 32) &&
         read_file(p + "gate_proj_4bit.bin", L.gate, ih / 2) &&
         read_file(p + "gate_proj_scales.bin", L.gs, ih / 32) &&
         read_file(p + "up_proj_4bit.bin", L.up, ih / 2) &&
         read_file(p + "up_proj_scales.bin", L.us, ih / 32) &&
         read_file(p + "down_proj_4bit.bin", L.down, ih / 2) &&
         read_file(p + "down_proj_scales.bin", L.ds, ih / 32) &&
         read_file(p + "qkv_bias.bin", L.qkv_bias, kHidden + 2 * kKVDim) &&
         read_file(p + "o_bias.bin", L.o_bias, kHidden) &&
         read_file(p + "mlp_down_bias.bin", L.down_bias, kHidden);
  }
  if (!ok) {
    delete m;
    return nullptr;
  }
  return m;
}

static void fill_normal_f32(std::vector<float>& v, uint64_t seed, float mean, float sd) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)v.size(); i += 2) {
    const uint64_t r = splitmix64(seed ^ splitmix64((uint64_t)i));
    const float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)((r >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
    const float rad = std::sqrt(-2.0f * std::log(u1));
    v[i] = mean + sd * rad * std::cos(6.2831853f * u2);
    if (i + 1 < (long long)v.size()) v[i + 1] = mean + sd * rad * std::sin(6.2831853f * u2);
  }
}

oracle_model* oracle_model_random(int n_layers, uint64_t seed) {
  auto* m = new oracle_model();
  m->n_layers = n_layers;
  uint64_t sid = seed * 1000003ull;
  auto f16 = [&](std::vector<uint16_t>& dst, size_t n, float mean, float sd) {
    std::vector<float> tmp(n);
    fill_normal_f32(tmp, ++sid, mean, sd);
    dst.resize(n);
    for (size_t i = 0; i < n; ++i) dst[i] = f2h(tmp[i]);
  };
  auto q4 = [&](std::vector<uint8_t>& p, std::vector<uint16_t>& s, size_t rows, size_t k) {
    std::vector<float> tmp(rows * k);
    fill_normal_f32(tmp, ++sid, 0.0f, 0.02f);
    p.resize(rows * k / 2);
    s.resize(rows * k / 32);
    oracle_quantize_q4(tmp.data(), tmp.size(), p.data(), s.data());
  };
  f16(m->embed, (size_t)kVocab * kHidden, 0.0f, 0.02f);
  f16(m->final_norm, kHidden, 1.0f, 0.02f);
  m->layers.resize(n_layers);
  for (auto& L : m->layers) {
    f16(L.in_norm, kHidden, 1.0f, 0.02f);
    f16(L.post_norm, kHidden, 1.0f, 0.02f);
    q4(L.q, L.qs, kHidden, kHidden);
    q4(L.k, L.ks, kKVDim, kHidden);
    q4(L.v, L.vs, kKVDim, kHidden);
    q4(L.o, L.os, kHidden, kHidden);
    q4(L.gate, L.gs, kInter, kHidden);
    q4(L.up, L.us, kInter, kHidden);
    q4(L.down, L.ds, kHidden, kInter);
    f16(L.qkv_bias, kHidden + 2 * kKVDim, 0.0f, 0.02f);
    L.o_bias.assign(kHidden, 0);
    L.down_bias.assign(kHidden, 0);
  }
  return m;
}

void oracle_model_free(oracle_model* m) { delete m; }

oracle_state* oracle_state_create(const oracle_model* m, int max_ctx) {
  auto* s = new oracle_state();
  s->max_ctx = max_ctx;
  s->x.assign(kHidden, 0);
  s->residual.assign(kHidden, 0);
  s->q.assign(kHidden, 0);
  s->k.assign(kKVDim, 0);
  s->v.assign(kKVDim, 0);
  s->attn_out.assign(kHidden, 0);
  s->gate.assign(kInter, 0);
  s->up.assign(kInter, 0);
  s->mlp_out.assign(kHidden, 0);
  s->scores.assign((size_t)kHeads * max_ctx, 0.0f);
  s->kc.assign(m->n_layers, std::vector<uint16_t>((size_t)max_ctx * kKVDim, 0));
  s->vc.assign(m->n_layers, std::vector<uint16_t>((size_t)max_ctx * kKVDim, 0));
  return s;
}

void oracle_state_free(oracle_state* s) { delete s; }
uint16_t* oracle_state_k_cache(oracle_state* s, int layer) { return s->kc[layer].data(); }
uint16_t* oracle_state_v_cache(oracle_state* s, int layer) { return s->vc[layer].data(); }
const uint16_t* oracle_state_x(const oracle_state* s) { return s->x.data(); }

// InferenceEngine.swift:54-268.
void oracle_forward(const oracle_model* m, oracle_state* s, int token, int position,
                    uint16_t* logits) {
  const int safe_pos = std::min(position, s->max_ctx - 1);        // :55
  std::memcpy(s->x.data(), m->embed.data() + (size_t)token * kHidden, kHidden * 2);  // :57-60
  const uint32_t seq_len = (uint32_t)safe_pos + 1;                 // :66-67
  for (int i = 0; i < m->n_layers; ++i) {
    const OracleLayer& L = m->layers[i];
    oracle_rms_norm(s->x.data(), L.in_norm.data(), s->residual.data(), kNormThreads);  // :107-111
    oracle_gemv_q4_0(L.q.data(), L.qs.data(), s->residual.data(), s->q.data(),
                     L.qkv_bias.data(), kHidden, kHidden, kGemvThreads);              // :116-122
    oracle_gemv_q4_0(L.k.data(), L.ks.data(), s->residual.data(), s->k.data(),
                     L.qkv_bias.data() + kHidden, kKVDim, kHidden, kGemvThreads);     // :124-130
    oracle_gemv_q4_0(L.v.data(), L.vs.data(), s->residual.data(), s->v.data(),
                     L.qkv_bias.data() + kHidden + kKVDim, kKVDim, kHidden, kGemvThreads);
    oracle_rope(s->q.data(), kHeads, seq_len);                                        // :141-144
    oracle_rope(s->k.data(), 2, seq_len);                                             // :146-148
    oracle_write_kv_cache(s->k.data(), s->v.data(), s->kc[i].data(), s->vc[i].data(),
                          seq_len);                                                   // :154-160
    oracle_attention(s->q.data(), s->kc[i].data(), s->vc[i].data(), s->attn_out.data(),
                     seq_len, s->scores.data());                                      // :163-182
    oracle_gemv_q4_0(L.o.data(), L.os.data(), s->attn_out.data(), s->q.data(),
                     L.o_bias.data(), kHidden, kHidden, kGemvThreads);                // :185-192
    oracle_residual_add(s->x.data(), s->q.data(), s->x.data(), kHidden);              // :195-199
    oracle_rms_norm(s->x.data(), L.post_norm.data(), s->residual.data(), kNormThreads);
    static const std::vector<uint16_t> zero_bias(kInter, 0);                          // :82-85
    oracle_gemv_q4_0(L.gate.data(), L.gs.data(), s->residual.data(), s->gate.data(),
                     zero_bias.data(), kInter, kHidden, kGemvThreads);                // :209-216
    oracle_gemv_q4_0(L.up.data(), L.us.data(), s->residual.data(), s->up.data(),
                     zero_bias.data(), kInter, kHidden, kGemvThreads);                // :218-224
    oracle_swiglu(s->gate.data(), s->up.data(), kInter);                              // :227-230
    oracle_gemv_q4_0(L.down.data(), L.ds.data(), s->gate.data(), s->mlp_out.data(),
                     L.down_bias.data(), kHidden, kInter, kGemvThreads);              // :233-240
    oracle_residual_add(s->x.data(), s->mlp_out.data(), s->x.data(), kHidden);        // :243-247
  }
  if (logits) {
    oracle_rms_norm(s->x.data(), m->final_norm.data(), s->residual.data(), kNormThreads);  // :252-256
    oracle_gemv_fp16(m->embed.data(), s->residual.data(), logits, kVocab, kHidden,
                     kGemvThreads);                                                   // :259-264
  }
}

int oracle_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
}

}  // extern "C"
