// ref_metal.cpp -- launches the reference's own Metal kernels, compiled as C++
// through oracle/metal_shim, on the CPU (test infrastructure: builds
// oracle/_ref/libqwen_metal_ref.so; see oracle/Makefile).
//
// The kernel sources are included by name from the reference tree
// (kernels/matmul.metal, rmsnorm.metal, rope.metal, attention.metal,
// activations.metal); nothing from them is copied here.  Each launcher
// reproduces the dispatch the reference encodes in InferenceEngine.swift.
#include <metal_stdlib>

#include "matmul.metal"
#include "rmsnorm.metal"
#include "rope.metal"
#include "attention.metal"
#include "activations.metal"

#include <cstring>

namespace {
inline half* H(uint16_t* p) { return reinterpret_cast<half*>(p); }
inline const half* H(const uint16_t* p) { return reinterpret_cast<const half*>(p); }
}  // namespace

extern "C" {

// InferenceEngine.swift:113-122 etc.: gemv_q4_0 with constants [K, threads/32, threads].
void ref_gemv_q4_0(const uint8_t* packed, const uint16_t* scales, const uint16_t* x,
                   uint16_t* y, const uint16_t* bias, int n_rows, int k, int threads) {
  const uint constants[3] = {(uint)k, (uint)threads / 32, (uint)threads};
#pragma omp parallel for schedule(dynamic, 4)
  for (int row = 0; row < n_rows; ++row) {
    std::function<void(uint)> body = [&](uint tid) {
      gemv_q4_0(packed, H(scales), H(x), H(y), constants, H(bias), tid, (uint)row);
    };
    metal_shim::run_threadgroup(threads, body);
  }
}

// InferenceEngine.swift:259-264.
void ref_gemv_fp16(const uint16_t* w, const uint16_t* x, uint16_t* y, int n_rows, int k,
                   int threads) {
  const uint constants[3] = {(uint)k, (uint)threads / 32, (uint)threads};
#pragma omp parallel for schedule(dynamic, 4)
  for (int row = 0; row < n_rows; ++row) {
    std::function<void(uint)> body = [&](uint tid) {
      gemv_fp16(H(w), H(x), H(y), constants, tid, (uint)row);
    };
    metal_shim::run_threadgroup(threads, body);
  }
}

// InferenceEngine.swift:91-111: one threadgroup of 256 threads.
void ref_rms_norm(const uint16_t* x, const uint16_t* gamma, uint16_t* out, int threads) {
  std::function<void(uint)> body = [&](uint tid) {
    rms_norm_q4(H(x), H(gamma), H(out), tid, (uint)threads);
  };
  metal_shim::run_threadgroup(threads, body);
}

// InferenceEngine.swift:141-148: one thread per rotated pair.
void ref_rope(uint16_t* vec, int n_heads, uint32_t seq_len) {
  const uint sl = seq_len;
  for (int tid = 0; tid < n_heads * 64; ++tid) apply_rope_q4(H(vec), &sl, (uint)tid);
}

void ref_write_kv_cache(const uint16_t* k, const uint16_t* v, uint16_t* k_cache,
                        uint16_t* v_cache, uint32_t seq_len) {
  const uint sl = seq_len;
  for (int tid = 0; tid < 256; ++tid)
    write_kv_cache(H(k), H(v), H(k_cache), H(v_cache), &sl, (uint)tid);
}

// InferenceEngine.swift:162-182: scores (12 threads), softmax (12), sum (1536).
void ref_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                   uint16_t* out, uint32_t seq_len, float* scores) {
  const uint sl = seq_len;
  for (int t = 0; t < 12; ++t) attention_scores(H(q), H(k_cache), scores, &sl, (uint)t);
  for (int t = 0; t < 12; ++t) softmax(scores, &sl, (uint)t);
  for (int t = 0; t < 1536; ++t) attn_weighted_sum(scores, H(v_cache), H(out), &sl, (uint)t);
}

void ref_residual_add(const uint16_t* x, const uint16_t* y, uint16_t* out, int n) {
  for (int t = 0; t < n; ++t) residual_add(H(x), H(y), H(out), (uint)t);
}

void ref_swiglu(uint16_t* gate, const uint16_t* up, int n) {
  for (int t = 0; t < n; ++t) swiglu(H(gate), H(up), (uint)t);
}

}  // extern "C"
