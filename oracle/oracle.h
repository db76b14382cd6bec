/*
 * oracle.h -- CPU oracle for the Qwen2.5-1.5B Q4 decode step.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm load it.
 * The product (qweninferenceengine_b200, libqwen_b200.so) never links, loads or
 * calls anything in this directory.
 *
 * It is a scalar C++ restatement of the reference engine's arithmetic,
 * written to reproduce the reference's rounding points and summation order:
 *
 *   kernels/matmul.metal:9-73      gemv_q4_0        -> oracle_gemv_q4_0
 *   kernels/matmul.metal:75-113    gemv_fp16        -> oracle_gemv_fp16
 *   kernels/rmsnorm.metal:9-46     rms_norm_q4      -> oracle_rms_norm
 *   kernels/rope.metal:12-39       apply_rope_q4    -> oracle_rope
 *   kernels/attention.metal:67-84  write_kv_cache   -> oracle_write_kv_cache
 *   kernels/attention.metal:9-32   attention_scores -> oracle_attention (scores)
 *   kernels/activations.metal:29-55 softmax         -> oracle_attention (softmax)
 *   kernels/attention.metal:34-56  attn_weighted_sum-> oracle_attention (sum)
 *   kernels/attention.metal:58-65  residual_add     -> oracle_residual_add
 *   kernels/activations.metal:9-27 swiglu           -> oracle_swiglu
 *   QwenPipelines.swift:97-145     packAndSave4Bit  -> oracle_quantize_q4
 *   InferenceEngine.swift:54-271   forward          -> oracle_forward
 *   InferenceEngine.swift:273-368  extractNextTokenID -> oracle_sample_*
 *
 * Parity is pinned by compiling the reference's own kernels/ *.metal sources as
 * C++ through oracle/metal_shim (oracle/_ref/, built by oracle/Makefile) and
 * comparing bit for bit (tests/test_oracle_pin.py).
 *
 * fp16 values cross this interface as uint16_t bit patterns.
 */
#ifndef QWEN_ORACLE_H
#define QWEN_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- kernels (one call = one reference dispatch) ------------------------ */
void oracle_gemv_q4_0(const uint8_t* packed, const uint16_t* scales, const uint16_t* x,
                      uint16_t* y, const uint16_t* bias, int n_rows, int k, int threads);
void oracle_gemv_fp16(const uint16_t* w, const uint16_t* x, uint16_t* y, int n_rows, int k,
                      int threads);
void oracle_rms_norm(const uint16_t* x, const uint16_t* gamma, uint16_t* out, int threads);
void oracle_rope(uint16_t* vec, int n_heads, uint32_t seq_len);
void oracle_write_kv_cache(const uint16_t* k, const uint16_t* v, uint16_t* k_cache,
                           uint16_t* v_cache, uint32_t seq_len);
/* scores: fp32 scratch of 12*seq_len floats (the reference's state.scores) */
void oracle_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                      uint16_t* out, uint32_t seq_len, float* scores);
void oracle_residual_add(const uint16_t* x, const uint16_t* y, uint16_t* out, int n);
void oracle_swiglu(uint16_t* gate, const uint16_t* up, int n);

/* ---- offline quantizer: QwenPipelines.swift:97-145 --------------------- */
void oracle_quantize_q4(const float* w, size_t n, uint8_t* packed, uint16_t* scales);
/* (q-8)*scale for every nibble, low nibble first (matmul.metal:37-42) */
void oracle_dequant_q4(const uint8_t* packed, const uint16_t* scales, size_t n_weights,
                       float* out);

/* ---- sampler ------------------------------------------------------------ */
/* Greedy branch, InferenceEngine.swift:277-294. */
int oracle_sample_greedy(const uint16_t* logits, int vocab);
/* Deterministic top-p sampler (fixed-point nucleus, see oracle.cpp). */
int oracle_sample_top_p(const uint16_t* logits, int vocab, float temperature, float top_p,
                        uint32_t u24);
/* Float restatement of InferenceEngine.swift:296-367 with a given uniform u in [0,1)
 * and ties broken by ascending id (the Swift sort is unstable). */
int oracle_sample_reference_float(const uint16_t* logits, int vocab, float temperature,
                                  float top_p, float u);
/* The oracle's own exp for the sampler (Cody-Waite + Taylor, see oracle.cpp). */
float oracle_sampler_exp(float x);
/* 24-bit uniform for (seed, sequence, step) -- SplitMix64 (Steele et al. 2014). */
uint32_t oracle_uniform24(uint64_t seed, uint64_t sequence, uint64_t step);

/* OpenMP threads for the row/head loops (n < 1: leave the runtime's default);
 * returns the thread count now in effect. */
int oracle_set_threads(int n);

/* ---- whole model -------------------------------------------------------- */
typedef struct oracle_model oracle_model;
typedef struct oracle_state oracle_state;

/* Loads the reference weight directory layout (WeightLoader.swift:49-52,
 * QwenLayer.swift:31-51, QwenModel.swift:25-27). Returns NULL on error. */
oracle_model* oracle_model_load(const char* dir, int n_layers);
/* Random-init model in memory (same distributions as the test fixtures, own
 * generator) for timing the CPU baseline without writing weight files. */
oracle_model* oracle_model_random(int n_layers, uint64_t seed);
void oracle_model_free(oracle_model* m);
oracle_state* oracle_state_create(const oracle_model* m, int max_ctx);
void oracle_state_free(oracle_state* s);
/* One forward(tokenID:position:), InferenceEngine.swift:54-268.  Writes the
 * 151936 fp16 logits if logits != NULL (skips the LM head when NULL). */
void oracle_forward(const oracle_model* m, oracle_state* s, int token, int position,
                    uint16_t* logits);
/* KV-cache access for teacher-forced checks: [max_ctx][256] fp16 per layer. */
uint16_t* oracle_state_k_cache(oracle_state* s, int layer);
uint16_t* oracle_state_v_cache(oracle_state* s, int layer);
/* Final hidden state x (1536 fp16) after the last forward. */
const uint16_t* oracle_state_x(const oracle_state* s);

#ifdef __cplusplus
}
#endif
#endif
