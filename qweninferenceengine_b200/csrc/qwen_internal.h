// qwen_internal.h -- declarations shared by the CUDA translation units and the
// C++ host engine of libqwen_b200.so (not installed; include/qwen_b200.h is
// the public ABI).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <mutex>

namespace qwen {

// ------------------------------------------------- __device__ symbols ----
// Per-device cache of a __device__ symbol's address, keyed on the CUDA
// context it was looked up in (a reset device gets a new lookup).
struct DeviceSymbolCache {
  static constexpr int kMaxDevices = 64;
  std::mutex mu;
  void* ctx[kMaxDevices] = {};
  void* addr[kMaxDevices] = {};
};
// lookup: cudaGetSymbolAddress of the symbol, called in the symbol's own file.
int symbol_address_cached(DeviceSymbolCache& cache, int (*lookup)(void**), void** out);
// Device address of the operator status word (ops_status.cu) on the current
// device: int[4], [0] the first DeviceError recorded by an operator kernel.
int ops_status_word(int** out);

// ---------------------------------------------------------- attention ----
struct AttnParams {
  const __half* q;          // [n_seq][12][128] (after RoPE)
  long long q_seq_stride;   // elements between sequences
  const __half* k;          // cache bases (element (seq,pos,head,d) at
  const __half* v;          //   seq*kv_seq_stride + pos*kv_pos_stride + head*kv_head_stride + d)
  long long kv_seq_stride, kv_pos_stride, kv_head_stride;
  const uint32_t* seq_len;  // L per sequence (device)
  int seq_len_stride;       // uint32 elements between sequences' L
  uint32_t max_ctx;         // L must be in [1, max_ctx]
  __half* out;              // [n_seq][1536]
  long long out_seq_stride;
  uint8_t* act_out;         // if set: the output goes here instead, in the
  int act_nb;               //   tensor-core activation tile layout of act_nb rows
  const int32_t* row_seq;   // if set: KV sequence of each row (rows = positions of
                            //   one sequence in a chunked prefill); else row = sequence
  int kv_n_seq;             // sequences in the caches (0: as many as rows)
  float* part_o;            // scratch: [n_seq][2][max_splits][6][128]
  float* part_ml;           // scratch: [n_seq][2][max_splits][6][2]
  uint32_t* counters;       // scratch: [n_seq][2], zero between launches
  int* err;                 // device error word (may be null)
  // Decode steps of the batched engine: q and the step's new k / v rows are
  // formed here from the QKV projection's split-K partial sums (split order,
  // + bias, fp16 rounding, RoPE at position seq_len - 1) instead of by a finish
  // kernel: q never leaves the CTA, the new rows are patched into the tile
  // that holds that position and appended to the caches by the unit that owns
  // it.  qkv_part = null: q comes from `q` and the caches already hold the row.
  const float* qkv_part;    // [splits][rows][2048] fp32
  int qkv_splits;
  int qkv_rows;             // rows of each split's block (the GEMM's batch)
  const __half* qkv_bias;   // [2048] this layer's q | k | v biases
  const float* rope_cs;     // [max_ctx][64][2] cos / sin
};
int attn_max_splits(int max_ctx, int n_seq);
size_t attn_scratch_bytes(int max_splits, int n_seq);
void attn_bind_scratch(AttnParams& p, void* scratch, int max_splits, int n_seq);
// pdl: launch as a programmatic dependent of the previous kernel in the stream.
// Returns 0, or -1 for unsupported strides / split counts or a launch failure.
int launch_attention_decode(const AttnParams& p, int max_splits, int n_seq, cudaStream_t st,
                            bool pdl = false);

// ------------------------------------------------------- op launchers ----
int launch_gemv_q4_rowmajor(const uint8_t* packed, const __half* scales, const __half* x,
                            __half* y, const __half* bias, int n_rows, int k, void* stream);
int launch_gemv_fp16_rowmajor(const __half* w, const __half* x, __half* y, int n_rows, int k,
                              void* stream);
int launch_rms_norm(const __half* x, const __half* gamma, __half* out, void* stream);
int set_rope_inv_freq(const float* inv_freq64);
int launch_rope(__half* vec, int n_heads, const uint32_t* seq_len, void* stream);
int launch_write_kv_cache(const __half* k, const __half* v, __half* kc, __half* vc,
                          const uint32_t* seq_len, uint32_t max_ctx, void* stream);
int launch_attention_scores(const __half* q, const __half* kc, float* scores,
                            const uint32_t* seq_len, uint32_t max_seq, void* stream);
int launch_softmax(float* scores, const uint32_t* seq_len, void* stream);
int launch_attn_weighted_sum(const float* scores, const __half* vc, __half* out,
                             const uint32_t* seq_len, void* stream);
int launch_residual_add(const __half* a, const __half* b, __half* out, int n, void* stream);
int launch_swiglu(__half* gate, const __half* up, int n, void* stream);
int launch_dequant_q4(const uint8_t* packed, const __half* scales, size_t n_weights, float* out,
                      void* stream);

// ------------------------------------------------------------ sampler ----
// Deterministic sampler (greedy when temperature <= 0).  scratch: see
// sampler_scratch_bytes.
size_t sampler_scratch_bytes(int n_seq);
// Host set-up of the sampler for the current device (cluster-size query); call
// before capturing a launch_sample into a CUDA graph.
void sampler_prepare();
// wait_ns bounds the grid path's barrier waits; stall: test hook (CTA 0
// skips one arrival so that the others' waits run out).
int launch_sample(const __half* logits, int n_seq, int row_stride, int vocab, float temperature,
                  float top_p, const uint32_t* u24, int32_t* out_ids, void* scratch,
                  int* err, cudaStream_t st, unsigned long long wait_ns = 2000000000ull,
                  int stall = 0);

// ------------------------------------------------------ weight helpers ----
int launch_quantize_q4(const float* w, size_t n, uint8_t* packed, __half* scales,
                       cudaStream_t st);
// Fills n floats with N(0,1)*stddev + mean from (seed, stream id).
int launch_fill_normal(float* out, size_t n, uint64_t seed, uint64_t stream_id, float mean,
                       float stddev, cudaStream_t st);
int launch_f32_to_f16(const float* in, __half* out, size_t n, cudaStream_t st);

// Host-side helpers.
uint64_t splitmix64(uint64_t z);
uint32_t uniform24(uint64_t seed, uint64_t sequence, uint64_t step);
void rope_inv_freq(float* inv_freq64);

}  // namespace qwen
