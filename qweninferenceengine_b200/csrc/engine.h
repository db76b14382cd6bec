// engine.h -- host-side engine classes of libqwen_b200.so.
//
// Mirrors the reference's Swift surface:
//   WeightLoader      WeightLoader.swift:16-53   (reference .bin directory layout)
//   QwenLayer         QwenLayer.swift:9-53       (19 buffers per layer)
//   QwenModel         QwenModel.swift:11-35      (embeddings, final norm, tied LM head)
//   InferenceManager  InferenceManager.swift:11-77 (activations, KV cache, logits)
//   QwenEngine        InferenceEngine.swift:9-369 (forward / generate / sampling)
// Every method returns a QWEN_* status instead of throwing or exiting.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/qwen_b200.h"
#include "qwen_internal.h"

namespace qwen {

// WeightLoader.swift:26-52: reads `<dir>/<relative path>`; a missing file is
// QWEN_ERR_FILE_NOT_FOUND (WeightLoadingError.fileNotFound), a file of the
// wrong size is QWEN_ERR_BAD_WEIGHT_FILE.
class WeightLoader {
 public:
  explicit WeightLoader(std::string dir) : dir_(std::move(dir)) {}
  int load_buffer(const std::string& relative_path, size_t expect_bytes, void* device_dst,
                  cudaStream_t st, std::vector<uint8_t>& staging) const;
  int load_layer_weight(int layer, const std::string& name, size_t expect_bytes, void* device_dst,
                        cudaStream_t st, std::vector<uint8_t>& staging) const {
    return load_buffer("layer" + std::to_string(layer) + "/" + name + ".bin", expect_bytes,
                       device_dst, st, staging);
  }

 private:
  std::string dir_;
};

// One Q4 linear in the reference layout: packed [rows][k/2], scales [rows][k/32].
struct Q4Linear {
  uint8_t* packed = nullptr;
  __half* scales = nullptr;
  int rows = 0, k = 0;
  size_t packed_bytes() const { return (size_t)rows * k / 2; }
  size_t scale_bytes() const { return (size_t)rows * (k / 32) * 2; }
};

// QwenLayer.swift:9-53.
struct QwenLayer {
  __half* input_norm = nullptr;
  __half* post_attn_norm = nullptr;
  Q4Linear q, k, v, o, gate, up, down;
  __half* qkv_bias = nullptr;   // q | k | v biases, 2048 (QwenPipelines.swift:177-181)
  __half* o_bias = nullptr;     // zeros for Qwen2.5 (QwenPipelines.swift:184)
  __half* down_bias = nullptr;  // zeros for Qwen2.5 (QwenPipelines.swift:194)
};

// Weights in the layouts the fused decode kernels stream (built from the
// reference layout on the device; see layout.cu).
struct FusedWeights {
  uint8_t* blob = nullptr;          // Q4 tiles of every layer, fragment order (fused.h)
  size_t blob_bytes = 0;
  uint8_t* lm_tiles = nullptr;      // fp16 LM head in mma tile order
  __half* norms = nullptr;          // [layer][2][1536] + final [1536]
  __half* qkv_bias = nullptr;       // [layer][2048]
  __half* o_bias = nullptr;         // [layer][1536]
  __half* down_bias = nullptr;      // [layer][1536]
  float* rope_cs = nullptr;         // [rope_ctx][64][2] cos, sin
  int rope_ctx = 0;
  unsigned long long* items = nullptr;  // per-CTA work lists (packed items, fused.h)
  uint32_t* item_begin = nullptr;   // [grid + 1]
  int grid = 0;
  void release();
};

// Weights of the tensor-core batched step (tc_gemm.h blob layouts): per layer
// the QKV (q, k, v rows concatenated: 16 tiles), O (12), gate/up (gate rows
// then up rows: 140) and down (12) Q4 blobs back to back, and the fp16 LM head.
struct TcWeights {
  uint8_t* blob = nullptr;
  size_t layer_bytes = 0;
  uint8_t* lm = nullptr;
  float* rope_cs = nullptr;         // [rope_ctx][64][2] cos, sin
  int rope_ctx = 0;
  void release();
};

// QwenModel.swift:11-35.
class QwenModel {
 public:
  ~QwenModel();
  int allocate(int n_layers);
  int load(const std::string& weights_dir, cudaStream_t st);
  int init_random(uint64_t seed, cudaStream_t st);
  int build_fused(int max_ctx, cudaStream_t st);

  int n_layers = 0;
  std::vector<QwenLayer> layers;
  __half* embed = nullptr;       // [151936][1536]; also the tied LM head (QwenModel.swift:27)
  __half* final_norm = nullptr;
  __half* zero_bias = nullptr;   // the zero bias buffer of InferenceEngine.swift:82-85
  FusedWeights fused;
  TcWeights tc;
  bool loaded = false;

 private:
  void* dev_alloc(size_t bytes, int* rc);
  std::vector<void*> allocs_;
};

// Device control block of one sequence; updated on the device so a step can be
// replayed from a CUDA graph without host work.
struct SeqCtl {
  int32_t pos;         // position the next step processes
  int32_t n_prompt;    // prompt tokens (positions < n_prompt read prompt[pos])
  int32_t last_token;  // last sampled id
  uint32_t seq_len;    // min(pos, max_ctx-1) + 1 for the running step
  int32_t token;       // token of the running step
  int32_t n_out;       // generated ids recorded so far
  int32_t done;        // a stop token was sampled (stop_on_eos)
  uint32_t u24;        // uniform of the running step
};

// InferenceManager.swift:11-77, per sequence of the batch.
class InferenceManager {
 public:
  ~InferenceManager();
  int allocate(int batch, int n_layers, int max_ctx, int max_out);

  int batch = 0, n_layers = 0, max_ctx = 0, max_out = 0;
  __half *x = nullptr, *residual = nullptr, *q = nullptr, *k = nullptr, *v = nullptr;
  __half *attn_out = nullptr, *gate = nullptr, *up = nullptr, *mlp_out = nullptr;
  __half* logits = nullptr;      // [batch][151936] (the reference sizes 151666; all rows are written)
  float* scores = nullptr;       // [12][max_ctx] (ops mode)
  __half *kc = nullptr, *vc = nullptr;  // [layer][batch][max_ctx][256]
  SeqCtl* ctl = nullptr;         // [batch]
  int32_t* prompt = nullptr;     // [batch][max_ctx]
  int32_t* out_tokens = nullptr; // [batch][max_out]
  int32_t* sampled = nullptr;    // [batch]
  uint32_t* u24_ = nullptr;      // [batch] uniforms of the running step
  int* err = nullptr;            // device error word
  uint32_t* epoch = nullptr;     // step counter (tags of the fused step's exchanges)
  unsigned long long* trace = nullptr;  // optional fused-step phase stamps
  void* attn_scratch = nullptr;
  int attn_splits = 0;
  void* samp_scratch = nullptr;  // batch-1 grid sampler's exchanges (zero between launches)
  size_t samp_scratch_bytes = 0;
  void* fused_scratch = nullptr;
  size_t fused_scratch_bytes = 0;
  // tensor-core batched step (tc_gemm.h layouts)
  uint8_t* act_h = nullptr;      // activation tiles, k = 1536
  uint8_t* act_i = nullptr;      // activation tiles, k = 8960
  float* tc_part = nullptr;      // fp32 split-K partials
  int tc_rows = 0;               // activation rows the buffers hold
  int tc_nb = 0;                 // tc_rows padded to 16
  // chunked prefill (rows = (sequence, position) pairs of a chunk)
  __half *tc_px = nullptr, *tc_pq = nullptr;  // [tc_rows][1536]
  __half* tc_plogits = nullptr;  // [tc_rows][151936]
  uint32_t* tc_row_len = nullptr;  // [tc_rows] position + 1 of each row
  int32_t* tc_row_seq = nullptr;   // [tc_rows] KV sequence of each row
  void* tc_pattn = nullptr;      // attention scratch for tc_rows rows
  int tc_psplits = 0;

  // cudaMalloc + zero, freed with the state.
  int alloc_tracked(size_t bytes, void** out);

  size_t kv_layer_stride() const { return (size_t)batch * max_ctx * 256; }
  size_t kv_seq_stride() const { return (size_t)max_ctx * 256; }

 private:
  std::vector<void*> allocs_;
};

// QwenEngine, InferenceEngine.swift:9-369.
class QwenEngine {
 public:
  ~QwenEngine();
  int init(const qwen_engine_config& cfg);
  int load_weights(const std::string& dir);
  int init_random(uint64_t seed);
  int reset();
  int forward(int32_t token, int32_t position, int32_t* next_token);
  int prefill(const int32_t* prompt_ids, int32_t n_prompt);
  int decode(int32_t n_steps, int32_t* out_ids);
  int generate(const int32_t* prompt_ids, int32_t n_prompt, int32_t max_tokens, int32_t* out_ids,
               int32_t* n_out);
  int get_logits(int32_t seq, uint16_t* host);
  int get_kv(int32_t seq, int32_t layer, int32_t n_pos, uint16_t* hk, uint16_t* hv);
  int set_kv(int32_t seq, int32_t layer, int32_t n_pos, const uint16_t* hk, const uint16_t* hv);
  int position(int32_t seq, int32_t* pos);
  int kernels_per_step(int* n) const;
  int set_trace(int enable);
  int get_trace(unsigned long long* host, size_t n, size_t* needed);
  int time_steps(int n, float* ms_step, float* ms_model);
  int profile_step(float* ms, int cap, int* n);
  int set_wait_timeout(uint64_t ns);
  int test_stall(int site);
  cudaStream_t stream() const { return stream_; }

 private:
  int ensure_graph();
  int run_steps(int n);
  int check_device_error();
  // ev (optional, outside capture): events recorded at step start, model
  // start, model end, step end.
  int enqueue_step_ops(cudaEvent_t* ev);
  int enqueue_step_fused(cudaEvent_t* ev);
  int enqueue_step_tc(cudaEvent_t* ev);
  int prefill_chunked(const int32_t* prompt_ids, int32_t n_prompt);
  int enqueue_step(cudaEvent_t* ev);
  int build_step_weights();
  bool uses_tc_layout() const;
  int upload_prompt(const int32_t* prompt_ids, int32_t n_prompt, int32_t start_pos);

  qwen_engine_config cfg_{};
  QwenModel model_;
  InferenceManager state_;
  cudaStream_t stream_ = nullptr;
  cudaGraphExec_t graph_exec_ = nullptr;
  cudaGraph_t graph_ = nullptr;
  bool initialised_ = false;
  int sm_count_ = 0;
  uint64_t wait_ns_ = 2000000000ull;  // device wait limit of the fused step
  int stall_site_ = 0;                // test hook of the fused step
  void drop_graph();
  struct HostStaging {
    int32_t token;
    SeqCtl ctl;
    int32_t result;
    int32_t err;
  };
  HostStaging* pinned_ = nullptr;  // pinned host buffers for forward()
};

// Fused decode step (decode_fused.cu).
struct FusedStepArgs {
  const QwenModel* model;
  InferenceManager* state;
  int n_layers;
  int sm_count;
  unsigned long long wait_ns;  // device wait limit
  int stall_site;              // test hook (0: none)
};
// Wait site of the fused step's poll for the down partial sums, for the
// stall test hook.
constexpr int kFusedStallDownPart = 9;
// Stall hook site of the batch-1 grid sampler's first exchange barrier.
constexpr int kSamplerStallSite = 20;
int fused_scratch_bytes(int batch, int max_ctx, int sm_count, size_t* bytes);
int enqueue_fused_step(const FusedStepArgs& a, cudaStream_t st);
int build_fused_weights(QwenModel& m, int max_ctx, cudaStream_t st);
int upload_rope_table(float** cs_dev, int* ctx, int max_ctx, cudaStream_t st);

// Tensor-core batched step (batched.cu): weights, state, and the model part of
// one step over a set of activation rows (x -> logits).
int build_tc_weights(QwenModel& m, int max_ctx, cudaStream_t st);
int tc_state_allocate(InferenceManager& s, int sm_count);
// The rows one launch of the model processes: the batch's sequences (decode),
// or consecutive positions of one sequence (chunked prefill).
struct TcRows {
  int rows;
  __half* x;                 // [rows][1536] inputs (embeddings), residual stream
  __half* q;                 // [rows][1536] scratch for the rotated queries
  const uint32_t* seq_len;   // row r: position + 1 at seq_len[r * seq_len_stride]
  int seq_len_stride;
  const int32_t* row_seq;    // KV sequence of each row; nullptr: row = sequence
  void* attn_scratch;
  int attn_splits;
  __half* logits;            // [rows][151936]; nullptr: no LM head
};
TcRows tc_decode_rows(InferenceManager& s);
// marks (optional): an event is recorded after every launch, (*n_marks)++.
int enqueue_tc_model(QwenModel& m, InferenceManager& s, const TcRows& v, int sm_count,
                     cudaStream_t st, cudaEvent_t* marks = nullptr, int* n_marks = nullptr);
// Rows for positions p0 .. p0+n_pos-1 of every sequence of the batch (row
// b * n_pos + j: sequence b, position p0 + j): embeddings of the prompt ids,
// lengths and KV sequences, on the device.
int launch_prefill_rows(InferenceManager& s, const __half* embed, int p0, int n_pos,
                        cudaStream_t st);
int tc_kernels_per_step(int n_layers);
constexpr int kTcPrefillRows = 128;  // positions per chunk of a batch-1 prefill

}  // namespace qwen
