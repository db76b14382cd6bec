// engine.cu -- QwenEngine / QwenModel / WeightLoader / InferenceManager and
// the engine half of the C ABI.
#include <sys/stat.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "engine.h"
#include "fused.h"
#include "qwen_common.cuh"
#include "status.h"

namespace qwen {

// ------------------------------------------------------------ step kernels --
__device__ __forceinline__ uint64_t dsplitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Start of a step for sequence blockIdx.x: choose the token (prompt or last
// sample), clamp the position as InferenceEngine.swift:55 does, gather the
// embedding row (:57-60) and draw the step's uniform.
__global__ void k_step_begin(SeqCtl* ctl, const int32_t* prompt, int prompt_stride,
                             const __half* embed, __half* x, uint32_t* u24, int max_ctx,
                             uint64_t seed, int* err, uint32_t* epoch) {
  const int seq = blockIdx.x;
  if (seq == 0 && threadIdx.x == 0) *epoch += 1;  // tags the fused step's exchanges
  __shared__ int32_t tok;
  if (threadIdx.x == 0) {
    SeqCtl c = ctl[seq];
    const int32_t slot = c.pos < max_ctx - 1 ? c.pos : max_ctx - 1;
    int32_t t = c.pos < c.n_prompt ? prompt[(size_t)seq * prompt_stride + slot] : c.last_token;
    if (t < 0 || t >= kVocab) {
      raise_error(err, kDevBadArgument);
      t = 0;
    }
    const int32_t safe = c.pos < max_ctx - 1 ? c.pos : max_ctx - 1;
    c.token = t;
    c.seq_len = (uint32_t)safe + 1;
    const uint64_t key = dsplitmix64(((uint64_t)seq << 32) ^ (uint64_t)(uint32_t)c.pos);
    c.u24 = (uint32_t)(dsplitmix64(seed ^ key) >> 40);
    u24[seq] = c.u24;
    ctl[seq] = c;
    tok = t;
  }
  __syncthreads();
  const uint4* src = reinterpret_cast<const uint4*>(embed + (size_t)tok * kHidden);
  uint4* dst = reinterpret_cast<uint4*>(x + (size_t)seq * kHidden);
  for (int i = threadIdx.x; i < kHidden / 8; i += blockDim.x) dst[i] = src[i];
}

// End of a step: record the sample (the reference prints every token from the
// last prompt forward on, InferenceEngine.swift:40-50) and advance.
__global__ void k_step_end(SeqCtl* ctl, const int32_t* sampled, int32_t* out_tokens, int max_out,
                           int stop_on_eos) {
  const int seq = blockIdx.x * blockDim.x + threadIdx.x;
  if (seq >= gridDim.x * blockDim.x) return;
  SeqCtl c = ctl[seq];
  const int32_t s = sampled[seq];
  c.last_token = s;
  if (c.pos >= c.n_prompt - 1 && !c.done) {
    if (stop_on_eos && (s == 151645 || s == 151643)) {
      c.done = 1;
    } else if (c.n_out < max_out) {
      out_tokens[(size_t)seq * max_out + c.n_out] = s;
      c.n_out += 1;
    }
  }
  c.pos += 1;
  ctl[seq] = c;
}

// ----------------------------------------------------------- WeightLoader --
int WeightLoader::load_buffer(const std::string& rel, size_t expect, void* dst, cudaStream_t st,
                              std::vector<uint8_t>& staging) const {
  const std::string path = dir_ + "/" + rel;
  struct stat sb;
  if (::stat(path.c_str(), &sb) != 0)
    return set_error(QWEN_ERR_FILE_NOT_FOUND, "weight file not found: %s", path.c_str());
  if ((size_t)sb.st_size != expect)
    return set_error(QWEN_ERR_BAD_WEIGHT_FILE, "weight file %s has %lld bytes, expected %zu",
                     path.c_str(), (long long)sb.st_size, expect);
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return set_error(QWEN_ERR_FILE_NOT_FOUND, "cannot open %s", path.c_str());
  staging.resize(expect);
  const size_t got = std::fread(staging.data(), 1, expect, f);
  std::fclose(f);
  if (got != expect)
    return set_error(QWEN_ERR_BAD_WEIGHT_FILE, "short read on %s (%zu of %zu)", path.c_str(), got,
                     expect);
  QWEN_CUDA(cudaMemcpyAsync(dst, staging.data(), expect, cudaMemcpyHostToDevice, st),
            "cudaMemcpyAsync(weights)");
  QWEN_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  return QWEN_OK;
}

// -------------------------------------------------------------- QwenModel --
void* QwenModel::dev_alloc(size_t bytes, int* rc) {
  void* p = nullptr;
  *rc = cuda_status(cudaMalloc(&p, bytes), "cudaMalloc(model)");
  if (*rc == QWEN_OK) allocs_.push_back(p);
  return p;
}

void FusedWeights::release() {
  void* ps[] = {blob, lm_tiles, norms, qkv_bias, o_bias, down_bias, rope_cs, items, item_begin};
  for (void* p : ps)
    if (p) cudaFree(p);
  blob = lm_tiles = nullptr;
  norms = qkv_bias = o_bias = down_bias = nullptr;
  rope_cs = nullptr;
  items = nullptr;
  item_begin = nullptr;
}

void TcWeights::release() {
  void* ps[] = {blob, lm, rope_cs};
  for (void* p : ps)
    if (p) cudaFree(p);
  blob = lm = nullptr;
  rope_cs = nullptr;
  rope_ctx = 0;
}

QwenModel::~QwenModel() {
  fused.release();
  tc.release();
  for (void* p : allocs_) cudaFree(p);
}

int QwenModel::allocate(int nl) {
  int rc = QWEN_OK;
  n_layers = nl;
  layers.assign(nl, QwenLayer{});
  embed = (__half*)dev_alloc((size_t)kVocab * kHidden * 2, &rc);
  QWEN_TRY(rc);
  final_norm = (__half*)dev_alloc(kHidden * 2, &rc);
  QWEN_TRY(rc);
  zero_bias = (__half*)dev_alloc(kInter * 2, &rc);
  QWEN_TRY(rc);
  QWEN_CUDA(cudaMemset(zero_bias, 0, kInter * 2), "cudaMemset");
  auto lin = [&](Q4Linear& l, int rows, int k) {
    l.rows = rows;
    l.k = k;
    l.packed = (uint8_t*)dev_alloc(l.packed_bytes(), &rc);
    if (rc) return rc;
    l.scales = (__half*)dev_alloc(l.scale_bytes(), &rc);
    return rc;
  };
  for (int i = 0; i < nl; ++i) {
    QwenLayer& L = layers[i];
    L.input_norm = (__half*)dev_alloc(kHidden * 2, &rc);
    QWEN_TRY(rc);
    L.post_attn_norm = (__half*)dev_alloc(kHidden * 2, &rc);
    QWEN_TRY(rc);
    QWEN_TRY(lin(L.q, kHidden, kHidden));
    QWEN_TRY(lin(L.k, kKVDim, kHidden));
    QWEN_TRY(lin(L.v, kKVDim, kHidden));
    QWEN_TRY(lin(L.o, kHidden, kHidden));
    QWEN_TRY(lin(L.gate, kInter, kHidden));
    QWEN_TRY(lin(L.up, kInter, kHidden));
    QWEN_TRY(lin(L.down, kHidden, kInter));
    L.qkv_bias = (__half*)dev_alloc(kQKVRows * 2, &rc);
    QWEN_TRY(rc);
    L.o_bias = (__half*)dev_alloc(kHidden * 2, &rc);
    QWEN_TRY(rc);
    L.down_bias = (__half*)dev_alloc(kHidden * 2, &rc);
    QWEN_TRY(rc);
  }
  return QWEN_OK;
}

// QwenModel.swift:22-34 and QwenLayer.swift:29-52: file names of the
// reference weight directory.
int QwenModel::load(const std::string& dir, cudaStream_t st) {
  WeightLoader wl(dir);
  std::vector<uint8_t> staging;
  QWEN_TRY(wl.load_buffer("global/embed_tokens.bin", (size_t)kVocab * kHidden * 2, embed, st, staging));
  QWEN_TRY(wl.load_buffer("global/final_norm.bin", kHidden * 2, final_norm, st, staging));
  for (int i = 0; i < n_layers; ++i) {
    QwenLayer& L = layers[i];
    const std::string n = "layer" + std::to_string(i);
    QWEN_TRY(wl.load_layer_weight(i, n + "_norm", kHidden * 2, L.input_norm, st, staging));
    QWEN_TRY(wl.load_layer_weight(i, n + "_post_attn_norm", kHidden * 2, L.post_attn_norm, st, staging));
    struct { Q4Linear* l; const char* name; } lins[] = {
        {&L.q, "q_proj"}, {&L.k, "k_proj"}, {&L.v, "v_proj"}, {&L.o, "o_proj"},
        {&L.gate, "gate_proj"}, {&L.up, "up_proj"}, {&L.down, "down_proj"}};
    for (auto& e : lins) {
      QWEN_TRY(wl.load_layer_weight(i, std::string(e.name) + "_4bit", e.l->packed_bytes(), e.l->packed, st, staging));
      QWEN_TRY(wl.load_layer_weight(i, std::string(e.name) + "_scales", e.l->scale_bytes(), e.l->scales, st, staging));
    }
    QWEN_TRY(wl.load_layer_weight(i, "qkv_bias", kQKVRows * 2, L.qkv_bias, st, staging));
    QWEN_TRY(wl.load_layer_weight(i, "o_bias", kHidden * 2, L.o_bias, st, staging));
    QWEN_TRY(wl.load_layer_weight(i, "mlp_down_bias", kHidden * 2, L.down_bias, st, staging));
  }
  loaded = true;
  return QWEN_OK;
}

int QwenModel::init_random(uint64_t seed, cudaStream_t st) {
  const size_t tmp_elems = (size_t)16 << 20;  // 16 Mi floats per chunk
  float* tmp = nullptr;
  QWEN_CUDA(cudaMalloc(&tmp, tmp_elems * sizeof(float)), "cudaMalloc(init tmp)");
  int rc = QWEN_OK;
  uint64_t sid = 1;
  auto normal_f16 = [&](__half* dst, size_t n, float mean, float sd) {
    for (size_t off = 0; off < n && rc == QWEN_OK; off += tmp_elems) {
      const size_t c = std::min(tmp_elems, n - off);
      if (launch_fill_normal(tmp, c, seed, sid++, mean, sd, st) ||
          launch_f32_to_f16(tmp, dst + off, c, st))
        rc = launch_status("init_random");
    }
  };
  auto q4 = [&](Q4Linear& l) {
    const size_t n = (size_t)l.rows * l.k;
    if (rc) return;
    if (launch_fill_normal(tmp, n, seed, sid++, 0.0f, 0.02f, st) ||
        launch_quantize_q4(tmp, n, l.packed, l.scales, st))
      rc = launch_status("init_random");
  };
  normal_f16(embed, (size_t)kVocab * kHidden, 0.0f, 0.02f);
  normal_f16(final_norm, kHidden, 1.0f, 0.02f);
  for (int i = 0; i < n_layers && rc == QWEN_OK; ++i) {
    QwenLayer& L = layers[i];
    normal_f16(L.input_norm, kHidden, 1.0f, 0.02f);
    normal_f16(L.post_attn_norm, kHidden, 1.0f, 0.02f);
    q4(L.q); q4(L.k); q4(L.v); q4(L.o); q4(L.gate); q4(L.up); q4(L.down);
    normal_f16(L.qkv_bias, kQKVRows, 0.0f, 0.02f);
    if (rc == QWEN_OK) rc = cuda_status(cudaMemsetAsync(L.o_bias, 0, kHidden * 2, st), "memset");
    if (rc == QWEN_OK) rc = cuda_status(cudaMemsetAsync(L.down_bias, 0, kHidden * 2, st), "memset");
  }
  cudaError_t e = cudaStreamSynchronize(st);
  cudaFree(tmp);
  QWEN_TRY(rc);
  QWEN_CUDA(e, "init_random sync");
  loaded = true;
  return QWEN_OK;
}

// ------------------------------------------------------- InferenceManager --
InferenceManager::~InferenceManager() {
  if (trace) cudaFree(trace);
  for (void* p : allocs_) cudaFree(p);
}

int InferenceManager::alloc_tracked(size_t bytes, void** out) {
  QWEN_CUDA(cudaMalloc(out, bytes), "cudaMalloc(state)");
  allocs_.push_back(*out);
  QWEN_CUDA(cudaMemset(*out, 0, bytes), "cudaMemset(state)");
  return QWEN_OK;
}

int InferenceManager::allocate(int b, int nl, int mc, int mo) {
  batch = b;
  n_layers = nl;
  max_ctx = mc;
  max_out = mo;
  auto alloc = [&](size_t bytes, void** out) {
    int rc = cuda_status(cudaMalloc(out, bytes), "cudaMalloc(state)");
    if (rc == QWEN_OK) {
      allocs_.push_back(*out);
      rc = cuda_status(cudaMemset(*out, 0, bytes), "cudaMemset(state)");
    }
    return rc;
  };
  const size_t B = (size_t)b;
  QWEN_TRY(alloc(B * kHidden * 2, (void**)&x));
  QWEN_TRY(alloc(B * kHidden * 2, (void**)&residual));
  QWEN_TRY(alloc(B * kHidden * 2, (void**)&q));
  QWEN_TRY(alloc(B * kKVDim * 2, (void**)&k));
  QWEN_TRY(alloc(B * kKVDim * 2, (void**)&v));
  QWEN_TRY(alloc(B * kHidden * 2, (void**)&attn_out));
  QWEN_TRY(alloc(B * kInter * 2, (void**)&gate));
  QWEN_TRY(alloc(B * kInter * 2, (void**)&up));
  QWEN_TRY(alloc(B * kHidden * 2, (void**)&mlp_out));
  QWEN_TRY(alloc(B * kVocab * 2, (void**)&logits));
  QWEN_TRY(alloc((size_t)kHeads * mc * 4, (void**)&scores));
  QWEN_TRY(alloc((size_t)nl * B * mc * kKVDim * 2, (void**)&kc));
  QWEN_TRY(alloc((size_t)nl * B * mc * kKVDim * 2, (void**)&vc));
  QWEN_TRY(alloc(B * sizeof(SeqCtl), (void**)&ctl));
  QWEN_TRY(alloc(B * mc * sizeof(int32_t), (void**)&prompt));
  QWEN_TRY(alloc(B * mo * sizeof(int32_t), (void**)&out_tokens));
  // sampled[B] and the error words in one allocation, the error words right
  // after the ids: a batch-1 forward() reads the id and error word 0 back in
  // one 8-byte copy
  QWEN_TRY(alloc(B * sizeof(int32_t) + sizeof(int) * 32, (void**)&sampled));
  err = reinterpret_cast<int*>(sampled + B);
  QWEN_TRY(alloc(B * sizeof(uint32_t) + 64, (void**)&u24_));
  QWEN_TRY(alloc(sizeof(uint32_t) * 4, (void**)&epoch));
  attn_splits = attn_max_splits(mc, b);
  QWEN_TRY(alloc(attn_scratch_bytes(attn_splits, b), &attn_scratch));
  samp_scratch_bytes = sampler_scratch_bytes(b);
  if (samp_scratch_bytes) QWEN_TRY(alloc(samp_scratch_bytes, &samp_scratch));
  return QWEN_OK;
}

// ------------------------------------------------------------ QwenEngine --
QwenEngine::~QwenEngine() {
  if (pinned_) cudaFreeHost(pinned_);
  if (graph_exec_) cudaGraphExecDestroy(graph_exec_);
  if (graph_) cudaGraphDestroy(graph_);
  if (stream_) {
    cudaStreamSynchronize(stream_);
    cudaStreamDestroy(stream_);
  }
}

int QwenEngine::init(const qwen_engine_config& cfg) {
  cfg_ = cfg;
  if (cfg.max_ctx < 1 || cfg.max_ctx > (1 << 20))
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "max_ctx=%d out of range", cfg.max_ctx);
  if (cfg.batch < 1 || cfg.batch > 1024)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "batch=%d out of range", cfg.batch);
  if (cfg.n_layers < 1 || cfg.n_layers > kLayers)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "n_layers=%d out of range", cfg.n_layers);
  if (cfg.kernels != QWEN_KERNELS_FUSED && cfg.kernels != QWEN_KERNELS_OPS &&
      cfg.kernels != QWEN_KERNELS_TC)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "unknown kernels mode %d", cfg.kernels);
  if (cfg.prefill_mode != QWEN_PREFILL_CHUNKED && cfg.prefill_mode != QWEN_PREFILL_STEPS)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "unknown prefill mode %d", cfg.prefill_mode);
  if (cfg.ctx_overflow != QWEN_CTX_CLAMP && cfg.ctx_overflow != QWEN_CTX_ERROR)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "unknown ctx_overflow mode %d", cfg.ctx_overflow);
  if (cfg.kernels == QWEN_KERNELS_OPS && cfg.batch != 1)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "the per-op kernel path decodes one sequence");
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess || ndev == 0)
    return set_error(QWEN_ERR_NO_DEVICE, "no CUDA device (%s)", cudaGetErrorString(e));
  if (cfg.device < 0 || cfg.device >= ndev)
    return set_error(QWEN_ERR_NO_DEVICE, "device %d not present (%d devices)", cfg.device, ndev);
  QWEN_CUDA(cudaSetDevice(cfg.device), "cudaSetDevice");
  QWEN_CUDA(cudaDeviceGetAttribute(&sm_count_, cudaDevAttrMultiProcessorCount, cfg.device),
            "cudaDeviceGetAttribute");
  QWEN_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  QWEN_CUDA(cudaHostAlloc((void**)&pinned_, sizeof(HostStaging), cudaHostAllocDefault), "cudaHostAlloc");
  std::memset(pinned_, 0, sizeof(HostStaging));
  QWEN_TRY(ensure_rope_table());
  QWEN_TRY(model_.allocate(cfg.n_layers));
  const int max_out = cfg.max_ctx + 1;
  QWEN_TRY(state_.allocate(cfg.batch, cfg.n_layers, cfg.max_ctx, max_out));
  initialised_ = true;
  return QWEN_OK;
}

int QwenEngine::load_weights(const std::string& dir) {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  QWEN_TRY(model_.load(dir, stream_));
  QWEN_TRY(build_step_weights());
  return QWEN_OK;
}

// The fused engine keeps the tensor-core layout too when it prefills on the
// tensor cores (both fit in HBM many times over: 1.2 GB each).
bool QwenEngine::uses_tc_layout() const {
  return cfg_.kernels == QWEN_KERNELS_TC ||
         (cfg_.kernels == QWEN_KERNELS_FUSED && cfg_.prefill_mode == QWEN_PREFILL_CHUNKED);
}

int QwenEngine::build_step_weights() {
  if (cfg_.kernels == QWEN_KERNELS_FUSED) QWEN_TRY(build_fused_weights(model_, cfg_.max_ctx, stream_));
  if (uses_tc_layout()) QWEN_TRY(build_tc_weights(model_, cfg_.max_ctx, stream_));
  return QWEN_OK;
}

int QwenEngine::init_random(uint64_t seed) {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  QWEN_TRY(model_.init_random(seed, stream_));
  QWEN_TRY(build_step_weights());
  return QWEN_OK;
}

int QwenEngine::reset() {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  QWEN_CUDA(cudaMemsetAsync(state_.ctl, 0, sizeof(SeqCtl) * state_.batch, stream_), "memset");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  return QWEN_OK;
}

int QwenEngine::enqueue_step_ops(cudaEvent_t* ev) {
  InferenceManager& s = state_;
  QwenModel& m = model_;
  cudaStream_t st = stream_;
  void* vs = st;
  const uint32_t* sl = &s.ctl[0].seq_len;
  if (ev) cudaEventRecord(ev[0], st);
  k_step_begin<<<s.batch, 256, 0, st>>>(s.ctl, s.prompt, s.max_ctx, m.embed, s.x, s.u24_,
                                        s.max_ctx, cfg_.seed, s.err, s.epoch);
  if (ev) cudaEventRecord(ev[1], st);
  for (int i = 0; i < m.n_layers; ++i) {
    QwenLayer& L = m.layers[i];
    __half* kc = s.kc + (size_t)i * s.kv_layer_stride();
    __half* vc = s.vc + (size_t)i * s.kv_layer_stride();
    launch_rms_norm(s.x, L.input_norm, s.residual, vs);
    launch_gemv_q4_rowmajor(L.q.packed, L.q.scales, s.residual, s.q, L.qkv_bias, kHidden, kHidden, vs);
    launch_gemv_q4_rowmajor(L.k.packed, L.k.scales, s.residual, s.k, L.qkv_bias + kHidden, kKVDim, kHidden, vs);
    launch_gemv_q4_rowmajor(L.v.packed, L.v.scales, s.residual, s.v, L.qkv_bias + kHidden + kKVDim, kKVDim, kHidden, vs);
    launch_rope(s.q, kHeads, sl, vs);
    launch_rope(s.k, kKVHeads, sl, vs);
    launch_write_kv_cache(s.k, s.v, kc, vc, sl, s.max_ctx, vs);
    launch_attention_scores(s.q, kc, s.scores, sl, s.max_ctx, vs);
    launch_softmax(s.scores, sl, vs);
    launch_attn_weighted_sum(s.scores, vc, s.attn_out, sl, vs);
    launch_gemv_q4_rowmajor(L.o.packed, L.o.scales, s.attn_out, s.q, L.o_bias, kHidden, kHidden, vs);
    launch_residual_add(s.x, s.q, s.x, kHidden, vs);
    launch_rms_norm(s.x, L.post_attn_norm, s.residual, vs);
    launch_gemv_q4_rowmajor(L.gate.packed, L.gate.scales, s.residual, s.gate, m.zero_bias, kInter, kHidden, vs);
    launch_gemv_q4_rowmajor(L.up.packed, L.up.scales, s.residual, s.up, m.zero_bias, kInter, kHidden, vs);
    launch_swiglu(s.gate, s.up, kInter, vs);
    launch_gemv_q4_rowmajor(L.down.packed, L.down.scales, s.gate, s.mlp_out, L.down_bias, kHidden, kInter, vs);
    launch_residual_add(s.x, s.mlp_out, s.x, kHidden, vs);
  }
  launch_rms_norm(s.x, m.final_norm, s.residual, vs);
  launch_gemv_fp16_rowmajor(m.embed, s.residual, s.logits, kVocab, kHidden, vs);
  if (ev) cudaEventRecord(ev[2], st);
  if (launch_sample(s.logits, s.batch, kVocab, kActualVocab, cfg_.temperature, cfg_.top_p, s.u24_,
                    s.sampled, s.samp_scratch, s.err, st, wait_ns_,
                    stall_site_ == kSamplerStallSite) != 0)
    return launch_status("sample");
  k_step_end<<<1, s.batch, 0, st>>>(s.ctl, s.sampled, s.out_tokens, s.max_out, cfg_.stop_on_eos);
  if (ev) cudaEventRecord(ev[3], st);
  return launch_status("decode step (ops)");
}

int QwenEngine::enqueue_step_fused(cudaEvent_t* ev) {
  InferenceManager& s = state_;
  cudaStream_t st = stream_;
  if (ev) cudaEventRecord(ev[0], st);
  k_step_begin<<<s.batch, 256, 0, st>>>(s.ctl, s.prompt, s.max_ctx, model_.embed, s.x, s.u24_,
                                        s.max_ctx, cfg_.seed, s.err, s.epoch);
  if (ev) cudaEventRecord(ev[1], st);
  FusedStepArgs a{&model_, &state_, model_.n_layers, sm_count_, wait_ns_, stall_site_};
  QWEN_TRY(enqueue_fused_step(a, st));
  if (ev) cudaEventRecord(ev[2], st);
  if (launch_sample(s.logits, s.batch, kVocab, kActualVocab, cfg_.temperature, cfg_.top_p, s.u24_,
                    s.sampled, s.samp_scratch, s.err, st, wait_ns_,
                    stall_site_ == kSamplerStallSite) != 0)
    return launch_status("sample");
  k_step_end<<<1, s.batch, 0, st>>>(s.ctl, s.sampled, s.out_tokens, s.max_out, cfg_.stop_on_eos);
  if (ev) cudaEventRecord(ev[3], st);
  return launch_status("decode step (fused)");
}

int QwenEngine::enqueue_step_tc(cudaEvent_t* ev) {
  InferenceManager& s = state_;
  cudaStream_t st = stream_;
  if (ev) cudaEventRecord(ev[0], st);
  k_step_begin<<<s.batch, 256, 0, st>>>(s.ctl, s.prompt, s.max_ctx, model_.embed, s.x, s.u24_,
                                        s.max_ctx, cfg_.seed, s.err, s.epoch);
  if (ev) cudaEventRecord(ev[1], st);
  QWEN_TRY(enqueue_tc_model(model_, state_, tc_decode_rows(state_), sm_count_, st));
  if (ev) cudaEventRecord(ev[2], st);
  if (launch_sample(s.logits, s.batch, kVocab, kActualVocab, cfg_.temperature, cfg_.top_p, s.u24_,
                    s.sampled, s.samp_scratch, s.err, st, wait_ns_,
                    stall_site_ == kSamplerStallSite) != 0)
    return launch_status("sample");
  k_step_end<<<1, s.batch, 0, st>>>(s.ctl, s.sampled, s.out_tokens, s.max_out, cfg_.stop_on_eos);
  if (ev) cudaEventRecord(ev[3], st);
  return launch_status("decode step (tensor cores)");
}

int QwenEngine::enqueue_step(cudaEvent_t* ev) {
  if (cfg_.kernels == QWEN_KERNELS_OPS) return enqueue_step_ops(ev);
  if (cfg_.kernels == QWEN_KERNELS_TC) return enqueue_step_tc(ev);
  return enqueue_step_fused(ev);
}

int QwenEngine::ensure_graph() {
  if (graph_exec_) return QWEN_OK;
  if (!model_.loaded) return set_error(QWEN_ERR_STATE, "no weights: call load_weights or init_random");
  if (cfg_.kernels == QWEN_KERNELS_FUSED && !state_.fused_scratch) {
    size_t bytes = 0;
    QWEN_TRY(fused_scratch_bytes(state_.batch, state_.max_ctx, sm_count_, &bytes));
    QWEN_CUDA(cudaMalloc(&state_.fused_scratch, bytes), "cudaMalloc(fused scratch)");
    QWEN_CUDA(cudaMemset(state_.fused_scratch, 0, bytes), "cudaMemset");
    state_.fused_scratch_bytes = bytes;
  }
  if (uses_tc_layout()) QWEN_TRY(tc_state_allocate(state_, sm_count_));
  sampler_prepare();
  QWEN_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "BeginCapture");
  const int rc = enqueue_step(nullptr);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(stream_, &g);
  if (rc != QWEN_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  QWEN_CUDA(e, "EndCapture");
  graph_ = g;
  QWEN_CUDA(cudaGraphInstantiate(&graph_exec_, graph_, 0), "cudaGraphInstantiate");
  return QWEN_OK;
}

int QwenEngine::check_device_error() {
  int h[16] = {0};
  QWEN_CUDA(cudaMemcpyAsync(h, state_.err, sizeof(h), cudaMemcpyDeviceToHost, stream_), "memcpy err");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  if (h[0] == 0) return QWEN_OK;
  cudaMemsetAsync(state_.err, 0, sizeof(h), stream_);
  // a wait that gave up can leave the grid sampler's exchange words set
  if (state_.samp_scratch) cudaMemsetAsync(state_.samp_scratch, 0, state_.samp_scratch_bytes, stream_);
  cudaStreamSynchronize(stream_);
  if (h[0] == kDevWaitTimeout)
    return set_error(QWEN_ERR_DEVICE_TIMEOUT,
                     "a device-side wait timed out (site %d, phase %d, CTA %d, thread %d; "
                     "detail %d %d %d | %d %d %d %d %d %d %d %d)",
                     h[1] / 100, h[1] % 100, h[2], h[3], h[4], h[5], h[6], h[7], h[8], h[9], h[10],
                     h[11], h[12], h[13], h[14]);
  return set_error(QWEN_ERR_INVALID_ARGUMENT, "device reported a bad argument (token id or length)");
}

int QwenEngine::run_steps(int n) {
  QWEN_TRY(ensure_graph());
  // At most kMaxQueuedSteps step graphs are queued on the stream at a time
  // (long prefills would otherwise queue thousands of launches).
  constexpr int kMaxQueuedSteps = 256;
  for (int i = 0; i < n; ++i) {
    if (i > 0 && i % kMaxQueuedSteps == 0) QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
    QWEN_CUDA(cudaGraphLaunch(graph_exec_, stream_), "cudaGraphLaunch");
  }
  return QWEN_OK;
}

int QwenEngine::upload_prompt(const int32_t* ids, int32_t n, int32_t start) {
  if (n < 0 || start < 0 || start + n > state_.max_ctx)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "prompt of %d tokens at %d exceeds max_ctx %d", n,
                     start, state_.max_ctx);
  for (int i = 0; i < n * state_.batch; ++i)
    if (ids[i] < 0 || ids[i] >= kVocab)
      return set_error(QWEN_ERR_INVALID_ARGUMENT, "token id %d out of range", ids[i]);
  for (int b = 0; b < state_.batch; ++b)
    QWEN_CUDA(cudaMemcpyAsync(state_.prompt + (size_t)b * state_.max_ctx + start, ids + (size_t)b * n,
                              n * sizeof(int32_t), cudaMemcpyHostToDevice, stream_),
              "cudaMemcpyAsync(prompt)");
  return QWEN_OK;
}

int QwenEngine::forward(int32_t token, int32_t position, int32_t* next) {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  if (state_.batch != 1) return set_error(QWEN_ERR_INVALID_ARGUMENT, "forward() drives a batch-1 engine");
  if (position < 0) return set_error(QWEN_ERR_INVALID_ARGUMENT, "negative position");
  if (token < 0 || token >= kVocab) return set_error(QWEN_ERR_INVALID_ARGUMENT, "token id %d out of range", token);
  if (cfg_.ctx_overflow == QWEN_CTX_ERROR && position >= state_.max_ctx)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "position %d past the context window (%d)", position,
                     state_.max_ctx);
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  QWEN_TRY(ensure_graph());
  // One step that reads `token` at `position` (as the step's last token, past
  // the prompt); positions past max_ctx-1 reuse the last slot, as
  // InferenceEngine.swift:55 clamps.  One copy in (the sequence's control
  // block, token included) and one out (the id and error word 0, adjacent).
  HostStaging* hs = pinned_;
  std::memset(&hs->ctl, 0, sizeof(hs->ctl));
  hs->ctl.pos = position;
  hs->ctl.n_prompt = position;
  hs->ctl.last_token = token;
  QWEN_CUDA(cudaMemcpyAsync(state_.ctl, &hs->ctl, sizeof(SeqCtl), cudaMemcpyHostToDevice, stream_), "memcpy");
  QWEN_TRY(run_steps(1));
  static_assert(offsetof(HostStaging, err) == offsetof(HostStaging, result) + sizeof(int32_t),
                "the id and the error word are read back together");
  QWEN_CUDA(cudaMemcpyAsync(&hs->result, state_.sampled, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost,
                            stream_),
            "memcpy");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  if (hs->err != 0) return check_device_error();
  *next = hs->result;
  return QWEN_OK;
}

int QwenEngine::set_trace(int enable) {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  const size_t n = (size_t)std::max(1, model_.fused.grid > 0 ? model_.fused.grid : sm_count_) *
                       trace_stride_for(model_.n_layers);
  if (enable && !state_.trace) {
    QWEN_CUDA(cudaMalloc(&state_.trace, n * sizeof(unsigned long long)), "cudaMalloc(trace)");
    QWEN_CUDA(cudaMemset(state_.trace, 0, n * sizeof(unsigned long long)), "memset");
  } else if (!enable && state_.trace) {
    cudaFree(state_.trace);
    state_.trace = nullptr;
  }
  drop_graph();  // the captured step graph bakes in the trace pointer
  return QWEN_OK;
}

void QwenEngine::drop_graph() {
  if (graph_exec_) cudaGraphExecDestroy(graph_exec_);
  if (graph_) cudaGraphDestroy(graph_);
  graph_exec_ = nullptr;
  graph_ = nullptr;
}

int QwenEngine::set_wait_timeout(uint64_t ns) {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  if (ns < 1000000ull || ns > 60000000000ull)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "wait timeout %llu ns outside [1 ms, 60 s]",
                     (unsigned long long)ns);
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  wait_ns_ = ns;
  drop_graph();  // the limit is a parameter of the captured launch
  return QWEN_OK;
}

int QwenEngine::test_stall(int site) {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  if (site != 0 && site != kFusedStallDownPart && site != kSamplerStallSite)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "no stall hook for wait site %d", site);
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  stall_site_ = site;
  drop_graph();
  return QWEN_OK;
}

int QwenEngine::get_trace(unsigned long long* host, size_t n, size_t* needed) {
  const size_t total = (size_t)std::max(1, model_.fused.grid > 0 ? model_.fused.grid : sm_count_) *
                           trace_stride_for(model_.n_layers);
  *needed = total;
  if (!state_.trace) return set_error(QWEN_ERR_STATE, "tracing is off");
  if (!host || n < total) return QWEN_OK;
  QWEN_CUDA(cudaMemcpy(host, state_.trace, total * sizeof(unsigned long long), cudaMemcpyDeviceToHost),
            "memcpy trace");
  return QWEN_OK;
}

int QwenEngine::kernels_per_step(int* n) const {
  // step begin + sampler + step end around the model kernels
  if (cfg_.kernels == QWEN_KERNELS_OPS)
    *n = 3 + model_.n_layers * 18 + 2;
  else if (cfg_.kernels == QWEN_KERNELS_TC)
    *n = 3 + tc_kernels_per_step(model_.n_layers);
  else
    *n = 3 + 1;
  return QWEN_OK;
}

int QwenEngine::time_steps(int n, float* ms_step, float* ms_model) {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  if (n < 1) return set_error(QWEN_ERR_INVALID_ARGUMENT, "time_steps: n < 1");
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  QWEN_TRY(ensure_graph());
  std::vector<cudaEvent_t> ev(4 * n);
  for (auto& e : ev) QWEN_CUDA(cudaEventCreate(&e), "cudaEventCreate");
  int rc = QWEN_OK;
  for (int i = 0; i < n && rc == QWEN_OK; ++i) {
    cudaEvent_t* e = &ev[4 * i];
    rc = enqueue_step(e);
  }
  if (rc == QWEN_OK) rc = cuda_status(cudaStreamSynchronize(stream_), "sync");
  double step = 0, model = 0;
  for (int i = 0; i < n && rc == QWEN_OK; ++i) {
    float a = 0, b = 0;
    cudaEventElapsedTime(&a, ev[4 * i], ev[4 * i + 3]);
    cudaEventElapsedTime(&b, ev[4 * i + 1], ev[4 * i + 2]);
    step += a;
    model += b;
  }
  for (auto& e : ev) cudaEventDestroy(e);
  QWEN_TRY(rc);
  *ms_step = (float)(step / n);
  *ms_model = (float)(model / n);
  return check_device_error();
}

// One eagerly launched step of the tensor-core path with an event after every
// model kernel: ms[i] = device time from the previous launch's end to launch
// i's end, in launch order (one entry per model kernel).
int QwenEngine::profile_step(float* ms, int cap, int* n) {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  if (cfg_.kernels != QWEN_KERNELS_TC)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "per-launch profile: tensor-core step only");
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  QWEN_TRY(ensure_graph());
  const int need = tc_kernels_per_step(model_.n_layers);
  *n = need;
  if (!ms || cap < need) return QWEN_OK;
  std::vector<cudaEvent_t> ev(need + 1);
  for (auto& e : ev) QWEN_CUDA(cudaEventCreate(&e), "cudaEventCreate");
  InferenceManager& s = state_;
  cudaStream_t st = stream_;
  k_step_begin<<<s.batch, 256, 0, st>>>(s.ctl, s.prompt, s.max_ctx, model_.embed, s.x, s.u24_,
                                        s.max_ctx, cfg_.seed, s.err, s.epoch);
  cudaEventRecord(ev[0], st);
  int marks = 0;
  int rc = enqueue_tc_model(model_, state_, tc_decode_rows(state_), sm_count_, st, ev.data() + 1,
                            &marks);
  if (rc == QWEN_OK && launch_sample(s.logits, s.batch, kVocab, kActualVocab, cfg_.temperature,
                                     cfg_.top_p, s.u24_, s.sampled, s.samp_scratch, s.err, st, wait_ns_,
                    stall_site_ == kSamplerStallSite) != 0)
    rc = launch_status("sample");
  if (rc == QWEN_OK)
    k_step_end<<<1, s.batch, 0, st>>>(s.ctl, s.sampled, s.out_tokens, s.max_out, cfg_.stop_on_eos);
  if (rc == QWEN_OK) rc = cuda_status(cudaStreamSynchronize(st), "sync");
  for (int i = 0; i < need && rc == QWEN_OK; ++i) {
    if (i >= marks) { ms[i] = 0.f; continue; }
    cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]);
  }
  for (auto& e : ev) cudaEventDestroy(e);
  QWEN_TRY(rc);
  return check_device_error();
}

int QwenEngine::prefill(const int32_t* ids, int32_t n) {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  if (n < 1) return set_error(QWEN_ERR_INVALID_ARGUMENT, "empty prompt");
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  QWEN_TRY(ensure_graph());
  if (cfg_.prefill_mode == QWEN_PREFILL_CHUNKED && state_.tc_px && n > 1) return prefill_chunked(ids, n);
  QWEN_TRY(upload_prompt(ids, n, 0));
  std::vector<SeqCtl> c(state_.batch);
  for (auto& x : c) {
    std::memset(&x, 0, sizeof(x));
    x.n_prompt = n;
  }
  QWEN_CUDA(cudaMemcpyAsync(state_.ctl, c.data(), sizeof(SeqCtl) * c.size(), cudaMemcpyHostToDevice,
                            stream_), "memcpy ctl");
  QWEN_TRY(run_steps(n));
  return check_device_error();
}

// Prefill on the tensor cores: the prompt positions of every sequence go
// through the model as the rows of batched steps, a chunk of positions at a
// time (kTcPrefillRows positions of a batch-1 engine, or as many positions as
// fit kTcMaxNb rows).  Each row attends to positions 0 .. its own, the rows
// before it in the chunk included, since the chunk's K/V rows are written
// before its attention runs.  Only the last chunk runs the LM head, and only
// each sequence's last position is sampled -- exactly as the sequential loop's
// last prompt step samples it (InferenceEngine.swift:29-52): same uniform,
// same record.  The reference's earlier prompt steps also sample, but their
// ids are discarded (:34-36).
int QwenEngine::prefill_chunked(const int32_t* ids, int32_t n) {
  InferenceManager& s = state_;
  cudaStream_t st = stream_;
  QWEN_TRY(upload_prompt(ids, n, 0));
  const int B = s.batch;
  const int C = std::max(1, s.tc_rows / B);  // positions per chunk
  int last = 0;
  for (int p0 = 0; p0 < n; p0 += C) {
    const int np = std::min(C, n - p0);
    const bool final = p0 + np == n;
    QWEN_TRY(launch_prefill_rows(s, model_.embed, p0, np, st));
    const TcRows v{B * np, s.tc_px, s.tc_pq, s.tc_row_len, 1, s.tc_row_seq, s.tc_pattn, s.tc_psplits,
                   final ? s.tc_plogits : nullptr};
    QWEN_TRY(enqueue_tc_model(model_, s, v, sm_count_, st));
    last = np;
  }
  std::vector<SeqCtl> c(B);
  for (auto& x : c) {
    std::memset(&x, 0, sizeof(x));
    x.pos = n - 1;
    x.n_prompt = n;
  }
  QWEN_CUDA(cudaMemcpyAsync(s.ctl, c.data(), sizeof(SeqCtl) * B, cudaMemcpyHostToDevice, st), "memcpy ctl");
  k_step_begin<<<B, 256, 0, st>>>(s.ctl, s.prompt, s.max_ctx, model_.embed, s.x, s.u24_, s.max_ctx,
                                  cfg_.seed, s.err, s.epoch);
  // each sequence's last row of the final chunk: row b * last + last - 1
  QWEN_CUDA(cudaMemcpy2DAsync(s.logits, (size_t)kVocab * 2, s.tc_plogits + (size_t)(last - 1) * kVocab,
                              (size_t)last * kVocab * 2, (size_t)kVocab * 2, B, cudaMemcpyDeviceToDevice,
                              st), "memcpy logits");
  if (launch_sample(s.logits, B, kVocab, kActualVocab, cfg_.temperature, cfg_.top_p, s.u24_,
                    s.sampled, s.samp_scratch, s.err, st, wait_ns_,
                    stall_site_ == kSamplerStallSite) != 0)
    return launch_status("sample");
  k_step_end<<<1, B, 0, st>>>(s.ctl, s.sampled, s.out_tokens, s.max_out, cfg_.stop_on_eos);
  QWEN_TRY(launch_status("chunked prefill"));
  QWEN_CUDA(cudaStreamSynchronize(st), "sync");
  return check_device_error();
}

int QwenEngine::decode(int32_t n_steps, int32_t* out) {
  if (!initialised_) return set_error(QWEN_ERR_STATE, "engine not initialised");
  if (n_steps < 0) return set_error(QWEN_ERR_INVALID_ARGUMENT, "negative step count");
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  std::vector<SeqCtl> c(state_.batch);
  QWEN_CUDA(cudaMemcpyAsync(c.data(), state_.ctl, sizeof(SeqCtl) * c.size(), cudaMemcpyDeviceToHost,
                            stream_), "memcpy ctl");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  if (out)
    for (auto& x : c)
      if (x.n_out + n_steps > state_.max_out)
        return set_error(QWEN_ERR_INVALID_ARGUMENT, "decode: %d more tokens exceed the output buffer", n_steps);
  if (cfg_.ctx_overflow == QWEN_CTX_ERROR)
    for (auto& x : c)
      if (x.pos + n_steps > state_.max_ctx)
        return set_error(QWEN_ERR_INVALID_ARGUMENT, "decode: %d more steps from position %d pass the "
                         "context window (%d)", n_steps, x.pos, state_.max_ctx);
  QWEN_TRY(run_steps(n_steps));
  QWEN_TRY(check_device_error());
  if (out) {
    for (int b = 0; b < state_.batch; ++b)
      QWEN_CUDA(cudaMemcpyAsync(out + (size_t)b * n_steps,
                                state_.out_tokens + (size_t)b * state_.max_out + c[b].n_out,
                                n_steps * sizeof(int32_t), cudaMemcpyDeviceToHost, stream_), "memcpy out");
    QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  }
  return QWEN_OK;
}

int QwenEngine::generate(const int32_t* ids, int32_t n_prompt, int32_t max_tokens, int32_t* out,
                         int32_t* n_out) {
  if (max_tokens < 1) return set_error(QWEN_ERR_INVALID_ARGUMENT, "max_tokens must be >= 1");
  if (max_tokens > state_.max_out) return set_error(QWEN_ERR_INVALID_ARGUMENT, "max_tokens too large");
  if (cfg_.ctx_overflow == QWEN_CTX_ERROR && (int64_t)n_prompt + max_tokens - 1 > state_.max_ctx)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "generate: %d prompt + %d generated positions pass the "
                     "context window (%d)", n_prompt, max_tokens - 1, state_.max_ctx);
  QWEN_TRY(prefill(ids, n_prompt));
  // The reference runs maxTokens decode forwards and prints the token before
  // each one (InferenceEngine.swift:40-50); the last forward's result is never
  // printed, so max_tokens - 1 further steps produce all printed tokens.
  QWEN_TRY(run_steps(max_tokens - 1));
  QWEN_TRY(check_device_error());
  std::vector<SeqCtl> c(state_.batch);
  QWEN_CUDA(cudaMemcpyAsync(c.data(), state_.ctl, sizeof(SeqCtl) * c.size(), cudaMemcpyDeviceToHost,
                            stream_), "memcpy ctl");
  for (int b = 0; b < state_.batch; ++b)
    QWEN_CUDA(cudaMemcpyAsync(out + (size_t)b * max_tokens, state_.out_tokens + (size_t)b * state_.max_out,
                              max_tokens * sizeof(int32_t), cudaMemcpyDeviceToHost, stream_), "memcpy out");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  for (int b = 0; b < state_.batch; ++b) n_out[b] = std::min(c[b].n_out, max_tokens);
  return QWEN_OK;
}

int QwenEngine::get_logits(int32_t seq, uint16_t* host) {
  if (seq < 0 || seq >= state_.batch) return set_error(QWEN_ERR_INVALID_ARGUMENT, "bad sequence %d", seq);
  QWEN_CUDA(cudaMemcpyAsync(host, state_.logits + (size_t)seq * kVocab, kVocab * 2,
                            cudaMemcpyDeviceToHost, stream_), "memcpy logits");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  return QWEN_OK;
}

int QwenEngine::get_kv(int32_t seq, int32_t layer, int32_t n_pos, uint16_t* hk, uint16_t* hv) {
  if (seq < 0 || seq >= state_.batch || layer < 0 || layer >= state_.n_layers || n_pos < 0 ||
      n_pos > state_.max_ctx)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "get_kv: bad arguments");
  const size_t off = (size_t)layer * state_.kv_layer_stride() + (size_t)seq * state_.kv_seq_stride();
  const size_t bytes = (size_t)n_pos * kKVDim * 2;
  if (hk) QWEN_CUDA(cudaMemcpyAsync(hk, state_.kc + off, bytes, cudaMemcpyDeviceToHost, stream_), "memcpy");
  if (hv) QWEN_CUDA(cudaMemcpyAsync(hv, state_.vc + off, bytes, cudaMemcpyDeviceToHost, stream_), "memcpy");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  return QWEN_OK;
}

int QwenEngine::set_kv(int32_t seq, int32_t layer, int32_t n_pos, const uint16_t* hk,
                       const uint16_t* hv) {
  if (seq < 0 || seq >= state_.batch || layer < 0 || layer >= state_.n_layers || n_pos < 0 ||
      n_pos > state_.max_ctx)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "set_kv: bad arguments");
  QWEN_CUDA(cudaSetDevice(cfg_.device), "cudaSetDevice");
  const size_t off = (size_t)layer * state_.kv_layer_stride() + (size_t)seq * state_.kv_seq_stride();
  const size_t bytes = (size_t)n_pos * kKVDim * 2;
  if (hk) QWEN_CUDA(cudaMemcpyAsync(state_.kc + off, hk, bytes, cudaMemcpyHostToDevice, stream_), "memcpy");
  if (hv) QWEN_CUDA(cudaMemcpyAsync(state_.vc + off, hv, bytes, cudaMemcpyHostToDevice, stream_), "memcpy");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  return QWEN_OK;
}

int QwenEngine::position(int32_t seq, int32_t* pos) {
  if (seq < 0 || seq >= state_.batch) return set_error(QWEN_ERR_INVALID_ARGUMENT, "bad sequence %d", seq);
  SeqCtl c;
  QWEN_CUDA(cudaMemcpyAsync(&c, state_.ctl + seq, sizeof(c), cudaMemcpyDeviceToHost, stream_), "memcpy");
  QWEN_CUDA(cudaStreamSynchronize(stream_), "sync");
  *pos = c.pos;
  return QWEN_OK;
}

}  // namespace qwen

// ------------------------------------------------------------------ C ABI --
struct qwen_engine {
  qwen::QwenEngine impl;
};

using qwen::set_error;

extern "C" {

void qwen_engine_config_default(qwen_engine_config* c) {
  if (!c) return;
  c->device = 0;
  c->max_ctx = 1024;
  c->batch = 1;
  c->n_layers = 28;
  c->kernels = QWEN_KERNELS_FUSED;
  c->temperature = 0.7f;
  c->top_p = 0.8f;
  c->seed = 0;
  c->stop_on_eos = 1;
  c->ctx_overflow = QWEN_CTX_CLAMP;
  c->prefill_mode = QWEN_PREFILL_CHUNKED;
}

int qwen_engine_create(const qwen_engine_config* cfg, qwen_engine** out) {
  if (!cfg || !out) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  auto* e = new (std::nothrow) qwen_engine();
  if (!e) return set_error(QWEN_ERR_OUT_OF_MEMORY, "host allocation failed");
  const int rc = e->impl.init(*cfg);
  if (rc != QWEN_OK) {
    delete e;
    return rc;
  }
  *out = e;
  return QWEN_OK;
}

int qwen_engine_destroy(qwen_engine* e) {
  delete e;
  return QWEN_OK;
}

#define ENGINE_OR_FAIL(e) \
  if (!(e)) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null engine")

int qwen_engine_load_weights(qwen_engine* e, const char* dir) {
  ENGINE_OR_FAIL(e);
  if (!dir) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null path");
  return e->impl.load_weights(dir);
}
int qwen_engine_init_random(qwen_engine* e, uint64_t seed) {
  ENGINE_OR_FAIL(e);
  return e->impl.init_random(seed);
}
int qwen_engine_reset(qwen_engine* e) {
  ENGINE_OR_FAIL(e);
  return e->impl.reset();
}
int qwen_engine_forward(qwen_engine* e, int32_t token, int32_t position, int32_t* next) {
  ENGINE_OR_FAIL(e);
  if (!next) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null output");
  return e->impl.forward(token, position, next);
}
int qwen_engine_generate(qwen_engine* e, const int32_t* prompt, int32_t n_prompt, int32_t max_tokens,
                         int32_t* out, int32_t* n_out) {
  ENGINE_OR_FAIL(e);
  if (!prompt || !out || !n_out) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null buffer");
  return e->impl.generate(prompt, n_prompt, max_tokens, out, n_out);
}
int qwen_engine_decode(qwen_engine* e, int32_t n_steps, int32_t* out) {
  ENGINE_OR_FAIL(e);
  return e->impl.decode(n_steps, out);
}
int qwen_engine_prefill(qwen_engine* e, const int32_t* prompt, int32_t n_prompt) {
  ENGINE_OR_FAIL(e);
  if (!prompt) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null prompt");
  return e->impl.prefill(prompt, n_prompt);
}
int qwen_engine_get_logits(qwen_engine* e, int32_t seq, uint16_t* host) {
  ENGINE_OR_FAIL(e);
  if (!host) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null buffer");
  return e->impl.get_logits(seq, host);
}
int qwen_engine_get_kv(qwen_engine* e, int32_t seq, int32_t layer, int32_t n_pos, uint16_t* hk,
                       uint16_t* hv) {
  ENGINE_OR_FAIL(e);
  return e->impl.get_kv(seq, layer, n_pos, hk, hv);
}
int qwen_engine_set_kv(qwen_engine* e, int32_t seq, int32_t layer, int32_t n_pos,
                       const uint16_t* hk, const uint16_t* hv) {
  ENGINE_OR_FAIL(e);
  return e->impl.set_kv(seq, layer, n_pos, hk, hv);
}
int qwen_engine_position(qwen_engine* e, int32_t seq, int32_t* pos) {
  ENGINE_OR_FAIL(e);
  if (!pos) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null output");
  return e->impl.position(seq, pos);
}
int qwen_engine_kernels_per_step(qwen_engine* e, int32_t* n) {
  ENGINE_OR_FAIL(e);
  if (!n) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null output");
  int v = 0;
  const int rc = e->impl.kernels_per_step(&v);
  *n = v;
  return rc;
}
int qwen_engine_trace(qwen_engine* e, int32_t enable) {
  ENGINE_OR_FAIL(e);
  return e->impl.set_trace(enable);
}
int qwen_engine_get_trace(qwen_engine* e, uint64_t* host, size_t n, size_t* needed) {
  ENGINE_OR_FAIL(e);
  if (!needed) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null output");
  return e->impl.get_trace(reinterpret_cast<unsigned long long*>(host), n, needed);
}
int qwen_engine_time_steps(qwen_engine* e, int32_t n_steps, float* ms_step, float* ms_model) {
  ENGINE_OR_FAIL(e);
  if (!ms_step || !ms_model) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null output");
  return e->impl.time_steps(n_steps, ms_step, ms_model);
}
int qwen_engine_profile_step(qwen_engine* e, float* ms, int32_t cap, int32_t* n) {
  ENGINE_OR_FAIL(e);
  if (!n) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null output");
  int v = 0;
  const int rc = e->impl.profile_step(ms, cap, &v);
  *n = v;
  return rc;
}
int qwen_engine_set_wait_timeout(qwen_engine* e, uint64_t timeout_ns) {
  ENGINE_OR_FAIL(e);
  return e->impl.set_wait_timeout(timeout_ns);
}
int qwen_engine_test_stall(qwen_engine* e, int32_t site) {
  ENGINE_OR_FAIL(e);
  return e->impl.test_stall(site);
}
int qwen_engine_stream(qwen_engine* e, void** stream) {
  ENGINE_OR_FAIL(e);
  if (!stream) return set_error(QWEN_ERR_INVALID_ARGUMENT, "null output");
  *stream = e->impl.stream();
  return QWEN_OK;
}

}  // extern "C"
