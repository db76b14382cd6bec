// capi_ops.cu -- extern "C" operator entry points of libqwen_b200.so
// (declared in include/qwen_b200.h) and the library's error reporting.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/qwen_b200.h"
#include "qwen_common.cuh"
#include "qwen_internal.h"
#include "status.h"

namespace qwen {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return QWEN_OK;
  int code = QWEN_ERR_CUDA;
  if (e == cudaErrorMemoryAllocation) code = QWEN_ERR_OUT_OF_MEMORY;
  if (e == cudaErrorNoDevice || e == cudaErrorInvalidDevice || e == cudaErrorInsufficientDriver)
    code = QWEN_ERR_NO_DEVICE;
  return set_error(code, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int launch_status(const char* what) { return cuda_status(cudaGetLastError(), what); }

// Per-device state the stateless operator entry points share: the RoPE
// frequency table (constant memory, per device) and scratch for the
// attention and sampler kernels, grown on demand and kept until exit.
struct OpDeviceState {
  bool rope_ready = false;
  void* attn_scratch = nullptr;
  size_t attn_scratch_bytes = 0;
};
static std::mutex g_ops_mu;
static std::unordered_map<int, OpDeviceState> g_ops;

static int current_device(int* dev) { return cuda_status(cudaGetDevice(dev), "cudaGetDevice"); }

int ensure_rope_table() {
  int dev;
  if (int rc = current_device(&dev)) return rc;
  std::lock_guard<std::mutex> lk(g_ops_mu);
  OpDeviceState& st = g_ops[dev];
  if (!st.rope_ready) {
    float inv[64];
    rope_inv_freq(inv);
    if (set_rope_inv_freq(inv) != 0) return set_error(QWEN_ERR_CUDA, "cannot set RoPE table");
    st.rope_ready = true;
  }
  return QWEN_OK;
}

static int attn_scratch(size_t bytes, void** out) {
  int dev;
  if (int rc = current_device(&dev)) return rc;
  std::lock_guard<std::mutex> lk(g_ops_mu);
  OpDeviceState& st = g_ops[dev];
  if (st.attn_scratch_bytes < bytes) {
    if (st.attn_scratch) cudaFree(st.attn_scratch);
    st.attn_scratch = nullptr;
    st.attn_scratch_bytes = 0;
    if (int rc = cuda_status(cudaMalloc(&st.attn_scratch, bytes), "cudaMalloc(attention scratch)"))
      return rc;
    if (int rc = cuda_status(cudaMemset(st.attn_scratch, 0, bytes), "cudaMemset")) return rc;
    st.attn_scratch_bytes = bytes;
  }
  *out = st.attn_scratch;
  return QWEN_OK;
}

}  // namespace qwen

using namespace qwen;

#define H(p) reinterpret_cast<const __half*>(p)
#define HM(p) reinterpret_cast<__half*>(p)

extern "C" {

const char* qwen_last_error(void) { return g_last_error.c_str(); }
int qwen_abi_version(void) { return 2; }

int qwen_gemv_q4_0(const uint8_t* packed, const uint16_t* scales, const uint16_t* x, uint16_t* y,
                   uint32_t k, const uint16_t* bias, uint32_t n_rows, void* stream) {
  if (!packed || !scales || !x || !y) return set_error(QWEN_ERR_INVALID_ARGUMENT, "gemv_q4_0: null buffer");
  if (k == 0 || k % 32 != 0 || k > 65536)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "gemv_q4_0: k=%u must be a positive multiple of 32 (<= 65536)", k);
  if (n_rows == 0) return QWEN_OK;
  launch_gemv_q4_rowmajor(packed, H(scales), H(x), HM(y), H(bias), (int)n_rows, (int)k, stream);
  return launch_status("gemv_q4_0");
}

int qwen_gemv_fp16(const uint16_t* w, const uint16_t* x, uint16_t* y, uint32_t k, uint32_t n_rows,
                   void* stream) {
  if (!w || !x || !y) return set_error(QWEN_ERR_INVALID_ARGUMENT, "gemv_fp16: null buffer");
  if (k == 0 || k % 16 != 0) return set_error(QWEN_ERR_INVALID_ARGUMENT, "gemv_fp16: k=%u must be a multiple of 16", k);
  if (n_rows == 0) return QWEN_OK;
  launch_gemv_fp16_rowmajor(H(w), H(x), HM(y), (int)n_rows, (int)k, stream);
  return launch_status("gemv_fp16");
}

int qwen_rms_norm_q4(const uint16_t* x, const uint16_t* gamma, uint16_t* out, void* stream) {
  if (!x || !gamma || !out) return set_error(QWEN_ERR_INVALID_ARGUMENT, "rms_norm_q4: null buffer");
  launch_rms_norm(H(x), H(gamma), HM(out), stream);
  return launch_status("rms_norm_q4");
}

int qwen_apply_rope_q4(uint16_t* vec, uint32_t n_heads, const uint32_t* seq_len, void* stream) {
  if (!vec || !seq_len) return set_error(QWEN_ERR_INVALID_ARGUMENT, "apply_rope_q4: null buffer");
  if (n_heads == 0 || n_heads > 1024) return set_error(QWEN_ERR_INVALID_ARGUMENT, "apply_rope_q4: n_heads=%u", n_heads);
  if (int rc = ensure_rope_table()) return rc;
  launch_rope(HM(vec), (int)n_heads, seq_len, stream);
  return launch_status("apply_rope_q4");
}

int qwen_write_kv_cache(const uint16_t* k, const uint16_t* v, uint16_t* k_cache, uint16_t* v_cache,
                        const uint32_t* seq_len, uint32_t max_ctx, void* stream) {
  if (!k || !v || !k_cache || !v_cache || !seq_len)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "write_kv_cache: null buffer");
  launch_write_kv_cache(H(k), H(v), HM(k_cache), HM(v_cache), seq_len, max_ctx, stream);
  return launch_status("write_kv_cache");
}

int qwen_attention_scores(const uint16_t* q, const uint16_t* k_cache, float* scores,
                          const uint32_t* seq_len, uint32_t max_ctx, void* stream) {
  if (!q || !k_cache || !scores || !seq_len)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "attention_scores: null buffer");
  if (max_ctx == 0) return set_error(QWEN_ERR_INVALID_ARGUMENT, "attention_scores: max_ctx=0");
  launch_attention_scores(H(q), H(k_cache), scores, seq_len, max_ctx, stream);
  return launch_status("attention_scores");
}

int qwen_softmax(float* scores, const uint32_t* seq_len, void* stream) {
  if (!scores || !seq_len) return set_error(QWEN_ERR_INVALID_ARGUMENT, "softmax: null buffer");
  launch_softmax(scores, seq_len, stream);
  return launch_status("softmax");
}

int qwen_attn_weighted_sum(const float* scores, const uint16_t* v_cache, uint16_t* out,
                           const uint32_t* seq_len, void* stream) {
  if (!scores || !v_cache || !out || !seq_len)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "attn_weighted_sum: null buffer");
  launch_attn_weighted_sum(scores, H(v_cache), HM(out), seq_len, stream);
  return launch_status("attn_weighted_sum");
}

int qwen_residual_add(const uint16_t* a, const uint16_t* b, uint16_t* out, uint32_t n, void* stream) {
  if (!a || !b || !out) return set_error(QWEN_ERR_INVALID_ARGUMENT, "residual_add: null buffer");
  if (n == 0) return QWEN_OK;
  launch_residual_add(H(a), H(b), HM(out), (int)n, stream);
  return launch_status("residual_add");
}

int qwen_swiglu(uint16_t* gate, const uint16_t* up, uint32_t n, void* stream) {
  if (!gate || !up) return set_error(QWEN_ERR_INVALID_ARGUMENT, "swiglu: null buffer");
  if (n == 0) return QWEN_OK;
  launch_swiglu(HM(gate), H(up), (int)n, stream);
  return launch_status("swiglu");
}

int qwen_attention_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                          uint16_t* out, const uint32_t* seq_len, uint32_t max_ctx, void* stream) {
  if (!q || !k_cache || !v_cache || !out || !seq_len)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "attention_decode: null buffer");
  if (max_ctx == 0 || max_ctx > (1u << 20))
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "attention_decode: max_ctx=%u", max_ctx);
  const int splits = attn_max_splits((int)max_ctx, 1);
  void* scratch = nullptr;
  if (int rc = attn_scratch(attn_scratch_bytes(splits, 1), &scratch)) return rc;
  AttnParams p{};
  p.q = H(q);
  p.q_seq_stride = kHidden;
  p.k = H(k_cache);
  p.v = H(v_cache);
  p.kv_seq_stride = 0;
  p.kv_pos_stride = kKVDim;
  p.kv_head_stride = kHeadDim;
  p.seq_len = seq_len;
  p.seq_len_stride = 1;
  p.max_ctx = max_ctx;
  p.out = HM(out);
  p.out_seq_stride = kHidden;
  if (int rc = ops_status_word(&p.err)) return rc;
  attn_bind_scratch(p, scratch, splits, 1);
  if (launch_attention_decode(p, splits, 1, reinterpret_cast<cudaStream_t>(stream)) != 0)
    return set_error(QWEN_ERR_CUDA, "attention_decode: launch failed (%s)",
                     cudaGetErrorString(cudaGetLastError()));
  return launch_status("attention_decode");
}

int qwen_dequant_q4(const uint8_t* packed, const uint16_t* scales, size_t n_weights, float* out,
                    void* stream) {
  if (!packed || !scales || !out) return set_error(QWEN_ERR_INVALID_ARGUMENT, "dequant_q4: null buffer");
  if (n_weights % 32 != 0) return set_error(QWEN_ERR_INVALID_ARGUMENT, "dequant_q4: n_weights must be a multiple of 32");
  if (n_weights == 0) return QWEN_OK;
  launch_dequant_q4(packed, H(scales), n_weights, out, stream);
  return launch_status("dequant_q4");
}

int qwen_quantize_q4(const float* w, size_t n, uint8_t* packed, uint16_t* scales, void* stream) {
  if (!w || !packed || !scales) return set_error(QWEN_ERR_INVALID_ARGUMENT, "quantize_q4: null buffer");
  if (n == 0) return QWEN_OK;
  launch_quantize_q4(w, n, packed, HM(scales), reinterpret_cast<cudaStream_t>(stream));
  return launch_status("quantize_q4");
}

int qwen_sample(const uint16_t* logits, uint32_t n_seq, uint32_t row_stride, uint32_t vocab,
                float temperature, float top_p, const uint32_t* u24, int32_t* out_ids, void* stream) {
  if (!logits || !out_ids) return set_error(QWEN_ERR_INVALID_ARGUMENT, "sample: null buffer");
  if (vocab == 0 || vocab > (uint32_t)kVocab || row_stride < vocab)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "sample: vocab=%u row_stride=%u", vocab, row_stride);
  if (temperature > 0.0f && !u24) return set_error(QWEN_ERR_INVALID_ARGUMENT, "sample: top-p needs u24");
  if (n_seq == 0) return QWEN_OK;
  if (n_seq > 65535) return set_error(QWEN_ERR_INVALID_ARGUMENT, "sample: n_seq=%u", n_seq);
  int* status = nullptr;
  if (int rc = ops_status_word(&status)) return rc;
  if (launch_sample(H(logits), (int)n_seq, (int)row_stride, (int)vocab, temperature, top_p, u24,
                    out_ids, nullptr, status, reinterpret_cast<cudaStream_t>(stream)) != 0)
    return launch_status("sample");
  return QWEN_OK;
}

size_t qwen_sample_scratch_bytes(uint32_t n_seq) { return sampler_scratch_bytes((int)n_seq); }

int qwen_sample_scratch(const uint16_t* logits, uint32_t n_seq, uint32_t row_stride, uint32_t vocab,
                        float temperature, float top_p, const uint32_t* u24, int32_t* out_ids,
                        void* scratch, void* stream) {
  if (!logits || !out_ids) return set_error(QWEN_ERR_INVALID_ARGUMENT, "sample: null buffer");
  if (vocab == 0 || vocab > (uint32_t)kVocab || row_stride < vocab)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "sample: vocab=%u row_stride=%u", vocab, row_stride);
  if (temperature > 0.0f && !u24) return set_error(QWEN_ERR_INVALID_ARGUMENT, "sample: top-p needs u24");
  if (sampler_scratch_bytes((int)n_seq) && !scratch)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "sample: null scratch");
  if (n_seq == 0) return QWEN_OK;
  if (n_seq > 65535) return set_error(QWEN_ERR_INVALID_ARGUMENT, "sample: n_seq=%u", n_seq);
  int* status = nullptr;
  if (int rc = ops_status_word(&status)) return rc;
  if (launch_sample(H(logits), (int)n_seq, (int)row_stride, (int)vocab, temperature, top_p, u24,
                    out_ids, scratch, status, reinterpret_cast<cudaStream_t>(stream)) != 0)
    return launch_status("sample");
  return QWEN_OK;
}

uint32_t qwen_uniform24(uint64_t seed, uint64_t sequence, uint64_t step) {
  return uniform24(seed, sequence, step);
}

}  // extern "C"
