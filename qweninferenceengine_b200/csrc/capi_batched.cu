// capi_batched.cu -- C ABI for the batched tensor-core projections
// (declared in include/qwen_b200.h).
#include "../../include/qwen_b200.h"
#include "qwen_common.cuh"
#include "qwen_internal.h"
#include "status.h"
#include "tc_gemm.h"

using namespace qwen;

namespace {

struct StreamBuffers {
  cudaStream_t st;
  void* p[3] = {nullptr, nullptr, nullptr};
  explicit StreamBuffers(cudaStream_t s) : st(s) {}
  ~StreamBuffers() {
    for (void* q : p)
      if (q) cudaFreeAsync(q, st);
  }
};

int check_shape(const char* op, uint32_t k, uint32_t n_rows, uint32_t n_batch) {
  if (k == 0 || k % kTcChunkK != 0 || k > 65536)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "%s: k=%u must be a positive multiple of 64", op, k);
  if (n_rows % kTcM != 0)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "%s: n_rows=%u must be a multiple of 128", op, n_rows);
  if (n_batch < 1 || n_batch > (uint32_t)kTcMaxNb)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "%s: n_batch=%u out of range [1, 256]", op, n_batch);
  return QWEN_OK;
}

int sm_count_of_current(int* n) {
  int dev = 0;
  QWEN_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  QWEN_CUDA(cudaDeviceGetAttribute(n, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
  return QWEN_OK;
}

// Shared driver: activations packed, GEMM with K splits, splits summed (+bias).
int run_batched(bool q4, const uint8_t* blob, const uint16_t* x, uint16_t* y, uint32_t k,
                const uint16_t* bias, uint32_t n_rows, uint32_t n_batch, StreamBuffers& buf) {
  int sms = 0;
  QWEN_TRY(sm_count_of_current(&sms));
  const int nb = act_rows((int)n_batch);
  QWEN_CUDA(cudaMallocAsync(&buf.p[1], act_bytes(nb, (int)k), buf.st), "cudaMallocAsync(act)");
  if (launch_pack_act(reinterpret_cast<const __half*>(x), k, (int)n_batch, (int)k, nb,
                      static_cast<uint8_t*>(buf.p[1]), buf.st) != 0)
    return launch_status("pack activations");
  const int tiles = (int)n_rows / kTcM, chunks = (int)k / kTcChunkK;
  const int splits = tc_choose_splits(tiles, chunks, sms);
  QWEN_CUDA(cudaMallocAsync(&buf.p[2], (size_t)splits * n_batch * n_rows * sizeof(float), buf.st),
            "cudaMallocAsync(partials)");
  TcGemmArgs a;
  a.w = blob;
  a.q4 = q4;
  a.act = static_cast<const uint8_t*>(buf.p[1]);
  a.nb = nb;
  a.nb_valid = (int)n_batch;
  a.n_rows = (int)n_rows;
  a.k = (int)k;
  a.splits = splits;
  a.part = static_cast<float*>(buf.p[2]);
  if (launch_tc_gemm(a, buf.st) != 0) return launch_status("tc gemm launch");
  if (launch_splits_to_f16(a.part, splits, (int)n_batch, (int)n_rows,
                           reinterpret_cast<const __half*>(bias), reinterpret_cast<__half*>(y),
                           n_rows, buf.st) != 0)
    return launch_status("tc gemm splits");
  return launch_status("gemm batched");
}

}  // namespace

extern "C" {

int qwen_gemm_q4_0_batched(const uint8_t* packed, const uint16_t* scales, const uint16_t* x,
                           uint16_t* y, uint32_t k, const uint16_t* bias, uint32_t n_rows,
                           uint32_t n_batch, void* stream) {
  if (!packed || !scales || !x || !y)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "gemm_q4_0_batched: null buffer");
  QWEN_TRY(check_shape("gemm_q4_0_batched", k, n_rows, n_batch));
  if (n_rows == 0) return QWEN_OK;
  StreamBuffers buf(static_cast<cudaStream_t>(stream));
  QWEN_CUDA(cudaMallocAsync(&buf.p[0], q4_tc_blob_bytes((int)n_rows, (int)k), buf.st),
            "cudaMallocAsync(blob)");
  if (launch_repack_q4_tc(packed, reinterpret_cast<const __half*>(scales), (int)n_rows, (int)k,
                          static_cast<uint8_t*>(buf.p[0]), buf.st) != 0)
    return launch_status("repack q4");
  return run_batched(true, static_cast<const uint8_t*>(buf.p[0]), x, y, k, bias, n_rows, n_batch,
                     buf);
}

int qwen_gemm_fp16_batched(const uint16_t* w, const uint16_t* x, uint16_t* y, uint32_t k,
                           uint32_t n_rows, uint32_t n_batch, void* stream) {
  if (!w || !x || !y) return set_error(QWEN_ERR_INVALID_ARGUMENT, "gemm_fp16_batched: null buffer");
  QWEN_TRY(check_shape("gemm_fp16_batched", k, n_rows, n_batch));
  if (n_rows == 0) return QWEN_OK;
  StreamBuffers buf(static_cast<cudaStream_t>(stream));
  QWEN_CUDA(cudaMallocAsync(&buf.p[0], f16_tc_blob_bytes((int)n_rows, (int)k), buf.st),
            "cudaMallocAsync(blob)");
  if (launch_repack_f16_tc(reinterpret_cast<const __half*>(w), (int)n_rows, (int)k,
                           static_cast<uint8_t*>(buf.p[0]), buf.st) != 0)
    return launch_status("repack fp16");
  return run_batched(false, static_cast<const uint8_t*>(buf.p[0]), x, y, k, nullptr, n_rows,
                     n_batch, buf);
}

int qwen_attention_decode_batched(const uint16_t* q, const uint16_t* k_cache,
                                  const uint16_t* v_cache, uint16_t* out,
                                  const uint32_t* seq_len, uint32_t n_seq, uint32_t max_ctx,
                                  void* stream) {
  if (!q || !k_cache || !v_cache || !out || !seq_len)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "attention_decode_batched: null buffer");
  if (max_ctx == 0 || max_ctx > (1u << 20))
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "attention_decode_batched: max_ctx=%u", max_ctx);
  if (n_seq == 0 || n_seq > 65535)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "attention_decode_batched: n_seq=%u", n_seq);
  StreamBuffers buf(static_cast<cudaStream_t>(stream));
  const int splits = attn_max_splits((int)max_ctx, (int)n_seq);
  const size_t bytes = attn_scratch_bytes(splits, (int)n_seq);
  QWEN_CUDA(cudaMallocAsync(&buf.p[0], bytes, buf.st), "cudaMallocAsync(attention scratch)");
  QWEN_CUDA(cudaMemsetAsync(buf.p[0], 0, bytes, buf.st), "cudaMemsetAsync");
  AttnParams p{};
  p.q = reinterpret_cast<const __half*>(q);
  p.q_seq_stride = kHidden;
  p.k = reinterpret_cast<const __half*>(k_cache);
  p.v = reinterpret_cast<const __half*>(v_cache);
  p.kv_seq_stride = (long long)max_ctx * kKVDim;
  p.kv_pos_stride = kKVDim;
  p.kv_head_stride = kHeadDim;
  p.seq_len = seq_len;
  p.seq_len_stride = 1;
  p.max_ctx = max_ctx;
  p.out = reinterpret_cast<__half*>(out);
  p.out_seq_stride = kHidden;
  attn_bind_scratch(p, buf.p[0], splits, (int)n_seq);
  if (launch_attention_decode(p, splits, (int)n_seq, buf.st) != 0)
    return set_error(QWEN_ERR_CUDA, "attention_decode_batched: launch failed (%s)",
                     cudaGetErrorString(cudaGetLastError()));
  return launch_status("attention_decode_batched");
}

}  // extern "C"
