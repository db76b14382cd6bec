// attention_noalloc.cu -- qwen_attention_decode_noalloc: the split-K decode
// attention of qwen_attention_decode, with its scratch (per-split partial
// results and the merge tickets) in a fixed device array owned by this library
// instead of memory it allocates.
//
// For callers that cannot allocate device memory: code running while another
// component has a stream in global capture mode (cudaMalloc is illegal
// there), latency-critical threads that must not enter the CUDA allocator
// (it can synchronise the device or take a process-wide lock), and plugins in
// hosts that reserve the whole device memory pool for themselves.
//
// Limits and sharing:
//   * The array holds kNoAllocScratchBytes (1 MiB) on every GPU that loads this
//     library, for the life of the process.  One sequence at a time needs at
//     most 256 + 2 * 32 * 780 * 4 bytes (199,936 B), for any max_ctx up to 2^20;
//     larger requests are rejected with QWEN_ERR_INVALID_ARGUMENT.
//   * Every call on a device shares the same array and leaves its contents
//     behind.  The merge tickets that must start at zero are cleared on the
//     caller's stream before each launch.  Calls that overlap on the GPU (two
//     streams, or two host threads) race on the array: serialise them.
//   * The first call on a device (and the first after the device's context
//     changes, e.g. after cudaDeviceReset) looks up the array's device address
//     with cudaGetSymbolAddress, with that device current, and caches it per
//     context; make that first call before any stream capture.
//   * A device-side failure (a bounded wait that gave up, a length beyond
//     max_ctx) is recorded in the operator status word, which qwen_ops_status
//     reports; that word is a __device__ array too, so recording it allocates
//     nothing either.
#include "../../include/qwen_b200.h"
#include "qwen_common.cuh"
#include "qwen_internal.h"
#include "status.h"

namespace qwen {

constexpr size_t kNoAllocScratchBytes = (size_t)1 << 20;

// Device-side scratch.  In host code this name is only a stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_attn_noalloc_scratch[kNoAllocScratchBytes];

static DeviceSymbolCache g_noalloc_cache;

// Set-up, with the device current: the array's device address.
static int lookup_scratch(void** p) {
  return cuda_status(cudaGetSymbolAddress(p, g_attn_noalloc_scratch),
                     "cudaGetSymbolAddress(attention scratch)");
}

static int noalloc_scratch_address(void** out) {
  return symbol_address_cached(g_noalloc_cache, lookup_scratch, out);
}

}  // namespace qwen

using namespace qwen;

extern "C" int qwen_attention_decode_noalloc(const uint16_t* q, const uint16_t* k_cache,
                                             const uint16_t* v_cache, uint16_t* out,
                                             const uint32_t* seq_len, uint32_t max_ctx,
                                             void* stream) {
  if (!q || !k_cache || !v_cache || !out || !seq_len)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "attention_decode_noalloc: null buffer");
  if (max_ctx == 0 || max_ctx > (1u << 20))
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "attention_decode_noalloc: max_ctx=%u", max_ctx);
  const int splits = attn_max_splits((int)max_ctx, 1);
  const size_t need = attn_scratch_bytes(splits, 1);
  if (need > kNoAllocScratchBytes)
    return set_error(QWEN_ERR_INVALID_ARGUMENT,
                     "attention_decode_noalloc: needs %zu scratch bytes, the fixed array holds %zu",
                     need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch_address(&scratch)) return rc;
  AttnParams p{};
  p.q = reinterpret_cast<const __half*>(q);
  p.q_seq_stride = kHidden;
  p.k = reinterpret_cast<const __half*>(k_cache);
  p.v = reinterpret_cast<const __half*>(v_cache);
  p.kv_seq_stride = 0;
  p.kv_pos_stride = kKVDim;
  p.kv_head_stride = kHeadDim;
  p.seq_len = seq_len;
  p.seq_len_stride = 1;
  p.max_ctx = max_ctx;
  p.out = reinterpret_cast<__half*>(out);
  p.out_seq_stride = kHidden;
  if (int rc = ops_status_word(&p.err)) return rc;
  attn_bind_scratch(p, scratch, splits, 1);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // The merge tickets must start at zero (an earlier call that failed part
  // way could have left them set).
  if (int rc = cuda_status(cudaMemsetAsync(p.counters, 0, kKVHeads * sizeof(uint32_t), st),
                           "cudaMemsetAsync(attention tickets)"))
    return rc;
  if (launch_attention_decode(p, splits, 1, st) != 0)
    return set_error(QWEN_ERR_CUDA, "attention_decode_noalloc: launch failed (%s)",
                     cudaGetErrorString(cudaGetLastError()));
  return launch_status("attention_decode_noalloc");
}
