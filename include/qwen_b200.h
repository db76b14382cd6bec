/*
 * qwen_b200.h -- C ABI of the B200 decode engine for the Qwen2.5-1.5B
 * architecture with Q4 block-32 weights (libqwen_b200.so).
 *
 * Plain C types only: device buffers are raw pointers, fp16 values are
 * uint16_t bit patterns, streams are cudaStream_t passed as void*.  Every
 * entry point returns a status (QWEN_OK == 0); qwen_last_error() gives a
 * thread-local message for the last failure.  Nothing here exits or aborts.
 * Operator entry points return once their kernels are enqueued: a failure
 * only the device can see (a bounded wait that gave up, a device-resident
 * length out of range) is recorded on the device and reported by
 * qwen_ops_status().  Engine calls synchronise and report such failures
 * themselves.
 *
 * Each declaration names the reference interface it replaces
 * (Raiden-Makoto/QwenInferenceEngine, file:line).
 */
#ifndef QWEN_B200_H
#define QWEN_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------
 * The reference throws WeightLoadingError.fileNotFound / bufferCreationFailed
 * (WeightLoader.swift:11-14) and MetalSetupError (MetalManager.swift:12-18)
 * and calls fatalError on device failures (InferenceEngine.swift:18,63,84,88);
 * here each of those is a status code. */
#define QWEN_OK 0
#define QWEN_ERR_INVALID_ARGUMENT 1
#define QWEN_ERR_CUDA 2
#define QWEN_ERR_FILE_NOT_FOUND 3   /* WeightLoadingError.fileNotFound */
#define QWEN_ERR_BAD_WEIGHT_FILE 4  /* WeightLoadingError.bufferCreationFailed, wrong size */
#define QWEN_ERR_OUT_OF_MEMORY 5
#define QWEN_ERR_DEVICE_TIMEOUT 6   /* a bounded device-side wait gave up */
#define QWEN_ERR_NO_DEVICE 7        /* MetalSetupError.deviceInitializationFailed */
#define QWEN_ERR_STATE 8            /* call order (e.g. forward before weights) */

const char* qwen_last_error(void);
int qwen_abi_version(void);

/* Synchronises `stream` and reports the first device-side failure recorded by
 * an operator kernel on the current device since the last call (then clears
 * it): QWEN_ERR_DEVICE_TIMEOUT for a bounded wait that gave up,
 * QWEN_ERR_INVALID_ARGUMENT for a device-resident length out of range, else
 * QWEN_OK.  The reference has no asynchronous operators (every Metal command
 * buffer is waited for, InferenceEngine.swift:266-268). */
int qwen_ops_status(void* stream);

/* ======================================================================
 * Operators: one entry per reference Metal pipeline (MetalManager.swift:43-49
 * registers them; InferenceEngine.swift:107-264 binds buffers by index).
 * Arguments keep the reference buffer meaning and layout.  All pointers are
 * device pointers; work is enqueued on `stream` (NULL = default stream).
 * ====================================================================== */

/* gemv_q4_0, matmul.metal:9-73 (buffers 0..5 = packed, scales, x, y,
 * constants[K,..], bias).  packed: [n_rows][k/2] bytes, low nibble = even k;
 * scales: [n_rows][k/32] fp16; y[r] = half(sum_k ((q-8)*s) x_k + bias[r]).
 * bias may be NULL.  k must be a multiple of 32.  For k <= 3072 with 16-byte
 * aligned packed and x, the kernel is launched as a programmatic dependent of
 * the previous kernel in the stream: it fetches packed and scales before
 * waiting for that kernel (x after), so they must not be produced by a kernel
 * that lets dependents start early (griddepcontrol.launch_dependents). */
int qwen_gemv_q4_0(const uint8_t* packed, const uint16_t* scales, const uint16_t* x,
                   uint16_t* y, uint32_t k, const uint16_t* bias, uint32_t n_rows,
                   void* stream);

/* gemv_fp16, matmul.metal:75-113 (LM head, InferenceEngine.swift:259-264).
 * w: [n_rows][k] fp16 row-major; y = half(w x), fp32 accumulation. */
int qwen_gemv_fp16(const uint16_t* w, const uint16_t* x, uint16_t* y, uint32_t k,
                   uint32_t n_rows, void* stream);

/* rms_norm_q4, rmsnorm.metal:9-46: out = half(half(x*s)*gamma) over 1536. */
int qwen_rms_norm_q4(const uint16_t* x, const uint16_t* gamma, uint16_t* out, void* stream);

/* apply_rope_q4, rope.metal:12-39: in place on n_heads*128 fp16, position =
 * *seq_len - 1 (device uint32, as the reference's seqLen buffer). */
int qwen_apply_rope_q4(uint16_t* vec, uint32_t n_heads, const uint32_t* seq_len,
                       void* stream);

/* write_kv_cache, attention.metal:67-84: cache[(seq_len-1)*256 + i] = k/v[i];
 * positions >= max_ctx are skipped (the reference guards 1024). */
int qwen_write_kv_cache(const uint16_t* k, const uint16_t* v, uint16_t* k_cache,
                        uint16_t* v_cache, const uint32_t* seq_len, uint32_t max_ctx,
                        void* stream);

/* attention_scores, attention.metal:9-32: scores[h*L + t] (fp32, L = *seq_len).
 * max_ctx bounds the launch (L must not exceed it). */
int qwen_attention_scores(const uint16_t* q, const uint16_t* k_cache, float* scores,
                          const uint32_t* seq_len, uint32_t max_ctx, void* stream);
/* softmax, activations.metal:29-55 (12 heads, in place). */
int qwen_softmax(float* scores, const uint32_t* seq_len, void* stream);
/* attn_weighted_sum, attention.metal:34-56. */
int qwen_attn_weighted_sum(const float* scores, const uint16_t* v_cache, uint16_t* out,
                           const uint32_t* seq_len, void* stream);

/* residual_add, attention.metal:58-65: out = half(a + b). */
int qwen_residual_add(const uint16_t* a, const uint16_t* b, uint16_t* out, uint32_t n,
                      void* stream);
/* swiglu, activations.metal:9-27: gate = half(silu(gate) * up), in place. */
int qwen_swiglu(uint16_t* gate, const uint16_t* up, uint32_t n, void* stream);

/* Fused GQA decode attention (the engine's split-K kernel; replaces the
 * attention_scores -> softmax -> attn_weighted_sum chain,
 * InferenceEngine.swift:162-182).  q: 12x128 fp16 (after RoPE); caches in the
 * reference layout [pos][256]; L = *seq_len positions; out: 1536 fp16.
 * L outside [1, max_ctx] leaves `out` untouched and is reported by
 * qwen_ops_status. */
int qwen_attention_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                          uint16_t* out, const uint32_t* seq_len, uint32_t max_ctx,
                          void* stream);

/* qwen_attention_decode for n_seq independent sequences in one launch (the
 * tensor-core batched step's attention): q [n_seq][1536]; caches
 * [n_seq][max_ctx][256] (reference row layout per sequence); seq_len[n_seq]
 * device lengths in [1, max_ctx]; out [n_seq][1536].  Scratch from
 * stream-ordered allocations. */
int qwen_attention_decode_batched(const uint16_t* q, const uint16_t* k_cache,
                                  const uint16_t* v_cache, uint16_t* out,
                                  const uint32_t* seq_len, uint32_t n_seq, uint32_t max_ctx,
                                  void* stream);

/* qwen_attention_decode without any device allocation.  No counterpart in the
 * reference (it has no allocation-free entry points): this is for callers that
 * may not call cudaMalloc -- code running while another component holds a
 * stream in global capture mode, latency-critical threads that must stay out
 * of the CUDA allocator, plugins in hosts that own the whole memory pool.
 * Same arguments and results as qwen_attention_decode.  Its scratch is a fixed
 * 1 MiB device array inside this library (held on every GPU that loads it until
 * exit); requests needing more are rejected with QWEN_ERR_INVALID_ARGUMENT.
 * All calls on a device share that array: calls that overlap on the GPU race,
 * so serialise them.  The first call on a device (and the first after its
 * context changes) resolves the array's address and should come before any
 * stream capture.  Device-side failures go to the status word that
 * qwen_ops_status reads, itself a fixed device array. */
int qwen_attention_decode_noalloc(const uint16_t* q, const uint16_t* k_cache,
                                  const uint16_t* v_cache, uint16_t* out,
                                  const uint32_t* seq_len, uint32_t max_ctx, void* stream);

/* gemv_q4_0 (matmul.metal:9-73) for n_batch activation rows at once, on the
 * tcgen05 tensor cores: y[b][r] = half(sum_k ((q-8)*s) x[b][k] + bias[r]) for
 * b < n_batch (1..256); x is [n_batch][k], y is [n_batch][n_rows].  The weight
 * product (q-8)*s is rounded once to fp16 before the fp32-accumulating MMA.
 * n_rows a multiple of 128, k a multiple of 64.  Uses temporary device
 * memory (stream-ordered allocations) for the repacked weights. */
int qwen_gemm_q4_0_batched(const uint8_t* packed, const uint16_t* scales, const uint16_t* x,
                           uint16_t* y, uint32_t k, const uint16_t* bias, uint32_t n_rows,
                           uint32_t n_batch, void* stream);

/* gemv_fp16 (matmul.metal:75-113) for n_batch rows at once on tcgen05:
 * y[b][r] = half(sum_k w[r][k] x[b][k]).  Same shape rules as above. */
int qwen_gemm_fp16_batched(const uint16_t* w, const uint16_t* x, uint16_t* y, uint32_t k,
                           uint32_t n_rows, uint32_t n_batch, void* stream);

/* (q-8)*scale for n_weights weights, low nibble first (matmul.metal:37-42). */
int qwen_dequant_q4(const uint8_t* packed, const uint16_t* scales, size_t n_weights,
                    float* out, void* stream);

/* packAndSave4Bit, QwenPipelines.swift:97-145, on the device: symmetric
 * block-32 quantisation of n fp32 weights (flattened). */
int qwen_quantize_q4(const float* w, size_t n, uint8_t* packed, uint16_t* scales,
                     void* stream);

/* extractNextTokenID, InferenceEngine.swift:273-368, on the device.
 * logits: fp16 [n_seq][row_stride], the first `vocab` entries sampled.
 * temperature <= 0 -> greedy (:277-294).  Otherwise top-p with the fixed-point
 * nucleus rule: E_i = trunc(exp(l_i/T - max) * 2^31), keep the shortest prefix
 * of (E desc, id asc) whose sum reaches floor(sum(E) * trunc(top_p*2^24) / 2^24),
 * draw R = floor(kept * u24 / 2^24) and return the first kept id whose running
 * sum exceeds R.  u24[n_seq] are 24-bit uniforms (device).
 * out_ids: int32 [n_seq], device.
 * Each sequence runs on one thread-block cluster of 16, 8 or 4 CTAs, chosen
 * by batch size from occupancy-calculator counts that the first call on a
 * device asks for (no allocation); when capturing this call into a CUDA
 * graph, make one call on that device before the capture. */
int qwen_sample(const uint16_t* logits, uint32_t n_seq, uint32_t row_stride, uint32_t vocab,
                float temperature, float top_p, const uint32_t* u24, int32_t* out_ids,
                void* stream);

/* Device scratch bytes for qwen_sample_scratch (0 when n_seq > 1). */
size_t qwen_sample_scratch_bytes(uint32_t n_seq);

/* qwen_sample with device scratch of qwen_sample_scratch_bytes(n_seq) bytes,
 * zero before its first use (every call leaves it zero).  With one sequence
 * and temperature > 0 the sequence runs on every SM at once (a cooperative
 * launch; the CTAs exchange digit totals through the scratch), otherwise as
 * qwen_sample.  Calls that share a scratch must be ordered on one stream.
 * After a device-side wait gives up (qwen_ops_status reports
 * QWEN_ERR_DEVICE_TIMEOUT) the scratch may hold partial totals: zero it again.
 * The same ids as qwen_sample (InferenceEngine.swift:273-368); the batch-1
 * engine step samples this way. */
int qwen_sample_scratch(const uint16_t* logits, uint32_t n_seq, uint32_t row_stride, uint32_t vocab,
                        float temperature, float top_p, const uint32_t* u24, int32_t* out_ids,
                        void* scratch, void* stream);

/* 24-bit uniform for (seed, sequence, step), SplitMix64 based; host helper. */
uint32_t qwen_uniform24(uint64_t seed, uint64_t sequence, uint64_t step);

/* ======================================================================
 * Engine: QwenEngine (InferenceEngine.swift:9-52) with QwenModel /
 * QwenLayer / WeightLoader (weights) and InferenceManager (state) behind one
 * opaque handle.
 * ====================================================================== */
typedef struct qwen_engine qwen_engine;

#define QWEN_KERNELS_FUSED 0 /* fused decode step (default) */
#define QWEN_KERNELS_OPS 1   /* the reference dispatch order, one kernel per op */
#define QWEN_KERNELS_TC 2    /* batched step: every projection one tcgen05 GEMM over the batch */

typedef struct qwen_engine_config {
  int device;          /* CUDA device ordinal */
  int max_ctx;         /* KV slots per sequence (QwenConfig.maxContextWindow = 1024) */
  int batch;           /* independent sequences decoded together */
  int n_layers;        /* decoder layers (28; fewer only for tests) */
  int kernels;         /* QWEN_KERNELS_FUSED, QWEN_KERNELS_OPS or QWEN_KERNELS_TC */
  float temperature;   /* extractNextTokenID default 0.7 (:273); <= 0 -> greedy */
  float top_p;         /* default 0.8 (:273) */
  uint64_t seed;       /* uniform stream seed (the reference's RNG is unseeded) */
  int stop_on_eos;     /* generate() stops at 151645 / 151643 (:41) */
  int ctx_overflow;    /* QWEN_CTX_CLAMP (default) or QWEN_CTX_ERROR, below */
  int prefill_mode;    /* QWEN_PREFILL_CHUNKED (default) or QWEN_PREFILL_STEPS, below */
} qwen_engine_config;

/* Prompt processing.  QWEN_PREFILL_STEPS: the reference's loop, one full
 * decode step per prompt token (InferenceEngine.swift:34-36).
 * QWEN_PREFILL_CHUNKED (fused and tensor-core engines): the prompt positions of
 * every sequence run as the rows of batched tensor-core steps, a chunk at a
 * time, without the LM head and sampler except for each sequence's last
 * position, whose sample is drawn exactly as the loop's last step draws it.
 * The per-op engine (QWEN_KERNELS_OPS) always uses the loop. */
#define QWEN_PREFILL_CHUNKED 0
#define QWEN_PREFILL_STEPS 1

/* Positions past max_ctx - 1.  QWEN_CTX_CLAMP: the reference's rule,
 * min(position, maxContextWindow - 1) (InferenceEngine.swift:55) -- the step
 * overwrites the last KV slot and attends max_ctx positions.  QWEN_CTX_ERROR:
 * forward / decode / generate return QWEN_ERR_INVALID_ARGUMENT instead of
 * running such a step. */
#define QWEN_CTX_CLAMP 0
#define QWEN_CTX_ERROR 1

void qwen_engine_config_default(qwen_engine_config* cfg);

/* QwenEngine.init(weightsPath:kernelsPath:), InferenceEngine.swift:16-27:
 * selects the device and allocates state; weights come from
 * qwen_engine_load_weights or qwen_engine_init_random. */
int qwen_engine_create(const qwen_engine_config* cfg, qwen_engine** out);
int qwen_engine_destroy(qwen_engine* e);

/* QwenModel(device:weightsPath:), QwenModel.swift:22-34, with
 * WeightLoader.loadBuffer / loadLayerWeight (WeightLoader.swift:26-52): reads
 * the reference directory layout global/embed_tokens.bin, global/final_norm.bin,
 * layer{i}/{name}.bin (names QwenLayer.swift:31-51). */
int qwen_engine_load_weights(qwen_engine* e, const char* weights_dir);

/* Random-init weights on the device (linear N(0,0.02) quantised by the
 * packAndSave4Bit rule, embeddings N(0,0.02) fp16, norms 1+N(0,0.02),
 * biases N(0,0.02)). */
int qwen_engine_init_random(qwen_engine* e, uint64_t seed);

/* Clears positions (KV contents become unreachable). */
int qwen_engine_reset(qwen_engine* e);

/* forward(tokenID:position:), InferenceEngine.swift:54-271, for sequence 0 of
 * a batch-1 engine: runs one decode step, samples with the configured
 * temperature / top-p, returns the next token id.  Positions past max_ctx-1
 * are clamped as the reference does (:55). */
int qwen_engine_forward(qwen_engine* e, int32_t token, int32_t position, int32_t* next_token);

/* generate(prompt:maxTokens:), InferenceEngine.swift:29-52, on token ids for
 * every sequence of the batch: prompt_ids [batch][n_prompt]; out_ids
 * [batch][max_tokens] receives the generated ids (the reference prints them);
 * n_out[batch] how many each sequence produced. */
int qwen_engine_generate(qwen_engine* e, const int32_t* prompt_ids, int32_t n_prompt,
                         int32_t max_tokens, int32_t* out_ids, int32_t* n_out);

/* Decode `n_steps` further tokens for every sequence from the engine's current
 * state (after generate / prefill), without host synchronisation between
 * steps; writes the ids to out_ids [batch][n_steps] (host). */
int qwen_engine_decode(qwen_engine* e, int32_t n_steps, int32_t* out_ids);

/* Prefill only: consume prompt_ids [batch][n_prompt] and leave the first
 * sampled token pending (generate = prefill + decode). */
int qwen_engine_prefill(qwen_engine* e, const int32_t* prompt_ids, int32_t n_prompt);

/* fp16 logits of the last step for sequence `seq` (151936 values, host). */
int qwen_engine_get_logits(qwen_engine* e, int32_t seq, uint16_t* host_logits);

/* Copies one layer's KV cache of sequence `seq` to the host in the reference
 * layout [n_pos][256] fp16 (InferenceManager.swift:63-65). */
int qwen_engine_get_kv(qwen_engine* e, int32_t seq, int32_t layer, int32_t n_pos,
                       uint16_t* host_k, uint16_t* host_v);

/* The inverse of qwen_engine_get_kv: overwrites positions [0, n_pos) of one
 * layer's KV cache of sequence `seq` from host buffers in the reference layout
 * (either may be NULL).  For replaying a cache into the engine (the reference
 * has no such entry point; InferenceManager.swift:63-65 owns the buffers). */
int qwen_engine_set_kv(qwen_engine* e, int32_t seq, int32_t layer, int32_t n_pos,
                       const uint16_t* host_k, const uint16_t* host_v);

/* Current position (tokens consumed) of sequence `seq`. */
int qwen_engine_position(qwen_engine* e, int32_t seq, int32_t* position);

/* Kernel launches one decode step makes (all of them this library's). */
int qwen_engine_kernels_per_step(qwen_engine* e, int32_t* n);

/* Runs n_steps decode steps outside the CUDA graph with CUDA events around
 * the whole step and around the model kernels (everything between the
 * embedding gather and the sampler); returns the average milliseconds.
 * (The reference only times wall clock, main.swift:21-49.) */
int qwen_engine_time_steps(qwen_engine* e, int32_t n_steps, float* ms_step, float* ms_model);

/* Per-launch device times of one eagerly launched step of the tensor-core path
 * (QWEN_KERNELS_TC; the step advances every sequence like a decode step).
 * Launch order: rmsnorm, then per layer {qkv gemm, qkv finish, attention,
 * o gemm, o finish, gate/up gemm with SwiGLU, down gemm, down finish}, then
 * the LM head gemm; *n receives the count (1 + 8*layers + 1).
 * With ms == NULL or cap < *n only the count is returned. */
int qwen_engine_profile_step(qwen_engine* e, float* ms, int32_t cap, int32_t* n);

/* Fused-step tracing (the reference has none; main.swift:21-49 prints wall
 * clock only).  When enabled, every CTA of the fused step kernel records
 * %globaltimer stamps: [0] producer start, [1] producer done, [2] consumer
 * start, then 10 per layer at [3 + 10*layer + k]: k = 0 layer start, 1 x ready,
 * 2 QKV done, 3 attention done, 4 attention output ready, 5 O done, 6 gate/up
 * input ready, 7 gate/up done (h fragments ready), 8 the CTA's down partial
 * sums written, 9 its rows of the layer output written; then LM-head start and
 * consumer end; then 7 stamps inside the attention unit of layer n_layers/2
 * (unit start, q/k/v in, warp 0's positions done, the unit's warps merged,
 * partials written, all splits' partials in, output slice written; zero on
 * CTAs without a unit); stride 3 + 10*n_layers + 2 + 7.
 * qwen_engine_get_trace copies the last step's stamps ([grid][stride]) when
 * n >= *needed, and always reports *needed. */
int qwen_engine_trace(qwen_engine* e, int32_t enable);
int qwen_engine_get_trace(qwen_engine* e, uint64_t* host, size_t n, size_t* needed);

/* Every device-side dependency wait of the fused decode step gives up after
 * timeout_ns (default 2 s; 1 ms .. 60 s accepted), after which the step
 * finishes without its remaining work and the call that ran it returns
 * QWEN_ERR_DEVICE_TIMEOUT; the engine stays usable.  (The reference waits
 * without limit: commandBuffer.waitUntilCompleted, InferenceEngine.swift:266-268.) */
int qwen_engine_set_wait_timeout(qwen_engine* e, uint64_t timeout_ns);

/* Test hook, no reference counterpart: site 9 makes the fused step's waits for
 * the down projection's partial sums expect data that nothing writes, so the
 * waits run out and the timeout path runs; site 20 makes one CTA of the batch-1
 * grid sampler skip its arrival at the first exchange's barrier, so the other
 * CTAs' waits run out (reported as site 20, barrier 1); site 0 turns the hook
 * off.  The limit of both is qwen_engine_set_wait_timeout's. */
#define QWEN_STALL_NONE 0
#define QWEN_STALL_FUSED_DOWN 9
#define QWEN_STALL_SAMPLER 20
int qwen_engine_test_stall(qwen_engine* e, int32_t site);

/* Device and stream the engine runs on (for callers that time it). */
int qwen_engine_stream(qwen_engine* e, void** stream);

#ifdef __cplusplus
}
#endif
#endif
