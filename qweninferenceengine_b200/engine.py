"""QwenEngine: the reference's engine surface (InferenceEngine.swift:9-52) over
libqwen_b200.so.  Token ids in, token ids out; all arithmetic runs on the GPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import (QWEN_CTX_CLAMP, QWEN_CTX_ERROR, QWEN_KERNELS_FUSED, QWEN_KERNELS_OPS,
                   QWEN_KERNELS_TC, QWEN_PREFILL_CHUNKED, QWEN_PREFILL_STEPS, EngineConfig, check,
                   lib)

STOP_TOKENS = (151645, 151643)  # InferenceEngine.swift:41


@dataclass
class QwenConfig:
    """QwenConfig.swift:10-22 dimensions plus the runtime options the reference
    hard-codes (maxContextWindow, sampler defaults of InferenceEngine.swift:273)."""

    hidden_dim: int = 1536
    mlp_intermediate: int = 8960
    num_layers: int = 28
    num_attn_heads: int = 12
    num_kv_heads: int = 2
    head_dim: int = 128
    vocab_size: int = 151936
    actual_vocab_size: int = 151666
    max_context_window: int = 1024
    temperature: float = 0.7
    top_p: float = 0.8
    seed: int = 0
    batch: int = 1
    device: int = 0
    kernels: str = "fused"   # "fused", "ops" or "tc" (tensor-core batched step)
    stop_on_eos: bool = True
    ctx_overflow: str = "clamp"  # "clamp" (InferenceEngine.swift:55) or "error"
    prefill: str = "chunked"     # "chunked" (tensor cores) or "steps" (InferenceEngine.swift:34-36)


class QwenEngine:
    """QwenEngine (InferenceEngine.swift:9-369).

    QwenEngine(weights_path=...) loads the reference weight directory
    (WeightLoader.swift); QwenEngine(random_seed=...) builds a random-init model
    on the device instead."""

    def __init__(self, weights_path: str | None = None, config: QwenConfig | None = None,
                 random_seed: int | None = None):
        self.config = config or QwenConfig()
        c = self.config
        cfg = EngineConfig()
        lib().qwen_engine_config_default(ctypes.byref(cfg))
        cfg.device = c.device
        cfg.max_ctx = c.max_context_window
        cfg.batch = c.batch
        cfg.n_layers = c.num_layers
        cfg.kernels = {"fused": QWEN_KERNELS_FUSED, "ops": QWEN_KERNELS_OPS,
                       "tc": QWEN_KERNELS_TC}[c.kernels]
        cfg.temperature = c.temperature
        cfg.top_p = c.top_p
        cfg.seed = c.seed
        cfg.stop_on_eos = 1 if c.stop_on_eos else 0
        cfg.ctx_overflow = {"clamp": QWEN_CTX_CLAMP, "error": QWEN_CTX_ERROR}[c.ctx_overflow]
        cfg.prefill_mode = {"chunked": QWEN_PREFILL_CHUNKED, "steps": QWEN_PREFILL_STEPS}[c.prefill]
        h = ctypes.c_void_p()
        check(lib().qwen_engine_create(ctypes.byref(cfg), ctypes.byref(h)))
        self._h = h
        if weights_path is not None:
            check(lib().qwen_engine_load_weights(self._h, weights_path.encode()))
        elif random_seed is not None:
            check(lib().qwen_engine_init_random(self._h, random_seed))

    # -- lifecycle -----------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().qwen_engine_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- the reference surface ---------------------------------------------
    def forward(self, token_id: int, position: int) -> int:
        """forward(tokenID:position:) -> next token id (InferenceEngine.swift:54-271)."""
        out = ctypes.c_int32()
        check(lib().qwen_engine_forward(self._h, token_id, position, ctypes.byref(out)))
        return out.value

    def generate(self, prompt_ids, max_tokens: int = 64) -> list:
        """generate(prompt:maxTokens:) on token ids (InferenceEngine.swift:29-52).

        prompt_ids: [n] (batch 1) or [batch][n].  Returns the generated ids per
        sequence (a list of lists when batch > 1)."""
        p = np.ascontiguousarray(prompt_ids, dtype=np.int32)
        batched = p.ndim == 2
        if not batched:
            p = p[None, :]
        b, n = p.shape
        out = np.zeros((b, max_tokens), np.int32)
        n_out = np.zeros(b, np.int32)
        check(lib().qwen_engine_generate(self._h, p.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                         n, max_tokens,
                                         out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                         n_out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
        res = [out[i, : n_out[i]].tolist() for i in range(b)]
        return res if batched else res[0]

    def generate_text(self, prompt: str, tokenizer, max_tokens: int = 64, write=None) -> str:
        """generate(prompt:maxTokens:) on text (InferenceEngine.swift:29-52): the
        prompt (ChatML, see tokenizer.format_prompt) is encoded with a
        tokenizer.QwenTokenizer, fed through forward(), and each generated
        token's text is passed to `write` (e.g. sys.stdout.write) as it
        completes.  Returns the generated text."""
        from .tokenizer import stream_generate

        return stream_generate(self.forward, tokenizer, prompt, max_tokens, write)

    def prefill(self, prompt_ids) -> None:
        p = np.ascontiguousarray(prompt_ids, dtype=np.int32)
        if p.ndim == 1:
            p = p[None, :]
        check(lib().qwen_engine_prefill(self._h, p.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                        p.shape[1]))

    def decode(self, n_steps: int, record: bool = True) -> np.ndarray | None:
        if not record:
            check(lib().qwen_engine_decode(self._h, n_steps, None))
            return None
        out = np.zeros((self.config.batch, n_steps), np.int32)
        check(lib().qwen_engine_decode(self._h, n_steps,
                                       out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
        return out

    def reset(self) -> None:
        check(lib().qwen_engine_reset(self._h))

    # -- inspection ------------------------------------------------------------
    def logits(self, seq: int = 0) -> np.ndarray:
        out = np.zeros(self.config.vocab_size, np.uint16)
        check(lib().qwen_engine_get_logits(self._h, seq,
                                           out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))))
        return out.view(np.float16)

    def kv(self, seq: int, layer: int, n_pos: int):
        k = np.zeros((n_pos, 256), np.uint16)
        v = np.zeros((n_pos, 256), np.uint16)
        check(lib().qwen_engine_get_kv(self._h, seq, layer, n_pos,
                                       k.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)),
                                       v.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))))
        return k.view(np.float16), v.view(np.float16)

    def set_kv(self, seq: int, layer: int, k: np.ndarray, v: np.ndarray) -> None:
        """Writes positions [0, len(k)) of one layer's KV cache (fp16 [n][256])."""
        k = np.ascontiguousarray(k, np.float16).view(np.uint16)
        v = np.ascontiguousarray(v, np.float16).view(np.uint16)
        assert k.shape == v.shape and k.ndim == 2 and k.shape[1] == 256
        check(lib().qwen_engine_set_kv(self._h, seq, layer, k.shape[0],
                                       k.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)),
                                       v.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))))

    def position(self, seq: int = 0) -> int:
        out = ctypes.c_int32()
        check(lib().qwen_engine_position(self._h, seq, ctypes.byref(out)))
        return out.value

    def kernels_per_step(self) -> int:
        out = ctypes.c_int32()
        check(lib().qwen_engine_kernels_per_step(self._h, ctypes.byref(out)))
        return out.value

    def time_steps(self, n_steps: int):
        """(ms per step, ms in the model kernels) averaged over n_steps, CUDA events."""
        a, b = ctypes.c_float(), ctypes.c_float()
        check(lib().qwen_engine_time_steps(self._h, n_steps, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

    def profile_step(self) -> list:
        """Tensor-core step only: [(kernel, ms)] for one eagerly launched step, a
        CUDA event after every model kernel (advances every sequence one step)."""
        n = ctypes.c_int32()
        check(lib().qwen_engine_profile_step(self._h, None, 0, ctypes.byref(n)))
        ms = np.zeros(n.value, np.float32)
        check(lib().qwen_engine_profile_step(self._h, ms.ctypes.data_as(ctypes.c_void_p), n.value,
                                             ctypes.byref(n)))
        # a decode step: the attention forms q and the new k / v rows itself
        per_layer = ["qkv_gemm", "attention_qkv", "o_gemm", "o_finish",
                     "gu_gemm_swiglu", "down_gemm", "down_finish"]
        names = ["rmsnorm"] + per_layer * ((n.value - 2) // len(per_layer)) + ["lm_gemm"]
        return list(zip(names, ms.tolist()))

    def trace(self, enable: bool = True) -> None:
        """Per-CTA phase timestamps of the fused step (see qwen_engine_trace)."""
        check(lib().qwen_engine_trace(self._h, 1 if enable else 0))

    def get_trace(self) -> np.ndarray:
        need = ctypes.c_size_t()
        check(lib().qwen_engine_get_trace(self._h, None, 0, ctypes.byref(need)))
        out = np.zeros(need.value, np.uint64)
        check(lib().qwen_engine_get_trace(self._h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
                                          out.size, ctypes.byref(need)))
        return out

    def set_wait_timeout(self, ns: int) -> None:
        """Device wait limit of the fused step and the batch-1 sampler
        (qwen_engine_set_wait_timeout)."""
        check(lib().qwen_engine_set_wait_timeout(self._h, int(ns)))

    def test_stall(self, site: int) -> None:
        """Test hook: make device waits run out (qwen_engine_test_stall): 9, the
        fused step's wait for the down partial sums; 20, the batch-1 sampler's
        first exchange barrier; 0, off."""
        check(lib().qwen_engine_test_stall(self._h, site))

    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(lib().qwen_engine_stream(self._h, ctypes.byref(s)))
        return s.value or 0
