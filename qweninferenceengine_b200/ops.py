"""Operator entry points on torch CUDA tensors (one per reference Metal
pipeline; MetalManager.swift:43-49).  Tensors carry device memory only: each
function passes raw pointers to libqwen_b200.so and enqueues on the current
torch stream.
"""
from __future__ import annotations

import torch

from ._lib import check, lib

HIDDEN, INTER, HEADS, KV_DIM, HEAD_DIM = 1536, 8960, 12, 256, 128
VOCAB, ACTUAL_VOCAB = 151936, 151666


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def gemv_q4_0(packed: torch.Tensor, scales: torch.Tensor, x: torch.Tensor,
              bias: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """gemv_q4_0 (matmul.metal:9-73): y = half((W_deq x) + bias)."""
    k = x.numel()
    n = scales.numel() * 32 // k
    y = out if out is not None else torch.empty(n, dtype=torch.float16, device=x.device)
    check(lib().qwen_gemv_q4_0(_ptr(packed), _ptr(scales), _ptr(x), _ptr(y), k, _ptr(bias), n,
                               _stream()))
    return y


def gemv_fp16(w: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """gemv_fp16 (matmul.metal:75-113)."""
    n, k = w.shape
    y = out if out is not None else torch.empty(n, dtype=torch.float16, device=x.device)
    check(lib().qwen_gemv_fp16(_ptr(w), _ptr(x), _ptr(y), k, n, _stream()))
    return y


def gemm_q4_0_batched(packed: torch.Tensor, scales: torch.Tensor, x: torch.Tensor,
                      bias: torch.Tensor | None = None) -> torch.Tensor:
    """gemv_q4_0 (matmul.metal:9-73) for every row of x [n_batch][k] at once on
    the tcgen05 tensor cores: y [n_batch][n_rows]."""
    nb, k = x.shape
    n = scales.numel() * 32 // k
    y = torch.empty((nb, n), dtype=torch.float16, device=x.device)
    check(lib().qwen_gemm_q4_0_batched(_ptr(packed), _ptr(scales), _ptr(x), _ptr(y), k, _ptr(bias),
                                       n, nb, _stream()))
    return y


def gemm_fp16_batched(w: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """gemv_fp16 (matmul.metal:75-113) for every row of x [n_batch][k] at once."""
    n, k = w.shape
    nb = x.shape[0]
    y = torch.empty((nb, n), dtype=torch.float16, device=x.device)
    check(lib().qwen_gemm_fp16_batched(_ptr(w), _ptr(x), _ptr(y), k, n, nb, _stream()))
    return y


def rms_norm_q4(x: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
    """rms_norm_q4 (rmsnorm.metal:9-46)."""
    out = torch.empty_like(x)
    check(lib().qwen_rms_norm_q4(_ptr(x), _ptr(gamma), _ptr(out), _stream()))
    return out


def apply_rope_q4(vec: torch.Tensor, n_heads: int, seq_len: torch.Tensor) -> torch.Tensor:
    """apply_rope_q4 (rope.metal:12-39), in place; seq_len is a 1-element uint32/int32 tensor."""
    check(lib().qwen_apply_rope_q4(_ptr(vec), n_heads, _ptr(seq_len), _stream()))
    return vec


def write_kv_cache(k, v, k_cache, v_cache, seq_len, max_ctx: int) -> None:
    """write_kv_cache (attention.metal:67-84)."""
    check(lib().qwen_write_kv_cache(_ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), _ptr(seq_len),
                                    max_ctx, _stream()))


def attention_scores(q, k_cache, scores, seq_len, max_ctx: int) -> None:
    check(lib().qwen_attention_scores(_ptr(q), _ptr(k_cache), _ptr(scores), _ptr(seq_len), max_ctx,
                                      _stream()))


def softmax(scores, seq_len) -> None:
    check(lib().qwen_softmax(_ptr(scores), _ptr(seq_len), _stream()))


def attn_weighted_sum(scores, v_cache, out, seq_len) -> None:
    check(lib().qwen_attn_weighted_sum(_ptr(scores), _ptr(v_cache), _ptr(out), _ptr(seq_len),
                                       _stream()))


def residual_add(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    out = out if out is not None else torch.empty_like(a)
    check(lib().qwen_residual_add(_ptr(a), _ptr(b), _ptr(out), a.numel(), _stream()))
    return out


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """swiglu (activations.metal:9-27), in place on gate."""
    check(lib().qwen_swiglu(_ptr(gate), _ptr(up), gate.numel(), _stream()))
    return gate


def attention_decode(q, k_cache, v_cache, seq_len, max_ctx: int) -> torch.Tensor:
    """Fused split-K GQA decode attention over a reference-layout cache."""
    out = torch.empty(HIDDEN, dtype=torch.float16, device=q.device)
    check(lib().qwen_attention_decode(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out),
                                      _ptr(seq_len), max_ctx, _stream()))
    return out


def attention_decode_batched(q, k_cache, v_cache, seq_len, max_ctx: int) -> torch.Tensor:
    """attention_decode for every sequence: q [n][1536], caches [n][max_ctx][256],
    seq_len [n] (device uint32/int32)."""
    n = q.shape[0]
    out = torch.empty((n, HIDDEN), dtype=torch.float16, device=q.device)
    check(lib().qwen_attention_decode_batched(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out),
                                              _ptr(seq_len), n, max_ctx, _stream()))
    return out


def dequant_q4(packed: torch.Tensor, scales: torch.Tensor, n_weights: int) -> torch.Tensor:
    out = torch.empty(n_weights, dtype=torch.float32, device=packed.device)
    check(lib().qwen_dequant_q4(_ptr(packed), _ptr(scales), n_weights, _ptr(out), _stream()))
    return out


def quantize_q4(w: torch.Tensor):
    """packAndSave4Bit (QwenPipelines.swift:97-145) on the device."""
    w = w.contiguous().float().view(-1)
    nb = (w.numel() + 31) // 32
    packed = torch.empty(nb * 16, dtype=torch.uint8, device=w.device)
    scales = torch.empty(nb, dtype=torch.float16, device=w.device)
    check(lib().qwen_quantize_q4(_ptr(w), w.numel(), _ptr(packed), _ptr(scales), _stream()))
    return packed, scales


def sample(logits: torch.Tensor, temperature: float, top_p: float,
           u24: torch.Tensor | None = None, vocab: int = ACTUAL_VOCAB,
           scratch: torch.Tensor | None = None) -> torch.Tensor:
    """extractNextTokenID (InferenceEngine.swift:273-368) on the device.

    logits: [n_seq, row_stride] fp16; u24: [n_seq] 24-bit uniforms (int32).
    scratch: device bytes from sample_scratch(n_seq) (qwen_sample_scratch: one
    sequence over every SM); None runs qwen_sample (one cluster per sequence)."""
    if logits.dim() == 1:
        logits = logits.view(1, -1)
    n_seq, stride = logits.shape
    out = torch.empty(n_seq, dtype=torch.int32, device=logits.device)
    if scratch is None:
        check(lib().qwen_sample(_ptr(logits), n_seq, stride, vocab, temperature, top_p, _ptr(u24),
                                _ptr(out), _stream()))
    else:
        check(lib().qwen_sample_scratch(_ptr(logits), n_seq, stride, vocab, temperature, top_p,
                                        _ptr(u24), _ptr(out), _ptr(scratch), _stream()))
    return out


def sample_scratch(n_seq: int, device) -> torch.Tensor | None:
    """Zeroed scratch for sample(..., scratch=...) (None when n_seq needs none)."""
    n = lib().qwen_sample_scratch_bytes(n_seq)
    return torch.zeros(n, dtype=torch.uint8, device=device) if n else None


def uniform24(seed: int, sequence: int, step: int) -> int:
    return lib().qwen_uniform24(seed, sequence, step)
