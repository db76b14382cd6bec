"""ctypes bindings for the CPU oracle (test infrastructure only).

`Oracle` wraps oracle/liboracle.so (the C++ restatement of the reference's
arithmetic); `MetalRef` wraps oracle/_ref/libqwen_metal_ref.so (the reference's
own kernels/*.metal compiled as C++ through oracle/metal_shim).  Arrays are
numpy: fp16 data travels as np.float16 (bit patterns passed as uint16*).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_SO = os.path.join(ORACLE_DIR, "liboracle.so")
REF_SO = os.path.join(ORACLE_DIR, "_ref", "libqwen_metal_ref.so")

HIDDEN, INTER, HEADS, KV_DIM, HEAD_DIM = 1536, 8960, 12, 256, 128
VOCAB, ACTUAL_VOCAB = 151936, 151666

_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)


def _p(a: np.ndarray | None, typ):
    if a is None:
        return ctypes.cast(None, typ)
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(typ)


def ensure_oracle_built(ref: bool = False) -> None:
    target = REF_SO if ref else ORACLE_SO
    if not os.path.exists(target):
        subprocess.run(["make", "-s", "-C", ORACLE_DIR] + (["ref"] if ref else []), check=True)


class _Kernels:
    """Kernel entry points shared by the oracle and the compiled reference."""

    prefix = ""

    def __init__(self, path: str):
        self.lib = ctypes.CDLL(path)
        P = self.prefix
        L = self.lib
        getattr(L, P + "gemv_q4_0").argtypes = [_u8p, _u16p, _u16p, _u16p, _u16p,
                                                 ctypes.c_int, ctypes.c_int, ctypes.c_int]
        getattr(L, P + "gemv_fp16").argtypes = [_u16p, _u16p, _u16p, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int]
        getattr(L, P + "rms_norm").argtypes = [_u16p, _u16p, _u16p, ctypes.c_int]
        getattr(L, P + "rope").argtypes = [_u16p, ctypes.c_int, ctypes.c_uint32]
        getattr(L, P + "write_kv_cache").argtypes = [_u16p, _u16p, _u16p, _u16p, ctypes.c_uint32]
        getattr(L, P + "attention").argtypes = [_u16p, _u16p, _u16p, _u16p, ctypes.c_uint32, _f32p]
        getattr(L, P + "residual_add").argtypes = [_u16p, _u16p, _u16p, ctypes.c_int]
        getattr(L, P + "swiglu").argtypes = [_u16p, _u16p, ctypes.c_int]

    def gemv_q4_0(self, packed, scales, x, bias=None, threads=768):
        n = scales.size * 32 // (x.size)
        k = x.size
        y = np.zeros(n, np.float16)
        getattr(self.lib, self.prefix + "gemv_q4_0")(
            _p(packed, _u8p), _p(scales.view(np.uint16), _u16p), _p(x.view(np.uint16), _u16p),
            _p(y.view(np.uint16), _u16p),
            _p(None if bias is None else bias.view(np.uint16), _u16p), n, k, threads)
        return y

    def gemv_fp16(self, w, x, threads=768):
        n, k = w.shape
        y = np.zeros(n, np.float16)
        getattr(self.lib, self.prefix + "gemv_fp16")(
            _p(w.view(np.uint16), _u16p), _p(x.view(np.uint16), _u16p),
            _p(y.view(np.uint16), _u16p), n, k, threads)
        return y

    def rms_norm(self, x, gamma, threads=256):
        out = np.zeros(HIDDEN, np.float16)
        getattr(self.lib, self.prefix + "rms_norm")(
            _p(x.view(np.uint16), _u16p), _p(gamma.view(np.uint16), _u16p),
            _p(out.view(np.uint16), _u16p), threads)
        return out

    def rope(self, vec, n_heads, seq_len):
        v = vec.copy()
        getattr(self.lib, self.prefix + "rope")(_p(v.view(np.uint16), _u16p), n_heads, seq_len)
        return v

    def write_kv_cache(self, k, v, k_cache, v_cache, seq_len):
        getattr(self.lib, self.prefix + "write_kv_cache")(
            _p(k.view(np.uint16), _u16p), _p(v.view(np.uint16), _u16p),
            _p(k_cache.view(np.uint16), _u16p), _p(v_cache.view(np.uint16), _u16p), seq_len)

    def attention(self, q, k_cache, v_cache, seq_len):
        out = np.zeros(HIDDEN, np.float16)
        scores = np.zeros(HEADS * seq_len, np.float32)
        getattr(self.lib, self.prefix + "attention")(
            _p(q.view(np.uint16), _u16p), _p(k_cache.view(np.uint16), _u16p),
            _p(v_cache.view(np.uint16), _u16p), _p(out.view(np.uint16), _u16p), seq_len,
            _p(scores, _f32p))
        return out

    def residual_add(self, x, y):
        out = np.zeros_like(x)
        getattr(self.lib, self.prefix + "residual_add")(
            _p(x.view(np.uint16), _u16p), _p(y.view(np.uint16), _u16p),
            _p(out.view(np.uint16), _u16p), x.size)
        return out

    def swiglu(self, gate, up):
        g = gate.copy()
        getattr(self.lib, self.prefix + "swiglu")(_p(g.view(np.uint16), _u16p),
                                                  _p(up.view(np.uint16), _u16p), g.size)
        return g


class MetalRef(_Kernels):
    prefix = "ref_"

    def __init__(self):
        ensure_oracle_built(ref=True)
        super().__init__(REF_SO)


class Oracle(_Kernels):
    prefix = "oracle_"

    def set_threads(self, n: int) -> int:
        """OpenMP threads of the oracle's loops (returns the count in effect)."""
        return self.lib.oracle_set_threads(n)

    def __init__(self):
        ensure_oracle_built()
        super().__init__(ORACLE_SO)
        L = self.lib
        L.oracle_quantize_q4.argtypes = [_f32p, ctypes.c_size_t, _u8p, _u16p]
        L.oracle_dequant_q4.argtypes = [_u8p, _u16p, ctypes.c_size_t, _f32p]
        L.oracle_sample_greedy.argtypes = [_u16p, ctypes.c_int]
        L.oracle_sample_top_p.argtypes = [_u16p, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                          ctypes.c_uint32]
        L.oracle_sample_reference_float.argtypes = [_u16p, ctypes.c_int, ctypes.c_float,
                                                    ctypes.c_float, ctypes.c_float]
        L.oracle_sampler_exp.argtypes = [ctypes.c_float]
        L.oracle_sampler_exp.restype = ctypes.c_float
        L.oracle_uniform24.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64]
        L.oracle_uniform24.restype = ctypes.c_uint32
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_set_threads.restype = ctypes.c_int
        L.oracle_model_load.argtypes = [ctypes.c_char_p, ctypes.c_int]
        L.oracle_model_load.restype = ctypes.c_void_p
        L.oracle_model_free.argtypes = [ctypes.c_void_p]
        L.oracle_model_random.argtypes = [ctypes.c_int, ctypes.c_uint64]
        L.oracle_model_random.restype = ctypes.c_void_p
        L.oracle_state_create.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oracle_state_create.restype = ctypes.c_void_p
        L.oracle_state_free.argtypes = [ctypes.c_void_p]
        L.oracle_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                     _u16p]
        L.oracle_state_k_cache.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oracle_state_k_cache.restype = _u16p
        L.oracle_state_v_cache.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oracle_state_v_cache.restype = _u16p
        L.oracle_state_x.argtypes = [ctypes.c_void_p]
        L.oracle_state_x.restype = _u16p

    # -- quantizer ---------------------------------------------------------
    def quantize_q4(self, w: np.ndarray):
        w = np.ascontiguousarray(w, np.float32).ravel()
        nb = (w.size + 31) // 32
        packed = np.zeros(nb * 16, np.uint8)
        scales = np.zeros(nb, np.float16)
        self.lib.oracle_quantize_q4(_p(w, _f32p), w.size, _p(packed, _u8p),
                                    _p(scales.view(np.uint16), _u16p))
        return packed, scales

    def dequant_q4(self, packed, scales, n):
        out = np.zeros(n, np.float32)
        self.lib.oracle_dequant_q4(_p(packed, _u8p), _p(scales.view(np.uint16), _u16p), n,
                                   _p(out, _f32p))
        return out

    # -- sampler -----------------------------------------------------------
    def sample_greedy(self, logits):
        return self.lib.oracle_sample_greedy(_p(logits.view(np.uint16), _u16p), ACTUAL_VOCAB
                                             if logits.size >= ACTUAL_VOCAB else logits.size)

    def sample_top_p(self, logits, temperature, top_p, u24, vocab=None):
        vocab = vocab or min(logits.size, ACTUAL_VOCAB)
        return self.lib.oracle_sample_top_p(_p(logits.view(np.uint16), _u16p), vocab,
                                            temperature, top_p, u24)

    def sample_reference_float(self, logits, temperature, top_p, u, vocab=None):
        vocab = vocab or min(logits.size, ACTUAL_VOCAB)
        return self.lib.oracle_sample_reference_float(_p(logits.view(np.uint16), _u16p), vocab,
                                                      temperature, top_p, u)

    def sampler_exp(self, x: float) -> float:
        return self.lib.oracle_sampler_exp(x)

    def uniform24(self, seed, seq, step) -> int:
        return self.lib.oracle_uniform24(seed, seq, step)


class OracleModel:
    """Whole-model oracle over a reference-layout weight directory."""

    def __init__(self, oracle: Oracle, weights_dir: str | None, n_layers: int, max_ctx: int,
                 random_seed: int = 0):
        self.o = oracle
        self.n_layers = n_layers
        if weights_dir is None:
            self.m = oracle.lib.oracle_model_random(n_layers, random_seed)
        else:
            self.m = oracle.lib.oracle_model_load(weights_dir.encode(), n_layers)
        if not self.m:
            raise FileNotFoundError(f"oracle could not load {weights_dir}")
        self.s = oracle.lib.oracle_state_create(self.m, max_ctx)
        self.max_ctx = max_ctx

    def forward(self, token: int, position: int, want_logits: bool = True):
        logits = np.zeros(VOCAB, np.float16) if want_logits else None
        self.o.lib.oracle_forward(self.m, self.s, token, position,
                                  _p(None if logits is None else logits.view(np.uint16), _u16p))
        return logits

    def k_cache(self, layer):
        p = self.o.lib.oracle_state_k_cache(self.s, layer)
        return np.ctypeslib.as_array(p, shape=(self.max_ctx, KV_DIM)).view(np.float16)

    def v_cache(self, layer):
        p = self.o.lib.oracle_state_v_cache(self.s, layer)
        return np.ctypeslib.as_array(p, shape=(self.max_ctx, KV_DIM)).view(np.float16)

    def x(self):
        p = self.o.lib.oracle_state_x(self.s)
        return np.ctypeslib.as_array(p, shape=(HIDDEN,)).view(np.float16).copy()

    def close(self):
        if self.s:
            self.o.lib.oracle_state_free(self.s)
            self.s = None
        if self.m:
            self.o.lib.oracle_model_free(self.m)
            self.m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
