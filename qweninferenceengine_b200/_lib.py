"""ctypes binding of libqwen_b200.so (include/qwen_b200.h).

The library is built in-tree (python -m qweninferenceengine_b200.build).  Loading
fails loudly when it is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libqwen_b200.so")

QWEN_OK = 0
QWEN_ERR_INVALID_ARGUMENT = 1
QWEN_ERR_CUDA = 2
QWEN_ERR_FILE_NOT_FOUND = 3
QWEN_ERR_BAD_WEIGHT_FILE = 4
QWEN_ERR_OUT_OF_MEMORY = 5
QWEN_ERR_DEVICE_TIMEOUT = 6
QWEN_ERR_NO_DEVICE = 7
QWEN_ERR_STATE = 8

QWEN_KERNELS_FUSED = 0
QWEN_KERNELS_OPS = 1
QWEN_KERNELS_TC = 2

QWEN_CTX_CLAMP = 0
QWEN_CTX_ERROR = 1

QWEN_PREFILL_CHUNKED = 0
QWEN_PREFILL_STEPS = 1

c_void_p, c_int, c_uint32, c_int32, c_uint64, c_size_t, c_float = (
    ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_int32, ctypes.c_uint64,
    ctypes.c_size_t, ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u16p = ctypes.POINTER(ctypes.c_uint16)


class EngineConfig(ctypes.Structure):
    """qwen_engine_config."""

    _fields_ = [("device", c_int), ("max_ctx", c_int), ("batch", c_int), ("n_layers", c_int),
                ("kernels", c_int), ("temperature", c_float), ("top_p", c_float),
                ("seed", c_uint64), ("stop_on_eos", c_int), ("ctx_overflow", c_int),
                ("prefill_mode", c_int)]


# name -> (restype, argtypes)
SIGNATURES = {
    "qwen_last_error": (ctypes.c_char_p, []),
    "qwen_abi_version": (c_int, []),
    "qwen_ops_status": (c_int, [c_void_p]),
    "qwen_gemv_q4_0": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_uint32, c_void_p,
                               c_uint32, c_void_p]),
    "qwen_gemv_fp16": (c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_void_p]),
    "qwen_gemm_q4_0_batched": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_uint32, c_void_p,
                                       c_uint32, c_uint32, c_void_p]),
    "qwen_attention_decode_batched": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                              c_uint32, c_uint32, c_void_p]),
    "qwen_gemm_fp16_batched": (c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_uint32,
                                       c_void_p]),
    "qwen_rms_norm_q4": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "qwen_apply_rope_q4": (c_int, [c_void_p, c_uint32, c_void_p, c_void_p]),
    "qwen_write_kv_cache": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_uint32,
                                    c_void_p]),
    "qwen_attention_scores": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_uint32,
                                      c_void_p]),
    "qwen_softmax": (c_int, [c_void_p, c_void_p, c_void_p]),
    "qwen_attn_weighted_sum": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "qwen_residual_add": (c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_void_p]),
    "qwen_swiglu": (c_int, [c_void_p, c_void_p, c_uint32, c_void_p]),
    "qwen_attention_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_uint32,
                                      c_void_p]),
    "qwen_dequant_q4": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "qwen_quantize_q4": (c_int, [c_void_p, c_size_t, c_void_p, c_void_p, c_void_p]),
    "qwen_sample": (c_int, [c_void_p, c_uint32, c_uint32, c_uint32, c_float, c_float, c_void_p,
                            c_void_p, c_void_p]),
    "qwen_sample_scratch_bytes": (c_size_t, [c_uint32]),
    "qwen_sample_scratch": (c_int, [c_void_p, c_uint32, c_uint32, c_uint32, c_float, c_float,
                                    c_void_p, c_void_p, c_void_p, c_void_p]),
    "qwen_uniform24": (c_uint32, [c_uint64, c_uint64, c_uint64]),
    "qwen_engine_config_default": (None, [ctypes.POINTER(EngineConfig)]),
    "qwen_engine_create": (c_int, [ctypes.POINTER(EngineConfig), ctypes.POINTER(c_void_p)]),
    "qwen_engine_destroy": (c_int, [c_void_p]),
    "qwen_engine_load_weights": (c_int, [c_void_p, ctypes.c_char_p]),
    "qwen_engine_init_random": (c_int, [c_void_p, c_uint64]),
    "qwen_engine_reset": (c_int, [c_void_p]),
    "qwen_engine_forward": (c_int, [c_void_p, c_int32, c_int32, _i32p]),
    "qwen_engine_generate": (c_int, [c_void_p, _i32p, c_int32, c_int32, _i32p, _i32p]),
    "qwen_engine_decode": (c_int, [c_void_p, c_int32, _i32p]),
    "qwen_engine_prefill": (c_int, [c_void_p, _i32p, c_int32]),
    "qwen_engine_get_logits": (c_int, [c_void_p, c_int32, _u16p]),
    "qwen_engine_get_kv": (c_int, [c_void_p, c_int32, c_int32, c_int32, _u16p, _u16p]),
    "qwen_engine_set_kv": (c_int, [c_void_p, c_int32, c_int32, c_int32, _u16p, _u16p]),
    "qwen_engine_position": (c_int, [c_void_p, c_int32, _i32p]),
    "qwen_engine_stream": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "qwen_engine_set_wait_timeout": (c_int, [c_void_p, c_uint64]),
    "qwen_engine_test_stall": (c_int, [c_void_p, c_int32]),
    "qwen_engine_kernels_per_step": (c_int, [c_void_p, _i32p]),
    "qwen_engine_trace": (c_int, [c_void_p, c_int32]),
    "qwen_engine_get_trace": (c_int, [c_void_p, ctypes.POINTER(c_uint64), c_size_t,
                                      ctypes.POINTER(c_size_t)]),
    "qwen_engine_time_steps": (c_int, [c_void_p, c_int32, ctypes.POINTER(c_float),
                                       ctypes.POINTER(c_float)]),
    "qwen_engine_profile_step": (c_int, [c_void_p, c_void_p, c_int32, c_void_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Loads libqwen_b200.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m qweninferenceengine_b200.build` "
                "(the engine has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class QwenError(RuntimeError):
    """A QWEN_ERR_* status from the library, with qwen_last_error()'s message."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != QWEN_OK:
        raise QwenError(rc, lib().qwen_last_error().decode(errors="replace"))
