"""Engine configuration errors that the library reports before touching a
device (runs without a GPU): QWEN_ERR_INVALID_ARGUMENT for out-of-range
sizes and unknown modes, QWEN_ERR_NO_DEVICE for a device index that does not
exist (MetalSetupError.deviceInitializationFailed, MetalManager.swift:12-18)."""
import ctypes

import pytest

from qweninferenceengine_b200 import _lib


def create(**fields):
    L = _lib.lib()
    c = _lib.EngineConfig()
    L.qwen_engine_config_default(ctypes.byref(c))
    for k, v in fields.items():
        setattr(c, k, v)
    h = ctypes.c_void_p()
    rc = L.qwen_engine_create(ctypes.byref(c), ctypes.byref(h))
    if rc == _lib.QWEN_OK:
        L.qwen_engine_destroy(h)
    return rc, L.qwen_last_error().decode()


def test_defaults_match_the_reference():
    c = _lib.EngineConfig()
    _lib.lib().qwen_engine_config_default(ctypes.byref(c))
    assert (c.max_ctx, c.batch, c.n_layers) == (1024, 1, 28)       # QwenConfig.swift:10-22
    assert abs(c.temperature - 0.7) < 1e-6 and abs(c.top_p - 0.8) < 1e-6  # InferenceEngine.swift:273
    assert c.kernels == _lib.QWEN_KERNELS_FUSED and c.ctx_overflow == _lib.QWEN_CTX_CLAMP
    assert _lib.lib().qwen_abi_version() == 2


@pytest.mark.parametrize("field,value,text", [
    ("max_ctx", 0, "max_ctx"), ("max_ctx", (1 << 20) + 1, "max_ctx"),
    ("batch", 0, "batch"), ("batch", 1025, "batch"),
    ("n_layers", 0, "n_layers"), ("n_layers", 29, "n_layers"),
    ("kernels", 7, "kernels"), ("ctx_overflow", 2, "ctx_overflow"),
])
def test_invalid_configuration(field, value, text):
    rc, msg = create(**{field: value})
    assert rc == _lib.QWEN_ERR_INVALID_ARGUMENT and text in msg


def test_ops_path_is_batch_one():
    rc, msg = create(kernels=_lib.QWEN_KERNELS_OPS, batch=2)
    assert rc == _lib.QWEN_ERR_INVALID_ARGUMENT


def test_device_that_does_not_exist():
    rc, msg = create(device=99)
    assert rc == _lib.QWEN_ERR_NO_DEVICE


def test_engine_calls_on_a_null_handle():
    L = _lib.lib()
    assert L.qwen_engine_forward(None, 1, 0, None) == _lib.QWEN_ERR_INVALID_ARGUMENT
    assert L.qwen_engine_set_wait_timeout(None, 1000) == _lib.QWEN_ERR_INVALID_ARGUMENT
    assert L.qwen_engine_test_stall(None, 9) == _lib.QWEN_ERR_INVALID_ARGUMENT
