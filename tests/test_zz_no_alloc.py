"""qwen_attention_decode_noalloc against qwen_attention_decode, through the C ABI.

The no-allocation variant exists for callers that may not call cudaMalloc
(code inside another component's stream capture, threads that must stay out of
the CUDA allocator, plugins whose host owns the memory pool).  It must give the
same attention output as the allocating entry point, call after call, even
though every call reuses one fixed scratch array.  This file is collected last
so that a run stopping at the first failure has run everything else first.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from qweninferenceengine_b200._lib import QWEN_ERR_INVALID_ARGUMENT, QWEN_OK, lib  # noqa: E402
from test_gpu_ops import assert_close16  # noqa: E402


def _call(fn, q, kc, vc, out, sl, max_ctx):
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kc.data_ptr()),
            ctypes.c_void_p(vc.data_ptr()), ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(sl.data_ptr()), max_ctx, ctypes.c_void_p(stream))
    assert rc == QWEN_OK, lib().qwen_last_error().decode()


def test_noalloc_matches_allocating_entry_point(cuda):
    L = lib()
    L.qwen_attention_decode_noalloc.restype = ctypes.c_int
    L.qwen_attention_decode_noalloc.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_uint32, ctypes.c_void_p]
    L.qwen_ops_status.restype = ctypes.c_int
    L.qwen_ops_status.argtypes = [ctypes.c_void_p]
    rng = np.random.default_rng(99)
    # calls in a row that each reuse the array the one before left behind, with
    # different lengths and split counts per kv head (128-position tiles): 7 of
    # 8, 1, 32 of 32 (the split count that sizes the array, max_ctx >= 4096),
    # then 8 of 32 and 1 of 1 again
    for L_ctx, max_ctx in ((777, 1024), (40, 1024), (4000, 4096), (1000, 4096), (50, 64)):
        q = torch.from_numpy(rng.standard_normal(1536).astype(np.float16)).cuda()
        kc = torch.from_numpy(rng.standard_normal((max_ctx, 256)).astype(np.float16)).cuda()
        vc = torch.from_numpy(rng.standard_normal((max_ctx, 256)).astype(np.float16)).cuda()
        sl = torch.tensor([L_ctx], dtype=torch.int32, device="cuda")
        want = torch.empty(1536, dtype=torch.float16, device="cuda")
        got = torch.empty(1536, dtype=torch.float16, device="cuda")
        _call(L.qwen_attention_decode, q, kc, vc, want, sl, max_ctx)
        _call(L.qwen_attention_decode_noalloc, q, kc, vc, got, sl, max_ctx)
        torch.cuda.synchronize()
        assert_close16(got.cpu().numpy(), want.cpu().numpy())
    assert L.qwen_ops_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == QWEN_OK


def test_noalloc_reports_a_length_beyond_max_ctx(cuda):
    """A device-side length the kernel rejects (L > max_ctx) is recorded in the
    operator status word -- no allocation needed -- and qwen_ops_status reports
    it once; the output is left untouched and the next call works."""
    L = lib()
    L.qwen_attention_decode_noalloc.restype = ctypes.c_int
    L.qwen_attention_decode_noalloc.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_uint32, ctypes.c_void_p]
    L.qwen_ops_status.restype = ctypes.c_int
    L.qwen_ops_status.argtypes = [ctypes.c_void_p]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    q = torch.zeros(1536, dtype=torch.float16, device="cuda")
    kc = torch.zeros((64, 256), dtype=torch.float16, device="cuda")
    out = torch.full((1536,), 7.0, dtype=torch.float16, device="cuda")
    sl = torch.tensor([65], dtype=torch.int32, device="cuda")
    _call(L.qwen_attention_decode_noalloc, q, kc, kc, out, sl, 64)
    assert L.qwen_ops_status(stream) == QWEN_ERR_INVALID_ARGUMENT
    assert b"out-of-range" in L.qwen_last_error()
    assert bool((out == 7.0).all())
    assert L.qwen_ops_status(stream) == QWEN_OK          # reported once
    sl.fill_(64)
    _call(L.qwen_attention_decode_noalloc, q, kc, kc, out, sl, 64)
    assert L.qwen_ops_status(stream) == QWEN_OK
    assert bool((out == 0.0).all())                       # zero V rows: zero output


def test_noalloc_rejects_oversized_request(cuda):
    L = lib()
    L.qwen_attention_decode_noalloc.restype = ctypes.c_int
    L.qwen_attention_decode_noalloc.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_uint32, ctypes.c_void_p]
    buf = torch.zeros(16, dtype=torch.float16, device="cuda")
    rc = L.qwen_attention_decode_noalloc(*(ctypes.c_void_p(buf.data_ptr()),) * 5, (1 << 20) + 1, None)
    assert rc != QWEN_OK
    assert b"max_ctx" in L.qwen_last_error()
