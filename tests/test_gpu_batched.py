"""Batched projections on the tcgen05 tensor cores against the CPU oracle's
gemv_q4_0 / gemv_fp16 (matmul.metal:9-113), one oracle call per activation row.

Two checks per case:
  * against the oracle (the reference's arithmetic: (q-8)*s formed exactly in
    fp32): |d| <= 2 ulp(fp16) + 2e-3 -- the tensor-core path rounds each
    dequantised weight once to fp16 (relative error <= 2^-11);
  * against a float64 evaluation of the same fp16-rounded weights: |d| <=
    2 ulp + 1e-4 -- only the summation order differs, which pins the tile
    layouts, swizzles and descriptors exactly.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from qweninferenceengine_b200 import ops  # noqa: E402
from test_gpu_ops import N, T, q4_config1, ulp16  # noqa: E402


def assert_within(got, ref, abs_tol, ulps=2):
    g = np.asarray(got, np.float16).astype(np.float32)
    r = np.asarray(ref, np.float16).astype(np.float32)
    d = np.abs(g - r)
    lim = ulps * ulp16(r) + abs_tol
    bad = np.argwhere(d > lim)
    assert bad.size == 0, f"{len(bad)} elements off; worst {d.max()} at {np.unravel_index(d.argmax(), d.shape)}"


def dequant_f16_rounded(packed, scales, n, k):
    q = np.empty((n, k), np.float32)
    p = packed.reshape(n, k // 2)
    q[:, 0::2] = (p & 15).astype(np.float32) - 8
    q[:, 1::2] = (p >> 4).astype(np.float32) - 8
    s = scales.astype(np.float32).reshape(n, k // 32).repeat(32, axis=1)
    return (q * s).astype(np.float16)   # one rounding of the exact product


@pytest.mark.parametrize("n,k,nb", [(512, 1536, 1), (512, 1536, 3), (512, 1536, 64),
                                    (256, 1536, 200), (8960, 1536, 64), (1536, 8960, 17)])
def test_gemm_q4_batched(cuda, oracle, n, k, nb):
    packed, scales, _, bias = q4_config1(n + k + nb, n, k)
    rng = np.random.default_rng(nb)
    x = rng.standard_normal((nb, k)).astype(np.float16)
    got = N(ops.gemm_q4_0_batched(T(packed), T(scales), T(x), T(bias)))
    assert got.shape == (nb, n)
    rows = sorted({0, nb // 2, nb - 1})
    ref = np.stack([oracle.gemv_q4_0(packed, scales, x[b], bias) for b in rows])
    assert_within(got[rows], ref, 2e-3)
    w16 = dequant_f16_rounded(packed, scales, n, k).astype(np.float64)
    exact = (x.astype(np.float64) @ w16.T + bias.astype(np.float64)).astype(np.float16)
    assert_within(got, exact, 1e-4)


def test_gemm_q4_batched_config1_all_rows(cuda, oracle):
    # the 8960 x 1536 GEMV of the single-GEMV case (seed 0), 64 activation rows
    packed, scales, x0, bias = q4_config1(0, 8960, 1536)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((64, 1536)).astype(np.float16)
    x[0] = x0
    got = N(ops.gemm_q4_0_batched(T(packed), T(scales), T(x), T(bias)))
    assert_within(got[0], oracle.gemv_q4_0(packed, scales, x0, bias), 2e-3)
    ref = np.stack([oracle.gemv_q4_0(packed, scales, x[b], bias) for b in range(0, 64, 9)])
    assert_within(got[0:64:9], ref, 2e-3)


@pytest.mark.parametrize("n,nb", [(4096, 1), (4096, 64), (151936, 2)])
def test_gemm_fp16_batched(cuda, oracle, n, nb):
    rng = np.random.default_rng(n + nb)
    w = (rng.standard_normal((n, 1536)) * 0.02).astype(np.float16)
    x = rng.standard_normal((nb, 1536)).astype(np.float16)
    got = N(ops.gemm_fp16_batched(T(w), T(x)))
    ref = np.stack([oracle.gemv_fp16(w, x[b]) for b in range(nb)])
    assert_within(got, ref, 1e-4)


def test_gemm_batched_rejects_bad_shapes(cuda):
    x = torch.zeros((2, 100), dtype=torch.float16, device="cuda")
    w = torch.zeros((128, 100), dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        ops.gemm_fp16_batched(w, x)            # k not a multiple of 64
    x = torch.zeros((300, 128), dtype=torch.float16, device="cuda")
    w = torch.zeros((128, 128), dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        ops.gemm_fp16_batched(w, x)            # more than 256 rows


def test_attention_decode_batched(cuda, oracle):
    # ragged lengths, including a single position and a full cache
    lens = [1, 17, 64, 65, 300, 1000]
    max_ctx = 1000
    rng = np.random.default_rng(31)
    n = len(lens)
    q = rng.standard_normal((n, 1536)).astype(np.float16)
    kc = rng.standard_normal((n, max_ctx, 256)).astype(np.float16)
    vc = rng.standard_normal((n, max_ctx, 256)).astype(np.float16)
    sl = T(np.array(lens, np.int32))
    got = N(ops.attention_decode_batched(T(q), T(kc), T(vc), sl, max_ctx))
    for b, L in enumerate(lens):
        ref = oracle.attention(q[b], kc[b], vc[b], L)
        assert_within(got[b], ref, 1e-4)
