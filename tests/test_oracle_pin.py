"""Pins the CPU oracle to the reference.

1. Against tests/golden/metal_ref_vectors.npz: outputs of the reference's own
   kernels/*.metal compiled as C++ (tests/golden/make_golden.py).  Always runs.
2. Live against oracle/_ref/libqwen_metal_ref.so on fresh random inputs, when
   that library is present (it is built from the reference tree).
Both are bit-exact comparisons.
"""
import os

import numpy as np
import pytest

from oracle_lib import REF_SO, MetalRef

GOLD = os.path.join(os.path.dirname(__file__), "golden", "metal_ref_vectors.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def h(a):
    return a.view(np.float16)


def eq(a, b):
    return np.array_equal(np.asarray(a).view(np.uint16), np.asarray(b).view(np.uint16))


@pytest.mark.parametrize("tag", ["a", "b"])
def test_gemv_q4_golden(oracle, gold, tag):
    g = lambda n: gold[f"gemv_q4_{tag}_{n}"]
    y = oracle.gemv_q4_0(g("packed"), h(g("scales")), h(g("x")), h(g("bias")))
    assert eq(y, g("y"))


def test_gemv_fp16_golden(oracle, gold):
    w = h(gold["gemv_fp16_w"]).reshape(32, 1536)
    assert eq(oracle.gemv_fp16(w, h(gold["gemv_fp16_x"])), gold["gemv_fp16_y"])


def test_rms_norm_golden(oracle, gold):
    assert eq(oracle.rms_norm(h(gold["rms_x"]), h(gold["rms_g"])), gold["rms_y"])


@pytest.mark.parametrize("sl", [1, 2, 512, 1024, 8704])
def test_rope_golden(oracle, gold, sl):
    q = h(gold["rope_in"])
    assert eq(oracle.rope(q, 12, sl), gold[f"rope_q_{sl}"])
    assert eq(oracle.rope(q[:256].copy(), 2, sl), gold[f"rope_k_{sl}"])


def test_attention_golden(oracle, gold):
    k = h(gold["attn_k"]).reshape(-1, 256)
    v = h(gold["attn_v"]).reshape(-1, 256)
    assert eq(oracle.attention(h(gold["attn_q"]), k, v, k.shape[0]), gold["attn_out"])


def test_swiglu_golden(oracle, gold):
    assert eq(oracle.swiglu(h(gold["swiglu_gate"]), h(gold["swiglu_up"])), gold["swiglu_out"])


def test_residual_golden(oracle, gold):
    assert eq(oracle.residual_add(h(gold["resid_a"]), h(gold["resid_b"])), gold["resid_out"])


def test_write_kv_golden(oracle, gold):
    kc = np.zeros((8, 256), np.float16)
    vc = np.zeros((8, 256), np.float16)
    oracle.write_kv_cache(h(gold["kv_k"]), h(gold["kv_v"]), kc, vc, 5)
    assert eq(kc.reshape(-1), gold["kv_kc"].reshape(-1)) and eq(vc.reshape(-1), gold["kv_vc"].reshape(-1))


# ---------------------------------------------------------------- live -----
live = pytest.mark.skipif(not os.path.exists(REF_SO),
                          reason="oracle/_ref not built (needs the reference tree)")


@pytest.fixture(scope="module")
def ref():
    return MetalRef()


@live
@pytest.mark.parametrize("n,k,seed", [(40, 1536, 1), (24, 8960, 2), (7, 64, 3)])
def test_gemv_q4_live(oracle, ref, n, k, seed):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((n, k), dtype=np.float32) * 0.02
    packed, scales = oracle.quantize_q4(w)
    x = rng.standard_normal(k).astype(np.float16)
    b = (rng.standard_normal(n) * 0.01).astype(np.float16)
    assert eq(oracle.gemv_q4_0(packed, scales, x, b), ref.gemv_q4_0(packed, scales, x, b))
    assert eq(oracle.gemv_q4_0(packed, scales, x, None), ref.gemv_q4_0(packed, scales, x, None))


@live
def test_norm_rope_attention_live(oracle, ref):
    rng = np.random.default_rng(7)
    for _ in range(3):
        x = (rng.standard_normal(1536) * rng.uniform(0.1, 30)).astype(np.float16)
        g = (1 + rng.standard_normal(1536) * 0.02).astype(np.float16)
        assert eq(oracle.rms_norm(x, g), ref.rms_norm(x, g))
    q = rng.standard_normal(1536).astype(np.float16)
    for sl in (3, 129, 777, 4097):
        assert eq(oracle.rope(q, 12, sl), ref.rope(q, 12, sl))
    for L in (1, 16, 200):
        kc = rng.standard_normal((L, 256)).astype(np.float16)
        vc = rng.standard_normal((L, 256)).astype(np.float16)
        assert eq(oracle.attention(q, kc, vc, L), ref.attention(q, kc, vc, L))
