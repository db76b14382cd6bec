"""One Qwen2.5-1.5B decoder layer, decode step at position 511, as the workload
states it: hidden 1536, 12 Q / 2 KV heads, Q4 block-32 projections with fp16
QKV biases, RMSNorm eps 1e-6 with gamma ~ 1 + N(0, 0.02), RoPE theta 1e6,
SwiGLU, a KV cache prefilled with 511 entries ~ N(0, 1) and an fp16 input
x ~ N(0, 1) (InferenceEngine.swift:54-271 for one layer).

The input enters as the embedding row of the step's token (the row is
overwritten with N(0, 1) values, :57-60), the 511 cache rows through
qwen_engine_set_kv; the layer's output is observed through the final norm and
LM head of a 1-layer model (logits within max-abs 2e-2 and 1e-2 of the range)
and through the K/V row the step writes at position 511 (within 2e-2).
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from qweninferenceengine_b200 import QwenConfig, QwenEngine  # noqa: E402
from model_fixture import make_weight_dir  # noqa: E402
from oracle_lib import OracleModel  # noqa: E402
from test_gpu_engine import check_logits  # noqa: E402

POS = 511
TOKEN = 4242


@pytest.fixture(scope="module")
def layer_case(oracle):
    d = make_weight_dir(oracle, 1, 511)
    rng = np.random.default_rng(511)
    x = rng.standard_normal(1536).astype(np.float16)
    emb = np.memmap(os.path.join(d, "global", "embed_tokens.bin"), dtype=np.float16, mode="r+",
                    shape=(151936, 1536))
    emb[TOKEN] = x
    emb.flush()
    del emb
    k = rng.standard_normal((POS, 256)).astype(np.float16)
    v = rng.standard_normal((POS, 256)).astype(np.float16)
    om = OracleModel(oracle, d, 1, POS + 1)
    om.k_cache(0)[:POS] = k
    om.v_cache(0)[:POS] = v
    ref = om.forward(TOKEN, POS)
    ref_k, ref_v = om.k_cache(0)[POS].copy(), om.v_cache(0)[POS].copy()
    om.close()
    return d, k, v, ref, ref_k, ref_v


@pytest.mark.parametrize("kernels", ["fused", "ops", "tc"])
def test_one_layer_at_position_511(cuda, oracle, layer_case, kernels):
    d, k, v, ref, ref_k, ref_v = layer_case
    eng = QwenEngine(d, QwenConfig(num_layers=1, max_context_window=POS + 1, temperature=0.0,
                                   kernels=kernels, stop_on_eos=False))
    eng.set_kv(0, 0, k, v)
    nxt = eng.forward(TOKEN, POS)
    got = eng.logits()
    gk, gv = eng.kv(0, 0, POS + 1)
    eng.close()
    check_logits(got, ref)
    assert np.array_equal(gk[:POS], k) and np.array_equal(gv[:POS], v)   # the cache is intact
    assert np.abs(gk[POS].astype(np.float32) - ref_k.astype(np.float32)).max() < 2e-2
    assert np.abs(gv[POS].astype(np.float32) - ref_v.astype(np.float32)).max() < 2e-2
    assert nxt == oracle.sample_greedy(got)
