"""Long context, batch 1, full 28-layer model: an 8192-token prefill (random
ids, seed 2) then 512 top-p 0.9 / T 0.7 decode steps with uniforms from seed 3,
positions 8192..8703 of an 8704-position cache (the fused step's split-K
attention at its largest split count).

The oracle cannot replay 8192 full-model steps in test time, so the decode
step at position 8191 is checked teacher-forced: the oracle is given the
engine's K/V cache of positions 0..8190 and runs that one step
(InferenceEngine.swift:54-271); logits must agree within max-abs 2e-2 and 1e-2
of the logit range, the step's new K/V rows within 2e-2.  The 512 sampled
steps are checked for range, final position and run-to-run identity.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from qweninferenceengine_b200 import QwenConfig, QwenEngine  # noqa: E402
from model_fixture import make_weight_dir  # noqa: E402
from oracle_lib import OracleModel  # noqa: E402
from test_gpu_engine import check_logits  # noqa: E402

N_PROMPT = 8192
N_DECODE = 512
MAX_CTX = N_PROMPT + N_DECODE


@pytest.fixture(scope="module")
def model_dir(oracle):
    return make_weight_dir(oracle, 28, 3)


def test_long_context_prefill_step_and_decode(cuda, oracle, model_dir):
    prompt = np.random.default_rng(2).integers(0, 151936, size=N_PROMPT).astype(np.int32)
    cfg = QwenConfig(num_layers=28, max_context_window=MAX_CTX, temperature=0.7, top_p=0.9, seed=3,
                     stop_on_eos=False)
    eng = QwenEngine(model_dir, cfg)
    print("long context: engine ready", flush=True)
    eng.prefill(prompt)
    print("long context: prefill done", flush=True)
    got = eng.logits()

    om = OracleModel(oracle, model_dir, 28, MAX_CTX)
    for layer in range(28):
        k, v = eng.kv(0, layer, N_PROMPT - 1)
        om.k_cache(layer)[: N_PROMPT - 1] = k
        om.v_cache(layer)[: N_PROMPT - 1] = v
    ref = om.forward(int(prompt[-1]), N_PROMPT - 1)
    check_logits(got, ref)
    for layer in (0, 13, 27):
        k, v = eng.kv(0, layer, N_PROMPT)
        assert np.abs(k[-1].astype(np.float32) - om.k_cache(layer)[N_PROMPT - 1].astype(np.float32)).max() < 2e-2
        assert np.abs(v[-1].astype(np.float32) - om.v_cache(layer)[N_PROMPT - 1].astype(np.float32)).max() < 2e-2
    om.close()

    out = eng.decode(N_DECODE)[0]
    assert out.shape == (N_DECODE,)
    assert ((out >= 0) & (out < 151936)).all()
    assert eng.position() == MAX_CTX
    # the same seed gives the same draws
    eng.prefill(prompt)
    again = eng.decode(N_DECODE)[0]
    assert np.array_equal(out, again)
    eng.close()
