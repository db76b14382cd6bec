"""Full 28-layer model, batch 1: 128 random prompt ids (seed 1), greedy decode of
256 tokens with a 512-position KV cache, against golden ids produced by the CPU
oracle through the reference's generate loop (InferenceEngine.swift:29-52);
fixture and generator in tests/golden/ (make_config3.py).

The engine computes in a different summation order than the oracle, so a
greedy pick may flip where the oracle's two best logits are closer than the
logit tolerance; the test allows the sequences to part only at such a step.
"""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from qweninferenceengine_b200 import QwenConfig, QwenEngine  # noqa: E402
from model_fixture import make_weight_dir  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
LOGIT_ABS = 2e-2


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(HERE, "golden", "config3_greedy256.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def model_dir(oracle, golden):
    return make_weight_dir(oracle, 28, golden["weight_seed"])


@pytest.mark.parametrize("kernels", ["fused", "ops"])
def test_full_model_greedy_256(cuda, golden, model_dir, kernels):
    prompt = np.random.default_rng(golden["prompt_seed"]).integers(
        0, 151936, size=golden["n_prompt"]).astype(np.int32)
    want = golden["tokens"]
    cfg = QwenConfig(num_layers=28, max_context_window=512, temperature=0.0, kernels=kernels,
                     stop_on_eos=False)
    eng = QwenEngine(model_dir, cfg)
    got = eng.generate(prompt.tolist(), max_tokens=len(want))
    eng.close()
    assert len(got) == len(want)
    diff = [i for i in range(len(want)) if got[i] != want[i]]
    if diff:
        j = diff[0]
        assert golden["top2_margin"][j] < LOGIT_ABS, (
            f"greedy ids part at step {j} ({got[j]} vs {want[j]}) with oracle top-2 margin "
            f"{golden['top2_margin'][j]:.4f}")
