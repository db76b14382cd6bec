"""Batched replicated decode at the workload's size on the tensor-core step: the
28-layer model, 64 independent sequences, each a 1024-token random prompt
(seed = sequence index), top-p 0.9 / T 0.7 with per-sequence uniforms
(InferenceEngine.swift:29-52 and :54-368 per sequence).

For three steps (the last prompt step, position 1023, and the decode steps at
1024 and 1025):
  * every sequence's sampled id must equal the oracle sampler's pick on the
    engine's own logits of that sequence with the same uniform (the sampler runs
    on 4-CTA clusters at this batch);
  * for sequences 0, 31 and 63 the oracle is teacher-forced: given the engine's
    K/V cache of that sequence before the step, it runs the step; logits within
    max-abs 2e-2 and 1e-2 of the range, the new K/V rows within 2e-2.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from qweninferenceengine_b200 import QwenConfig, QwenEngine, ops  # noqa: E402
from model_fixture import make_weight_dir  # noqa: E402
from oracle_lib import OracleModel  # noqa: E402
from test_gpu_engine import check_logits  # noqa: E402

B, N_PROMPT, MAX_CTX = 64, 1024, 2048
SEED, T, TOP_P = 5, 0.7, 0.9
FORCED = (0, 31, 63)


@pytest.fixture(scope="module")
def model_dir(oracle):
    return make_weight_dir(oracle, 28, 3)


def test_batched_64_sequences_full_model(cuda, oracle, model_dir):
    prompts = np.stack([np.random.default_rng(b).integers(0, 151936, size=N_PROMPT)
                        for b in range(B)]).astype(np.int32)
    cfg = QwenConfig(num_layers=28, max_context_window=MAX_CTX, temperature=T, top_p=TOP_P,
                     seed=SEED, batch=B, kernels="tc", stop_on_eos=False)
    eng = QwenEngine(model_dir, cfg)
    om = OracleModel(oracle, model_dir, 28, MAX_CTX)

    def check_step(pos, ids, inputs):
        for b in range(B):
            lg = eng.logits(b)
            want = oracle.sample_top_p(lg, T, TOP_P, ops.uniform24(SEED, b, pos))
            assert ids[b] == want, (pos, b, ids[b], want)
            if b in FORCED:
                for layer in range(28):
                    k, v = eng.kv(b, layer, pos)
                    om.k_cache(layer)[:pos] = k
                    om.v_cache(layer)[:pos] = v
                ref = om.forward(int(inputs[b]), pos)
                check_logits(lg, ref)
                for layer in (0, 27):
                    k, v = eng.kv(b, layer, pos + 1)
                    assert np.abs(k[-1].astype(np.float32) - om.k_cache(layer)[pos].astype(np.float32)).max() < 2e-2
                    assert np.abs(v[-1].astype(np.float32) - om.v_cache(layer)[pos].astype(np.float32)).max() < 2e-2

    out = eng.generate(prompts, max_tokens=1)          # prefill; the last prompt step samples
    first = [o[0] for o in out]
    check_step(N_PROMPT - 1, first, prompts[:, -1])
    inputs = first
    for s in range(2):
        ids = eng.decode(1)[:, 0].tolist()
        check_step(N_PROMPT + s, ids, inputs)
        inputs = ids
    om.close()
    eng.close()
