"""Long context, batch 1, full 28-layer model: an 8192-token prefill (random
ids, seed 2) then 512 top-p 0.9 / T 0.7 decode steps with uniforms from seed 3,
positions 8192..8703 of an 8704-position cache (the fused step's split-K
attention at its largest split counts).

The oracle cannot replay 8192 full-model steps in test time, so steps are
checked teacher-forced: the oracle is given the engine's K/V cache of the
positions before the step and runs that one step (InferenceEngine.swift:54-271)
at positions 8191 (the last prompt step), 8447 and 8703 (the last decode step);
logits must agree within max-abs 2e-2 and 1e-2 of the logit range, the step's
new K/V rows within 2e-2.  Every one of the 512 sampled ids must equal the
oracle sampler's pick (the fixed-point top-p rule, bit-exact) on the engine's
own logits of that step with the same uniform (seed 3, sequence 0, position).
The decode() path must reproduce the ids of the step-by-step run.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from qweninferenceengine_b200 import QwenConfig, QwenEngine, ops  # noqa: E402
from model_fixture import make_weight_dir  # noqa: E402
from oracle_lib import OracleModel  # noqa: E402
from test_gpu_engine import check_logits  # noqa: E402

N_PROMPT = 8192
N_DECODE = 512
MAX_CTX = N_PROMPT + N_DECODE
SEED, T, TOP_P = 3, 0.7, 0.9
CHECK_AT = (N_PROMPT + 255, N_PROMPT + N_DECODE - 1)


@pytest.fixture(scope="module")
def model_dir(oracle):
    return make_weight_dir(oracle, 28, 3)


def teacher_forced(oracle, model_dir, eng, token, pos, got_logits):
    om = OracleModel(oracle, model_dir, 28, MAX_CTX)
    for layer in range(28):
        k, v = eng.kv(0, layer, pos)
        om.k_cache(layer)[:pos] = k
        om.v_cache(layer)[:pos] = v
    ref = om.forward(int(token), pos)
    check_logits(got_logits, ref)
    for layer in (0, 13, 27):
        k, v = eng.kv(0, layer, pos + 1)
        assert np.abs(k[-1].astype(np.float32) - om.k_cache(layer)[pos].astype(np.float32)).max() < 2e-2
        assert np.abs(v[-1].astype(np.float32) - om.v_cache(layer)[pos].astype(np.float32)).max() < 2e-2
    om.close()


def test_long_context_prefill_step_and_decode(cuda, oracle, model_dir):
    prompt = np.random.default_rng(2).integers(0, 151936, size=N_PROMPT).astype(np.int32)
    cfg = QwenConfig(num_layers=28, max_context_window=MAX_CTX, temperature=T, top_p=TOP_P,
                     seed=SEED, stop_on_eos=False)
    eng = QwenEngine(model_dir, cfg)
    eng.prefill(prompt)
    lg = eng.logits()
    teacher_forced(oracle, model_dir, eng, prompt[-1], N_PROMPT - 1, lg)
    # the last prompt step's sample, on its own logits
    tok = oracle.sample_top_p(lg, T, TOP_P, ops.uniform24(SEED, 0, N_PROMPT - 1))

    # 512 decode steps one at a time: each sampled id against the oracle sampler
    ids, saved = [], {}
    for pos in range(N_PROMPT, MAX_CTX):
        nxt = eng.forward(tok, pos)
        lg = eng.logits()
        want = oracle.sample_top_p(lg, T, TOP_P, ops.uniform24(SEED, 0, pos))
        assert nxt == want, (pos, nxt, want)
        if pos in CHECK_AT:
            saved[pos] = (tok, lg.copy())
        ids.append(nxt)
        tok = nxt
    for pos in CHECK_AT:
        teacher_forced(oracle, model_dir, eng, saved[pos][0], pos, saved[pos][1])

    # the decode path draws the same ids: after the prefill the sample of the
    # last prompt step is pending, and decode() returns those of 8192..8703
    eng.prefill(prompt)
    out = eng.decode(N_DECODE)[0]
    assert eng.position() == MAX_CTX
    assert out.tolist() == ids
    eng.close()
