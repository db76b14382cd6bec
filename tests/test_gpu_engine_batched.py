"""Batched decode on the tensor cores (kernels="tc"): every sequence of a batch
against the CPU oracle stepping that sequence alone (InferenceEngine.swift:54-271
per sequence; the batch shares nothing but the weights).

Same tolerances as the batch-1 engine tests: logits max-abs <= 2e-2 and <= 1e-2
of the logit range; greedy ids may part from the oracle only where its top-2
margin is below the logit tolerance.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from qweninferenceengine_b200 import QwenConfig, QwenEngine  # noqa: E402
from model_fixture import make_weight_dir  # noqa: E402
from oracle_lib import OracleModel  # noqa: E402
from test_gpu_engine import LOGIT_ABS, check_logits, top2_margin  # noqa: E402


@pytest.fixture(scope="module")
def small_model(oracle):
    return make_weight_dir(oracle, 2, 11)


def test_tc_batch_logits_match_oracle(cuda, oracle, small_model):
    B, n = 3, 20
    checks = (1, 7, 20)
    prompts = np.random.default_rng(21).integers(0, 151936, size=(B, n)).astype(np.int32)
    refs = {}
    for b in range(B):
        om = OracleModel(oracle, small_model, 2, 64)
        for pos in range(n):
            want = (pos + 1) in checks
            lg = om.forward(int(prompts[b, pos]), pos, want_logits=want)
            if want:
                refs[(b, pos + 1)] = lg
        om.close()
    cfg = QwenConfig(num_layers=2, max_context_window=64, temperature=0.0, kernels="tc", batch=B,
                     stop_on_eos=False)
    eng = QwenEngine(small_model, cfg)
    for m in checks:
        eng.prefill(prompts[:, :m])   # positions 0 .. m-1 of every sequence
        for b in range(B):
            check_logits(eng.logits(b), refs[(b, m)])
    k, v = eng.kv(2, 1, n)
    om = OracleModel(oracle, small_model, 2, 64)
    for pos in range(n):
        om.forward(int(prompts[2, pos]), pos, want_logits=False)
    assert np.abs(k.astype(np.float32) - om.k_cache(1)[:n].astype(np.float32)).max() < 2e-2
    assert np.abs(v.astype(np.float32) - om.v_cache(1)[:n].astype(np.float32)).max() < 2e-2
    om.close()
    eng.close()


def test_tc_batch_generate_greedy(cuda, oracle, small_model):
    B, n, gen = 4, 9, 8
    prompts = np.random.default_rng(22).integers(0, 151936, size=(B, n)).astype(np.int32)
    cfg = QwenConfig(num_layers=2, max_context_window=64, temperature=0.0, kernels="tc", batch=B,
                     stop_on_eos=False)
    eng = QwenEngine(small_model, cfg)
    outs = eng.generate(prompts, max_tokens=gen)
    eng.close()
    assert len(outs) == B
    for b in range(B):
        om = OracleModel(oracle, small_model, 2, 64)
        for i in range(n - 1):
            om.forward(int(prompts[b, i]), i, want_logits=False)
        lg = om.forward(int(prompts[b, -1]), n - 1)
        ref, margins = [], []
        for j in range(gen):
            cur = oracle.sample_greedy(lg)
            ref.append(cur)
            margins.append(top2_margin(lg))
            if j + 1 < gen:
                lg = om.forward(cur, n + j)
        om.close()
        assert len(outs[b]) == gen
        diff = [j for j in range(gen) if outs[b][j] != ref[j]]
        if diff:
            assert margins[diff[0]] < LOGIT_ABS, f"seq {b} parts at step {diff[0]}"


@pytest.mark.parametrize("kernels,B", [("tc", 1), ("fused", 1), ("tc", 4)])
def test_chunked_prefill_matches_sequential_oracle(cuda, oracle, small_model, kernels, B):
    """The tensor-core prefill (a batch-1 engine: 128 positions per chunk, 300
    positions = chunks of 128, 128, 44; a batch of 4: 64 positions of every
    sequence per chunk of 256 rows) must match the reference's
    one-token-at-a-time loop (InferenceEngine.swift:29-52) for every sequence:
    logits of the last prompt position, the K/V cache, and the greedy
    continuation decoded by the engine's own step (fused or tensor-core)."""
    n, gen = 300, 6
    prompts = np.stack([np.random.default_rng(23 + b).integers(0, 151936, size=n)
                        for b in range(B)]).astype(np.int32)
    cfg = QwenConfig(num_layers=2, max_context_window=512, temperature=0.0, kernels=kernels,
                     batch=B, stop_on_eos=False)
    eng = QwenEngine(small_model, cfg)
    eng.prefill(prompts)
    got = [eng.logits(b) for b in range(B)]
    kv = [eng.kv(b, 1, n) for b in range(B)]
    assert all(eng.position(b) == n for b in range(B))
    out = eng.decode(gen - 1)
    eng.close()
    for b in range(B):
        om = OracleModel(oracle, small_model, 2, 512)
        for i in range(n - 1):
            om.forward(int(prompts[b, i]), i, want_logits=False)
        ref = om.forward(int(prompts[b, -1]), n - 1)
        check_logits(got[b], ref)
        k, v = kv[b]
        assert np.abs(k.astype(np.float32) - om.k_cache(1)[:n].astype(np.float32)).max() < 2e-2
        assert np.abs(v.astype(np.float32) - om.v_cache(1)[:n].astype(np.float32)).max() < 2e-2
        # greedy continuation from the chunked prefill
        first = oracle.sample_greedy(ref)
        ref_ids, margins, lg, cur = [first], [top2_margin(ref)], ref, first
        for j in range(gen - 1):
            lg = om.forward(cur, n + j)
            cur = oracle.sample_greedy(lg)
            ref_ids.append(cur)
            margins.append(top2_margin(lg))
        om.close()
        seq = out[b].tolist()
        assert len(seq) == gen - 1
        diff = [j for j in range(gen - 1) if seq[j] != ref_ids[j + 1]]
        if diff:
            assert margins[diff[0] + 1] < LOGIT_ABS, f"seq {b} parts at step {diff[0] + 1}"


def test_prefill_modes_agree_on_the_fused_engine(cuda, oracle, small_model):
    """QWEN_PREFILL_STEPS (the reference's loop on the fused step) and the
    default chunked prefill leave logits within the oracle tolerance of each
    other, and the same greedy next token where the margin allows."""
    n = 150
    prompt = np.random.default_rng(31).integers(0, 151936, size=n).astype(np.int32)
    res = {}
    for mode in ("steps", "chunked"):
        eng = QwenEngine(small_model, QwenConfig(num_layers=2, max_context_window=256,
                                                  temperature=0.0, prefill=mode,
                                                  stop_on_eos=False))
        eng.prefill(prompt)
        res[mode] = eng.logits()
        eng.close()
    check_logits(res["chunked"], res["steps"])
