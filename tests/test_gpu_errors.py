"""Failure paths of the engine, made on the host (no GPU fault is caused):

  * weight directory faults -> WeightLoadingError.fileNotFound /
    bufferCreationFailed (WeightLoader.swift:26-40): a missing file, a
    truncated file, a file of the wrong size;
  * a device index that does not exist (MetalSetupError, MetalManager.swift:12-18);
  * token ids out of range, a prompt longer than the context window;
  * the all-NaN logits rule: the sampler returns 151645 (InferenceEngine.swift:311-315);
  * positions past max_ctx - 1: clamped as the reference does
    (InferenceEngine.swift:55), or an error in QWEN_CTX_ERROR mode;
  * a bounded device wait that runs out: the fused step's test hook makes its
    down-phase waits expect data nothing writes; with a 20 ms limit the step
    returns QWEN_ERR_DEVICE_TIMEOUT, and the engine's next step is correct.
"""
import os
import re
import shutil

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from qweninferenceengine_b200 import QwenConfig, QwenEngine  # noqa: E402
from qweninferenceengine_b200._lib import (QWEN_ERR_BAD_WEIGHT_FILE, QWEN_ERR_DEVICE_TIMEOUT,  # noqa: E402
                                           QWEN_ERR_FILE_NOT_FOUND, QWEN_ERR_INVALID_ARGUMENT,
                                           QWEN_ERR_NO_DEVICE, QwenError)
from model_fixture import make_weight_dir  # noqa: E402
from oracle_lib import OracleModel  # noqa: E402
from test_gpu_engine import check_logits  # noqa: E402


@pytest.fixture(scope="module")
def one_layer(oracle):
    return make_weight_dir(oracle, 1, 21)


def linked_copy(src, dst):
    """A copy of a weight directory whose files are hard links (cheap); files
    the test damages are replaced, never written through the link."""
    shutil.copytree(src, dst, copy_function=os.link)
    return dst


def cfg(**kw):
    base = dict(num_layers=1, max_context_window=32, temperature=0.0, stop_on_eos=False)
    base.update(kw)
    return QwenConfig(**base)


def load_error(path):
    with pytest.raises(QwenError) as ei:
        QwenEngine(path, cfg())
    return ei.value


def test_missing_truncated_and_wrong_size_weight_files(cuda, one_layer, tmp_path):
    d = linked_copy(one_layer, str(tmp_path / "missing"))
    os.remove(os.path.join(d, "layer0", "q_proj_scales.bin"))
    e = load_error(d)
    assert e.code == QWEN_ERR_FILE_NOT_FOUND and "q_proj_scales.bin" in str(e)

    d = linked_copy(one_layer, str(tmp_path / "truncated"))
    f = os.path.join(d, "layer0", "down_proj_4bit.bin")
    data = open(f, "rb").read()
    os.remove(f)
    open(f, "wb").write(data[: len(data) // 2])
    e = load_error(d)
    assert e.code == QWEN_ERR_BAD_WEIGHT_FILE and "down_proj_4bit.bin" in str(e)

    d = linked_copy(one_layer, str(tmp_path / "oversized"))
    f = os.path.join(d, "global", "final_norm.bin")
    data = open(f, "rb").read()
    os.remove(f)
    open(f, "wb").write(data + b"\0\0")
    e = load_error(d)
    assert e.code == QWEN_ERR_BAD_WEIGHT_FILE and "final_norm.bin" in str(e)

    with pytest.raises(QwenError) as ei:
        QwenEngine(str(tmp_path / "no_such_dir"), cfg())
    assert ei.value.code == QWEN_ERR_FILE_NOT_FOUND


def test_bad_device_index(cuda):
    with pytest.raises(QwenError) as ei:
        QwenEngine(config=cfg(device=99), random_seed=1)
    assert ei.value.code == QWEN_ERR_NO_DEVICE


@pytest.mark.parametrize("kernels", ["fused", "ops", "tc"])
def test_token_ids_and_prompt_length(cuda, one_layer, kernels):
    eng = QwenEngine(one_layer, cfg(kernels=kernels))
    for bad in (-1, 151936, 1 << 30):
        with pytest.raises(QwenError) as ei:
            eng.forward(bad, 0)
        assert ei.value.code == QWEN_ERR_INVALID_ARGUMENT
        with pytest.raises(QwenError) as ei:
            eng.generate([5, bad, 7], max_tokens=2)
        assert ei.value.code == QWEN_ERR_INVALID_ARGUMENT
    with pytest.raises(QwenError) as ei:
        eng.prefill(np.arange(33, dtype=np.int32))          # 33 > max_ctx 32
    assert ei.value.code == QWEN_ERR_INVALID_ARGUMENT
    with pytest.raises(QwenError) as ei:
        eng.forward(5, -1)
    assert ei.value.code == QWEN_ERR_INVALID_ARGUMENT
    assert eng.forward(5, 0) >= 0                             # still usable
    eng.close()


@pytest.mark.parametrize("kernels", ["fused", "ops", "tc"])
def test_all_nan_logits_give_im_end(cuda, one_layer, tmp_path, kernels):
    d = linked_copy(one_layer, str(tmp_path / "nan"))
    f = os.path.join(d, "global", "final_norm.bin")
    os.remove(f)
    np.full(1536, np.nan, np.float16).tofile(f)               # final RMSNorm -> NaN everywhere
    for t in (0.0, 0.7):
        eng = QwenEngine(d, cfg(kernels=kernels, temperature=t, top_p=0.9))
        assert eng.forward(11, 0) == 151645
        assert np.isnan(eng.logits()[:151666].astype(np.float32)).all()
        assert eng.generate([11, 12], max_tokens=3) == [151645, 151645, 151645]
        eng.close()


@pytest.mark.parametrize("kernels", ["fused", "ops", "tc"])
def test_positions_past_the_window_are_clamped(cuda, oracle, one_layer, kernels):
    max_ctx = 16
    eng = QwenEngine(one_layer, cfg(kernels=kernels, max_context_window=max_ctx))
    om = OracleModel(oracle, one_layer, 1, max_ctx)
    toks = np.random.default_rng(3).integers(0, 151936, size=max_ctx + 4)
    for pos, tok in enumerate(toks):                          # positions 16..19 reuse slot 15
        nxt = eng.forward(int(tok), pos)
        ref = om.forward(int(tok), pos)
        check_logits(eng.logits(), ref)
        assert eng.position() == pos + 1
        assert nxt == oracle.sample_greedy(eng.logits())
    k, _ = eng.kv(0, 0, max_ctx)
    assert np.abs(k[-1].astype(np.float32) - om.k_cache(0)[max_ctx - 1].astype(np.float32)).max() < 2e-2
    # generate past the window keeps clamping (the reference loop has no stop either)
    out = eng.generate([1, 2, 3], max_tokens=max_ctx + 1)    # positions 0..18
    assert len(out) == max_ctx + 1
    om.close()
    eng.close()


def test_positions_past_the_window_in_error_mode(cuda, one_layer):
    eng = QwenEngine(one_layer, cfg(max_context_window=16, ctx_overflow="error"))
    assert eng.forward(3, 15) >= 0
    with pytest.raises(QwenError) as ei:
        eng.forward(3, 16)
    assert ei.value.code == QWEN_ERR_INVALID_ARGUMENT
    with pytest.raises(QwenError) as ei:
        eng.generate([1, 2, 3], max_tokens=15)                # 3 + 14 positions > 16
    assert ei.value.code == QWEN_ERR_INVALID_ARGUMENT
    assert len(eng.generate([1, 2, 3], max_tokens=14)) == 14  # exactly fills the window
    eng.prefill([1, 2, 3])
    eng.decode(13, record=False)                              # positions 3..15
    with pytest.raises(QwenError) as ei:
        eng.decode(1)
    assert ei.value.code == QWEN_ERR_INVALID_ARGUMENT
    eng.close()


def test_sampler_wait_runs_out_and_the_engine_recovers(cuda, oracle, one_layer):
    """The batch-1 top-p sampler (every SM, digit totals exchanged through
    device memory behind grid barriers) bounds its barrier waits by the
    engine's wait limit: with one CTA held back from the first exchange's
    barrier (test hook site 20) the others give up, forward() returns
    QWEN_ERR_DEVICE_TIMEOUT naming the site and barrier, and once the hook is
    off the next steps draw the oracle sampler's ids on the engine's logits
    (the engine cleared the sampler's scratch)."""
    from qweninferenceengine_b200 import ops
    eng = QwenEngine(one_layer, cfg(kernels="fused", temperature=0.7, top_p=0.8, seed=3))
    nxt = eng.forward(7, 0)
    assert nxt == oracle.sample_top_p(eng.logits(), 0.7, 0.8, ops.uniform24(3, 0, 0))
    eng.set_wait_timeout(20_000_000)                          # 20 ms
    eng.test_stall(20)
    with pytest.raises(QwenError) as ei:
        eng.forward(8, 1)
    assert ei.value.code == QWEN_ERR_DEVICE_TIMEOUT
    assert re.search(r"timed out \(site 20, phase 1,", str(ei.value)), str(ei.value)
    eng.test_stall(0)
    eng.set_wait_timeout(2_000_000_000)
    for pos, tok in ((1, 8), (2, 9), (3, 10)):                # position 1 again, then on
        nxt = eng.forward(tok, pos)
        assert nxt == oracle.sample_top_p(eng.logits(), 0.7, 0.8, ops.uniform24(3, 0, pos)), pos
    eng.close()


def test_device_wait_runs_out_and_the_engine_recovers(cuda, oracle, one_layer):
    eng = QwenEngine(one_layer, cfg(kernels="fused"))
    om = OracleModel(oracle, one_layer, 1, 32)
    eng.forward(7, 0)
    om.forward(7, 0)
    eng.set_wait_timeout(20_000_000)                          # 20 ms
    eng.test_stall(9)                                         # the wait for the down partials
    with pytest.raises(QwenError) as ei:
        eng.forward(8, 1)
    assert ei.value.code == QWEN_ERR_DEVICE_TIMEOUT
    # the first wait to give up is the stalled wait for the down partial sums
    # (site 9) or the final x wait behind it (site 10)
    assert re.search(r"timed out \(site (9|10),", str(ei.value)), str(ei.value)
    eng.test_stall(0)
    eng.set_wait_timeout(2_000_000_000)
    for pos, tok in ((1, 8), (2, 9)):                         # position 1 again, then on
        nxt = eng.forward(tok, pos)
        ref = om.forward(tok, pos)
        check_logits(eng.logits(), ref)
        assert nxt == oracle.sample_greedy(eng.logits())
    om.close()
    eng.close()
