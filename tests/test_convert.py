"""safetensors -> weight-directory conversion (QwenPipelines.swift:44-195) on a
tiny synthetic checkpoint.

The CPU tests plug the oracle's quantizer into convert() (the product uses the
device kernel, which test_gpu_ops checks bit-exact against the same oracle
rule) and check the file set, the fp16 conversions, the bias handling and that
every Q4 file holds the tensor it is named for.  The GPU test runs the default
device quantizer and compares its files with the oracle's byte for byte.
"""
import json
import os

import numpy as np
import pytest

from qweninferenceengine_b200 import convert as cv
from qweninferenceengine_b200 import weights as wf

H, KV, INTER, VOCAB, LAYERS = 64, 16, 128, 96, 2


def bf16_bits(x):
    """fp32 -> bf16 bits, rounded to nearest even (how checkpoints are stored)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def write_safetensors(path, tensors):
    header, blobs, off = {"__metadata__": {"format": "pt"}}, [], 0
    for name, (dtype, shape, raw) in tensors.items():
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hj = json.dumps(header).encode()
    hj += b" " * (-len(hj) % 8)
    with open(path, "wb") as f:
        f.write(len(hj).to_bytes(8, "little"))
        f.write(hj)
        for b in blobs:
            f.write(b)


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    rng = np.random.default_rng(11)
    d = tmp_path_factory.mktemp("ckpt")
    t, ref = {}, {}

    def add(name, shape, dtype, scale=0.05):
        x = (rng.standard_normal(shape) * scale).astype(np.float32)
        if dtype == "BF16":
            bits = bf16_bits(x)
            ref[name] = (bits.astype(np.uint32) << 16).view(np.float32).ravel()
            t[name] = ("BF16", shape, bits.tobytes())
        else:
            h = x.astype(np.float16)
            ref[name] = h.astype(np.float32).ravel()
            t[name] = ("F16", shape, h.tobytes())

    add("model.embed_tokens.weight", (VOCAB, H), "BF16")
    add("model.norm.weight", (H,), "F16", 1.0)
    for i in range(LAYERS):
        p = f"model.layers.{i}."
        add(p + "input_layernorm.weight", (H,), "BF16", 1.0)
        add(p + "post_attention_layernorm.weight", (H,), "F16", 1.0)
        for k, rows in (("q", H), ("k", KV), ("v", KV), ("o", H)):
            add(p + f"self_attn.{k}_proj.weight", (rows, H), "BF16")
        for k, rows in (("q", H), ("k", KV), ("v", KV)):
            add(p + f"self_attn.{k}_proj.bias", (rows,), "BF16", 0.5)
        add(p + "mlp.gate_proj.weight", (INTER, H), "BF16")
        add(p + "mlp.up_proj.weight", (INTER, H), "BF16")
        add(p + "mlp.down_proj.weight", (H, INTER), "BF16")
    path = str(d / "model.safetensors")
    write_safetensors(path, t)
    return path, ref


def read(root, rel, dtype):
    return np.fromfile(os.path.join(root, rel), dtype)


def test_conversion_matches_the_pipeline(checkpoint, oracle, tmp_path):
    src, ref = checkpoint
    out = str(tmp_path / "weights")
    written = cv.convert(src, out, LAYERS, quantize=oracle.quantize_q4, hidden=H, kv_dim=KV)
    # the names the loader reads, plus the pipeline's 4-bit embedding copy
    want = set(wf.global_files()) | {"global/embed_tokens_4bit.bin", "global/embed_tokens_scales.bin"}
    for i in range(LAYERS):
        want |= set(wf.layer_files(i))
    assert set(written) == want
    f16 = lambda rel: read(out, rel, np.float16)  # noqa: E731
    assert np.array_equal(f16("global/embed_tokens.bin"), ref["model.embed_tokens.weight"].astype(np.float16))
    assert np.array_equal(f16("global/final_norm.bin"), ref["model.norm.weight"].astype(np.float16))
    for i in range(LAYERS):
        p, d = f"model.layers.{i}.", f"layer{i}/"
        assert np.array_equal(f16(d + f"layer{i}_norm.bin"), ref[p + "input_layernorm.weight"].astype(np.float16))
        assert np.array_equal(f16(d + f"layer{i}_post_attn_norm.bin"),
                              ref[p + "post_attention_layernorm.weight"].astype(np.float16))
        qkv = np.concatenate([ref[p + f"self_attn.{k}_proj.bias"] for k in "qkv"]).astype(np.float16)
        assert np.array_equal(f16(d + "qkv_bias.bin"), qkv)
        assert np.array_equal(f16(d + "o_bias.bin"), np.zeros(H, np.float16))        # absent in Qwen2.5
        assert np.array_equal(f16(d + "mlp_down_bias.bin"), np.zeros(H, np.float16))
        for name, src_name in (("q_proj", "self_attn.q_proj"), ("k_proj", "self_attn.k_proj"),
                               ("v_proj", "self_attn.v_proj"), ("o_proj", "self_attn.o_proj"),
                               ("gate_proj", "mlp.gate_proj"), ("up_proj", "mlp.up_proj"),
                               ("down_proj", "mlp.down_proj")):
            w = ref[p + src_name + ".weight"]
            packed = read(out, d + name + "_4bit.bin", np.uint8)
            scales = read(out, d + name + "_scales.bin", np.float16)
            assert packed.size == w.size // 2 and scales.size == w.size // 32
            back = oracle.dequant_q4(packed, scales, w.size)
            step = np.repeat(scales.astype(np.float32), 32)
            assert np.all(np.abs(back - w) <= 0.5 * step + 1e-3 * np.abs(w) + 1e-7), name


def test_missing_weight_writes_nothing_and_bad_dtype_fails(oracle, tmp_path):
    src = str(tmp_path / "m.safetensors")
    write_safetensors(src, {"model.norm.weight": ("F32", (H,), np.ones(H, np.float32).tobytes())})
    with pytest.raises(ValueError, match="unsupported dtype F32"):
        cv.convert(src, str(tmp_path / "w1"), 1, quantize=oracle.quantize_q4, hidden=H, kv_dim=KV)
    write_safetensors(src, {"model.norm.weight": ("F16", (H,), np.ones(H, np.float16).tobytes())})
    written = cv.convert(src, str(tmp_path / "w2"), 1, quantize=oracle.quantize_q4, hidden=H, kv_dim=KV)
    assert not any(r.endswith("_4bit.bin") for r in written)      # no weights, no Q4 files
    assert np.array_equal(read(str(tmp_path / "w2"), "layer0/qkv_bias.bin", np.float16),
                          np.zeros(H + 2 * KV, np.float16))


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_non_finite_weight_is_an_error_naming_the_tensor(oracle, tmp_path, bad):
    w = np.full((H, H), 0.01, np.float16)
    w[3, 5] = bad
    src = str(tmp_path / "m.safetensors")
    write_safetensors(src, {"model.layers.0.self_attn.q_proj.weight": ("F16", (H, H), w.tobytes())})
    with pytest.raises(ValueError, match=r"model\.layers\.0\.self_attn\.q_proj\.weight holds 1 non-finite"):
        cv.convert(src, str(tmp_path / "w"), 1, quantize=oracle.quantize_q4, hidden=H, kv_dim=KV)


def test_default_quantizer_needs_a_device(checkpoint, tmp_path):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a device is visible")
    with pytest.raises(RuntimeError, match="no CUDA device"):
        cv.convert(checkpoint[0], str(tmp_path / "w"), LAYERS, hidden=H, kv_dim=KV)


@pytest.mark.gpu
def test_device_quantizer_matches_the_rule(checkpoint, oracle, tmp_path):
    a, b = str(tmp_path / "dev"), str(tmp_path / "ref")
    wa = cv.convert(checkpoint[0], a, LAYERS, hidden=H, kv_dim=KV)
    wb = cv.convert(checkpoint[0], b, LAYERS, quantize=oracle.quantize_q4, hidden=H, kv_dim=KV)
    assert wa == wb
    for rel in wa:
        assert open(os.path.join(a, rel), "rb").read() == open(os.path.join(b, rel), "rb").read(), rel
