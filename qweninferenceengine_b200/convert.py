"""Hugging Face safetensors checkpoint -> the reference's weight directory.

The conversion QwenPipeline.run performs (QwenPipelines.swift:44-195) after its
download step, on a local `model.safetensors` (one file, as Qwen2.5-1.5B
ships):

  * tensors are read as fp32: BF16 by a 16-bit shift (:67-76), F16 by widening
    (:77-80); any other dtype is an error (:81-83);
  * embeddings, norms and biases are written as fp16, rounded to nearest
    (:86-95); a missing bias is written as zeros of its size (:91-92) -- Qwen2.5
    has no o_proj or down_proj bias, so those files are zeros;
  * q/k/v/o/gate/up/down weights (and the embedding once more) are quantized
    with the block-32 symmetric Q4 rule of packAndSave4Bit (:97-145) into
    `<name>_4bit.bin` + `<name>_scales.bin`; a missing weight writes nothing
    (:98);
  * the q, k and v biases are concatenated into `qkv_bias.bin` (:177-181).

The quantizer is the library's device kernel (qwen_quantize_q4, bit-exact
with the rule above), so a conversion needs a CUDA device; `quantize` can be
replaced by any function with the same contract (fp32 array -> packed uint8,
fp16 scales).

    python -m qweninferenceengine_b200.convert downloads/model.safetensors weights/
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from typing import Callable

import numpy as np

from .weights import write_file

HIDDEN, KV_DIM = 1536, 256


class SafeTensors:
    """Read-only view of one .safetensors file: 8-byte little-endian header
    length, a JSON header {name: {dtype, shape, data_offsets}}, then the data."""

    def __init__(self, path: str):
        with open(path, "rb") as f:
            n = int.from_bytes(f.read(8), "little")
            self.header = json.loads(f.read(n))
        self.header.pop("__metadata__", None)
        self.data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n)

    def names(self):
        return list(self.header)

    def f32(self, name: str) -> np.ndarray | None:
        """The tensor as fp32 (flattened), or None when the file lacks it.

        A NaN or infinite value is an error naming the tensor: the pipeline's
        quantizer would trap on Int(round(NaN)) (QwenPipelines.swift:124-131),
        and the device quantizer would otherwise turn it into a plausible nibble."""
        meta = self.header.get(name)
        if meta is None:
            return None
        b, e = meta["data_offsets"]
        raw = self.data[b:e]
        dtype = meta["dtype"]
        if dtype == "BF16":
            out = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        elif dtype == "F16":
            out = raw.view(np.float16).astype(np.float32)
        else:
            raise ValueError(f"unsupported dtype {dtype} for {name}")
        if not np.isfinite(out).all():
            bad = int(np.count_nonzero(~np.isfinite(out)))
            raise ValueError(f"tensor {name} holds {bad} non-finite value(s) (NaN or Inf)")
        return out


def device_quantizer(w: np.ndarray):
    """packAndSave4Bit on the device (qwen_quantize_q4)."""
    import torch

    from . import ops

    if not torch.cuda.is_available():
        raise RuntimeError("the Q4 quantizer runs on the device: no CUDA device is visible")
    packed, scales = ops.quantize_q4(torch.from_numpy(np.ascontiguousarray(w, np.float32)).cuda())
    return packed.cpu().numpy(), scales.cpu().numpy()


def convert(src: str, out_dir: str, n_layers: int = 28,
            quantize: Callable[[np.ndarray], tuple] | None = None,
            hidden: int = HIDDEN, kv_dim: int = KV_DIM, log=None) -> list:
    """Writes the weight directory; returns the relative paths written."""
    st = SafeTensors(src)
    q = quantize or device_quantizer
    written = []

    def f16(rel: str, x: np.ndarray | None, count: int) -> None:
        arr = x.astype(np.float16) if x is not None else np.zeros(count, np.float16)
        write_file(out_dir, rel, arr)
        written.append(rel)

    def q4(rel_prefix: str, x: np.ndarray | None) -> None:
        if x is None:
            return
        packed, scales = q(x)
        write_file(out_dir, rel_prefix + "_4bit.bin", np.asarray(packed, np.uint8))
        write_file(out_dir, rel_prefix + "_scales.bin", np.asarray(scales, np.float16))
        written.extend([rel_prefix + "_4bit.bin", rel_prefix + "_scales.bin"])

    emb = st.f32("model.embed_tokens.weight")
    vocab = emb.size // hidden if emb is not None else 151936
    f16("global/embed_tokens.bin", emb, vocab * hidden)
    q4("global/embed_tokens", emb)
    f16("global/final_norm.bin", st.f32("model.norm.weight"), hidden)
    for i in range(n_layers):
        if log:
            log(f"layer {i}/{n_layers - 1}")
        pre, d = f"model.layers.{i}.", f"layer{i}/"
        f16(d + f"layer{i}_norm.bin", st.f32(pre + "input_layernorm.weight"), hidden)
        f16(d + f"layer{i}_post_attn_norm.bin", st.f32(pre + "post_attention_layernorm.weight"), hidden)
        for key in ("q_proj", "k_proj", "v_proj", "o_proj"):
            q4(d + key, st.f32(pre + f"self_attn.{key}.weight"))
        parts = [(st.f32(pre + f"self_attn.{k}_proj.bias"), n)
                 for k, n in (("q", hidden), ("k", kv_dim), ("v", kv_dim))]
        qkv = np.concatenate([b if b is not None else np.zeros(n, np.float32) for b, n in parts])
        f16(d + "qkv_bias.bin", qkv, hidden + 2 * kv_dim)
        f16(d + "o_bias.bin", st.f32(pre + "self_attn.o_proj.bias"), hidden)
        for key in ("gate_proj", "up_proj", "down_proj"):
            q4(d + key, st.f32(pre + f"mlp.{key}.weight"))
        f16(d + "mlp_down_bias.bin", st.f32(pre + "mlp.down_proj.bias"), hidden)
    return written


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("safetensors")
    ap.add_argument("out_dir")
    ap.add_argument("--layers", type=int, default=28)
    a = ap.parse_args(argv)
    written = convert(a.safetensors, a.out_dir, a.layers, log=lambda m: print(m, file=sys.stderr))
    print(f"wrote {len(written)} files under {os.path.abspath(a.out_dir)}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
