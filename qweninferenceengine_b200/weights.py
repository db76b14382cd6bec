"""Reference weight-directory layout (WeightLoader.swift:49-52, QwenLayer.swift:31-51,
QwenModel.swift:25-27, files written by QwenPipelines.swift:147-195):

    global/embed_tokens.bin           fp16 [151936][1536]  (also the tied LM head)
    global/final_norm.bin             fp16 [1536]
    layer{i}/layer{i}_norm.bin        fp16 [1536]
    layer{i}/layer{i}_post_attn_norm.bin
    layer{i}/{q,k,v,o,gate,up,down}_proj_4bit.bin    uint8 [rows][k/2]
    layer{i}/{q,k,v,o,gate,up,down}_proj_scales.bin  fp16 [rows][k/32]
    layer{i}/qkv_bias.bin             fp16 [2048] (q | k | v)
    layer{i}/o_bias.bin, mlp_down_bias.bin  fp16 [1536]
"""
from __future__ import annotations

import os

import numpy as np

HIDDEN, INTER, KV_DIM, VOCAB = 1536, 8960, 256, 151936

# (name, rows, k)
LINEARS = (("q_proj", HIDDEN, HIDDEN), ("k_proj", KV_DIM, HIDDEN), ("v_proj", KV_DIM, HIDDEN),
           ("o_proj", HIDDEN, HIDDEN), ("gate_proj", INTER, HIDDEN), ("up_proj", INTER, HIDDEN),
           ("down_proj", HIDDEN, INTER))


def layer_files(i: int) -> dict:
    """Relative path -> expected byte size for layer i."""
    d = f"layer{i}/"
    files = {d + f"layer{i}_norm.bin": HIDDEN * 2, d + f"layer{i}_post_attn_norm.bin": HIDDEN * 2,
             d + "qkv_bias.bin": (HIDDEN + 2 * KV_DIM) * 2, d + "o_bias.bin": HIDDEN * 2,
             d + "mlp_down_bias.bin": HIDDEN * 2}
    for name, rows, k in LINEARS:
        files[d + f"{name}_4bit.bin"] = rows * k // 2
        files[d + f"{name}_scales.bin"] = rows * (k // 32) * 2
    return files


def global_files() -> dict:
    return {"global/embed_tokens.bin": VOCAB * HIDDEN * 2, "global/final_norm.bin": HIDDEN * 2}


def write_file(root: str, rel: str, arr: np.ndarray) -> None:
    path = os.path.join(root, rel)
    os.makedirs(os.path.dirname(path), exist_ok=True)
    np.ascontiguousarray(arr).tofile(path)


def check_dir(root: str, n_layers: int) -> list:
    """Lists missing or mis-sized files (empty when the directory is complete)."""
    bad = []
    want = dict(global_files())
    for i in range(n_layers):
        want.update(layer_files(i))
    for rel, size in want.items():
        p = os.path.join(root, rel)
        if not os.path.exists(p):
            bad.append(f"missing {rel}")
        elif os.path.getsize(p) != size:
            bad.append(f"{rel}: {os.path.getsize(p)} bytes, expected {size}")
    return bad
