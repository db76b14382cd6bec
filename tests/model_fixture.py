"""Random-init Qwen2.5-1.5B-shaped weight directories in the reference layout
(test infrastructure).

Linear weights N(0, 0.02) quantised by the oracle's restatement of
packAndSave4Bit (QwenPipelines.swift:97-145); embeddings (tied LM head)
N(0, 0.02) fp16; norms 1 + N(0, 0.02); q/k/v biases N(0, 0.02); o and down
biases zero (QwenPipelines.swift:184,194).  Deterministic for a seed.
"""
from __future__ import annotations

import os
import tempfile

import numpy as np

from qweninferenceengine_b200.weights import HIDDEN, KV_DIM, LINEARS, VOCAB, check_dir, write_file

_CACHE = {}


def make_weight_dir(oracle, n_layers: int, seed: int, root: str | None = None) -> str:
    key = (n_layers, seed)
    if key in _CACHE and not check_dir(_CACHE[key], n_layers):
        return _CACHE[key]
    root = root or tempfile.mkdtemp(prefix=f"qwen_w{n_layers}_s{seed}_")
    rng = np.random.default_rng(seed)
    emb = (rng.standard_normal((VOCAB, HIDDEN), dtype=np.float32) * 0.02).astype(np.float16)
    write_file(root, "global/embed_tokens.bin", emb)
    del emb
    write_file(root, "global/final_norm.bin",
               (1 + rng.standard_normal(HIDDEN, dtype=np.float32) * 0.02).astype(np.float16))
    for i in range(n_layers):
        d = f"layer{i}/"
        write_file(root, d + f"layer{i}_norm.bin",
                   (1 + rng.standard_normal(HIDDEN, dtype=np.float32) * 0.02).astype(np.float16))
        write_file(root, d + f"layer{i}_post_attn_norm.bin",
                   (1 + rng.standard_normal(HIDDEN, dtype=np.float32) * 0.02).astype(np.float16))
        for name, rows, k in LINEARS:
            w = rng.standard_normal((rows, k), dtype=np.float32) * 0.02
            packed, scales = oracle.quantize_q4(w)
            write_file(root, d + f"{name}_4bit.bin", packed)
            write_file(root, d + f"{name}_scales.bin", scales)
        write_file(root, d + "qkv_bias.bin",
                   (rng.standard_normal(HIDDEN + 2 * KV_DIM, dtype=np.float32) * 0.02).astype(np.float16))
        write_file(root, d + "o_bias.bin", np.zeros(HIDDEN, np.float16))
        write_file(root, d + "mlp_down_bias.bin", np.zeros(HIDDEN, np.float16))
    assert not check_dir(root, n_layers)
    _CACHE[key] = root
    return root
