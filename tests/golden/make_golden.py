"""Generates tests/golden/metal_ref_vectors.npz from the reference's own Metal
kernels compiled as C++ (oracle/_ref/libqwen_metal_ref.so, built by
`make -C oracle ref REF_DIR=<reference tree>`).

These fixtures pin the oracle where the reference tree is absent: every entry
holds the inputs and the compiled reference's outputs (fp16 as uint16 bit
patterns).  Run from the repository root:

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from oracle_lib import MetalRef  # noqa: E402


def q4_matrix(rng, n, k):
    """Config-1 style Q4 matrix: q uniform in [-8,7] stored as q+8, one fp16
    scale per 32 weights = |N(0,0.02)|/7."""
    q = rng.integers(0, 16, size=(n, k), dtype=np.uint8)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8).reshape(-1)
    scales = (np.abs(rng.standard_normal(n * k // 32)) * 0.02 / 7).astype(np.float16)
    return packed, scales


def main() -> None:
    ref = MetalRef()
    rng = np.random.default_rng(20240601)
    out = {}

    for tag, n, k in (("a", 64, 1536), ("b", 16, 8960)):
        packed, scales = q4_matrix(rng, n, k)
        x = rng.standard_normal(k).astype(np.float16)
        bias = (rng.standard_normal(n) * 0.01).astype(np.float16)
        y = ref.gemv_q4_0(packed, scales, x, bias)
        out.update({f"gemv_q4_{tag}_packed": packed, f"gemv_q4_{tag}_scales": scales.view(np.uint16),
                    f"gemv_q4_{tag}_x": x.view(np.uint16), f"gemv_q4_{tag}_bias": bias.view(np.uint16),
                    f"gemv_q4_{tag}_y": y.view(np.uint16)})

    w = (rng.standard_normal((32, 1536)) * 0.02).astype(np.float16)
    x = rng.standard_normal(1536).astype(np.float16)
    out.update({"gemv_fp16_w": w.view(np.uint16), "gemv_fp16_x": x.view(np.uint16),
                "gemv_fp16_y": ref.gemv_fp16(w, x).view(np.uint16)})

    x = (rng.standard_normal(1536) * 3).astype(np.float16)
    g = (1 + rng.standard_normal(1536) * 0.02).astype(np.float16)
    out.update({"rms_x": x.view(np.uint16), "rms_g": g.view(np.uint16),
                "rms_y": ref.rms_norm(x, g).view(np.uint16)})

    q = rng.standard_normal(1536).astype(np.float16)
    out["rope_in"] = q.view(np.uint16)
    for sl in (1, 2, 512, 1024, 8704):
        out[f"rope_q_{sl}"] = ref.rope(q, 12, sl).view(np.uint16)
        out[f"rope_k_{sl}"] = ref.rope(q[:256], 2, sl).view(np.uint16)

    L = 37
    kc = rng.standard_normal((L, 256)).astype(np.float16)
    vc = rng.standard_normal((L, 256)).astype(np.float16)
    out.update({"attn_q": q.view(np.uint16), "attn_k": kc.view(np.uint16), "attn_v": vc.view(np.uint16),
                "attn_out": ref.attention(q, kc, vc, L).view(np.uint16)})

    gate = np.concatenate([rng.standard_normal(500) * 8,
                           np.array([15.0, 15.01, -15.0, -15.01, 16, -16, 0.0, -0.0, 30, -30])]
                          ).astype(np.float16)
    up = rng.standard_normal(gate.size).astype(np.float16)
    out.update({"swiglu_gate": gate.view(np.uint16), "swiglu_up": up.view(np.uint16),
                "swiglu_out": ref.swiglu(gate, up).view(np.uint16)})

    a = (rng.standard_normal(1536) * 4).astype(np.float16)
    b = (rng.standard_normal(1536) * 4).astype(np.float16)
    out.update({"resid_a": a.view(np.uint16), "resid_b": b.view(np.uint16),
                "resid_out": ref.residual_add(a, b).view(np.uint16)})

    kc = np.zeros((8, 256), np.float16)
    vc = np.zeros((8, 256), np.float16)
    kk = rng.standard_normal(256).astype(np.float16)
    vv = rng.standard_normal(256).astype(np.float16)
    ref.write_kv_cache(kk, vv, kc, vc, 5)
    out.update({"kv_k": kk.view(np.uint16), "kv_v": vv.view(np.uint16),
                "kv_kc": kc.view(np.uint16), "kv_vc": vc.view(np.uint16)})

    path = os.path.join(HERE, "metal_ref_vectors.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
