"""Profiling helpers for the decode engine.

    python -m qweninferenceengine_b200.profiling case  [--layers 4] [--steps 2]
        A small decode run (random-init model with `--layers` layers, a short
        prompt, a few decode steps): the workload for `ncu --set full --clock-control
        none -k regex:k_decode_fused -s 3 -c 1` captures, small enough to capture in
        seconds while its 1.2 GB+ of weights still exceed the L2.

    python -m qweninferenceengine_b200.profiling gemm [--rows 17920] [--k 1536] [--batch 64]
        One batched Q4 projection on the tensor cores (qwen_gemm_q4_0_batched,
        eager launches: repack, pack, k_tc_gemm, split sum), repeated --reps
        times -- the workload for `ncu --clock-control none -k regex:k_tc_gemm`
        captures.

    python -m qweninferenceengine_b200.profiling attention [--batch 64] [--ctx 2000]
        Batched decode attention over random caches (qwen_attention_decode_batched),
        repeated --reps times -- the workload for `ncu --clock-control none -k
        regex:k_attention_decode`.

    python -m qweninferenceengine_b200.profiling tcstep [--batch 64] [--ctx 1024]
        The batched tensor-core step: prefill, then --reps eagerly launched steps
        with an event after every kernel (qwen_engine_profile_step); prints the
        per-kernel device times and is the workload for ncu launch lists of it.

    python -m qweninferenceengine_b200.profiling trace [--layers 28] [--ctx 512] [--save f.npy]
        Per-phase critical-path summary of one fused decode step from the
        kernel's %globaltimer stamps (qwen_engine_trace): for each traced layer,
        min / median / max over CTAs of every stamp relative to the layer start.
"""
from __future__ import annotations

import argparse

import numpy as np

from .engine import QwenConfig, QwenEngine

STAMPS = ["start", "x_ready", "qkv_done", "attn_done", "o_ready", "o_done", "gu_ready",
          "gu_done", "parts_out", "reduced"]
ATTN_STAMPS = ["unit_start", "qkv_in", "warp0_done", "warps_merged", "partials_out",
               "splits_in", "output_out"]
EXTRA_WORDS = 0


def run_case(layers: int, steps: int) -> None:
    cfg = QwenConfig(num_layers=layers, max_context_window=1024, temperature=0.0,
                     stop_on_eos=False)
    eng = QwenEngine(config=cfg, random_seed=5)
    eng.prefill(np.arange(1, 5, dtype=np.int32))
    eng.decode(steps, record=False)
    eng.close()


def run_gemm(rows: int, k: int, batch: int, reps: int) -> None:
    import torch

    from . import ops

    g = torch.Generator(device="cpu").manual_seed(0)
    packed = torch.randint(0, 256, (rows * k // 2,), dtype=torch.uint8, generator=g).cuda()
    scales = (torch.rand(rows * k // 32, generator=g) * 0.003).half().cuda()
    x = torch.randn(batch, k, generator=g).half().cuda()
    for _ in range(reps):
        ops.gemm_q4_0_batched(packed, scales, x)
    torch.cuda.synchronize()


def run_attention(batch: int, ctx: int, reps: int) -> None:
    import torch

    from . import ops

    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randn(batch, 1536, generator=g).half().cuda()
    kc = torch.randn(batch, ctx, 256, generator=g).half().cuda()
    vc = torch.randn(batch, ctx, 256, generator=g).half().cuda()
    sl = torch.full((batch,), ctx, dtype=torch.int32).cuda()
    for _ in range(reps):
        ops.attention_decode_batched(q, kc, vc, sl, ctx)
    torch.cuda.synchronize()


def run_tcstep(batch: int, ctx: int, reps: int, layers: int = 28) -> list:
    import torch
    cfg = QwenConfig(num_layers=layers, max_context_window=max(2048, ctx + 64), temperature=0.7,
                     top_p=0.9, batch=batch, kernels="tc", stop_on_eos=False)
    eng = QwenEngine(config=cfg, random_seed=7)
    prompts = np.stack([np.random.default_rng(s).integers(0, 151936, size=ctx)
                        for s in range(batch)]).astype(np.int32)
    eng.prefill(prompts)
    prof = []
    torch.cuda.nvtx.range_push("tcstep")  # ncu --clock-control none --nvtx --nvtx-include tcstep/ selects these launches
    for _ in range(reps):
        prof = eng.profile_step()
    torch.cuda.nvtx.range_pop()
    eng.close()
    return prof


def run_trace(layers: int, ctx: int, show_layers, save: str | None = None) -> dict:
    cfg = QwenConfig(num_layers=layers, max_context_window=max(1024, ctx + 64), temperature=0.7,
                     top_p=0.8, stop_on_eos=False)
    eng = QwenEngine(config=cfg, random_seed=5)
    rng = np.random.default_rng(0)
    eng.prefill(rng.integers(0, 151936, size=ctx - 1).astype(np.int32))
    eng.decode(5, record=False)
    ms_step, ms_model = eng.time_steps(10)
    eng.trace(True)
    eng.decode(3, record=False)
    tr = eng.get_trace().astype(np.int64)
    eng.trace(False)
    eng.close()
    if save:
        np.save(save, tr)
    k = len(STAMPS)
    grid = tr.size // (3 + k * layers + 2 + len(ATTN_STAMPS) + EXTRA_WORDS)
    tr = tr.reshape(grid, -1)
    t0 = tr[:, 2].min()
    rel = np.where(tr > 0, (tr - t0) / 1000.0, np.nan)
    ph = rel[:, 3:3 + k * layers].reshape(grid, layers, k)
    out = {"ms_step": ms_step, "ms_model": ms_model, "grid": grid,
           "lm_start_us": float(np.nanmedian(rel[:, 3 + k * layers])),
           "end_us": float(np.nanmax(rel[:, 4 + k * layers])), "layers": {}}
    periods = np.diff(np.nanmedian(ph[:, :, 0], axis=0))
    out["layer_period_us"] = float(np.median(periods)) if periods.size else None
    mid = layers // 2
    att = rel[:, 3 + k * layers + 2:3 + k * layers + 2 + len(ATTN_STAMPS)]
    have = ~np.isnan(att[:, 0])
    if have.any():
        base = np.nanmedian(ph[:, mid, 0])
        out["attention_unit"] = {name: (float(np.nanmin(att[have, j]) - base),
                                        float(np.nanmedian(att[have, j]) - base),
                                        float(np.nanmax(att[have, j]) - base))
                                 for j, name in enumerate(ATTN_STAMPS)}
    for layer in show_layers:
        if layer >= layers:
            continue
        base = np.nanmedian(ph[:, layer, 0])
        rows = {}
        for j, name in enumerate(STAMPS):
            col = ph[:, layer, j]
            col = col[~np.isnan(col)]
            if col.size:
                rows[name] = (int(col.size), float(col.min() - base), float(np.median(col) - base),
                              float(col.max() - base))
        out["layers"][layer] = rows
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("case")
    c.add_argument("--layers", type=int, default=4)
    c.add_argument("--steps", type=int, default=2)
    gm = sub.add_parser("gemm")
    gm.add_argument("--rows", type=int, default=17920)
    gm.add_argument("--k", type=int, default=1536)
    gm.add_argument("--batch", type=int, default=64)
    gm.add_argument("--reps", type=int, default=3)
    at = sub.add_parser("attention")
    at.add_argument("--batch", type=int, default=64)
    at.add_argument("--ctx", type=int, default=2000)
    at.add_argument("--reps", type=int, default=3)
    ts = sub.add_parser("tcstep")
    ts.add_argument("--batch", type=int, default=64)
    ts.add_argument("--ctx", type=int, default=1024)
    ts.add_argument("--reps", type=int, default=2)
    ts.add_argument("--layers", type=int, default=28)
    t = sub.add_parser("trace")
    t.add_argument("--layers", type=int, default=28)
    t.add_argument("--ctx", type=int, default=512)
    t.add_argument("--save", default=None, help="also write the raw stamps (.npy)")
    a = ap.parse_args()
    if a.cmd == "case":
        run_case(a.layers, a.steps)
        print("ok")
        return
    if a.cmd == "gemm":
        run_gemm(a.rows, a.k, a.batch, a.reps)
        print("ok")
        return
    if a.cmd == "tcstep":
        prof = run_tcstep(a.batch, a.ctx, a.reps, a.layers)
        agg = {}
        for name, ms in prof:
            n, t = agg.get(name, (0, 0.0))
            agg[name] = (n + 1, t + ms)
        for name, (n, t) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
            print(f"{name:16s} x{n:3d} {t:8.3f} ms {1000 * t / n:8.1f} us each")
        return
    if a.cmd == "attention":
        run_attention(a.batch, a.ctx, a.reps)
        print("ok")
        return
    r = run_trace(a.layers, a.ctx, [1, a.layers // 2, a.layers - 1], a.save)
    print(f"step {r['ms_step']:.3f} ms, model kernels {r['ms_model']:.3f} ms, grid {r['grid']}, "
          f"median layer period {r['layer_period_us']:.2f} us, LM head from {r['lm_start_us']:.1f} "
          f"to {r['end_us']:.1f} us")
    if "attention_unit" in r:
        print(f"attention units of layer {a.layers // 2} (us from the layer's median start; min / med / max)")
        for name, (lo, med, hi) in r["attention_unit"].items():
            print(f"  {name:14s} {lo:7.2f} {med:7.2f} {hi:7.2f}")
    for layer, rows in r["layers"].items():
        print(f"layer {layer} (us from the layer's median start; n = CTAs with the stamp)")
        for name, (n, lo, med, hi) in rows.items():
            print(f"  {name:10s} n={n:3d}  min {lo:7.2f}  med {med:7.2f}  max {hi:7.2f}")


if __name__ == "__main__":
    main()
