"""Decode benchmark: Qwen2.5-1.5B (Q4 block-32), batch 1 at context 512 per B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one decode token of the full 28-layer random-init model (weights on
the device, 1.22 GB per token, larger than L2 so nothing needs flushing),
sampling with the reference's defaults (temperature 0.7, top-p 0.8).  N > 1
runs independent replicas, one per GPU (torchrun, one rank per GPU), with no
collective on the data path; the value is the sum over ranks.

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS, VOCAB = 28, 151936
CTX = 512
LAYER_BYTES = 26_337_280          # Q4 tiles + fp16 scales + norms + biases per layer
LM_BYTES = VOCAB * 1536 * 2       # tied fp16 LM head
KV_BYTES_PER_POS = LAYERS * 256 * 2 * 2
EMBED_ROW = 1536 * 2
METRIC = "decode tokens/s (bs1 ctx512 per B200)"


# DRAM traffic of one launch of the fused step kernel (dram__bytes_read.sum +
# dram__bytes_write.sum from one ncu capture of the 28-layer model at context 6:
# 1.006 x the algorithmic bytes there).  Weights and LM head are read once per
# launch, so the traffic at another context adds the KV bytes of the extra
# positions.
FUSED_TRAFFIC_CTX6 = 1_212_492_544


def fused_traffic(ctx: float) -> float:
    return FUSED_TRAFFIC_CTX6 + KV_BYTES_PER_POS * (ctx - 6)


def bytes_per_token(ctx: float) -> float:
    return LAYERS * LAYER_BYTES + LM_BYTES + KV_BYTES_PER_POS * ctx + EMBED_ROW


def peak_gbs():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # Start timing only once the sampler is live (its first line is in).
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def replica_barrier(world: int) -> None:
    """Device work of this rank finished, then a host barrier over the replicas
    (gloo; replicas exchange no data)."""
    import torch

    if torch.cuda.is_available():
        torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def replica_max(x: float, world: int) -> float:
    """The maximum of x over the replicas (the job's time is the slowest rank's)."""
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def replica_tokens_per_s(world: int, tokens_per_rank: int, ms_max: float) -> float:
    """Whole-job throughput of weak-scaled replicas: every rank decodes
    tokens_per_rank tokens; the job takes the slowest rank's time."""
    return world * tokens_per_rank / (ms_max * 1e-3)


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def cpu_baseline(n_tokens: int = 3, warmup: int = 1):
    """Oracle port (the reference's arithmetic restated in C++, OpenMP over all
    host cores) decoding at ctx 512 on a random-init 28-layer model with a
    random KV cache; returns tokens/s over a bounded sample."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracle_lib import Oracle, OracleModel

    o = Oracle()
    # every host thread (torchrun sets OMP_NUM_THREADS=1 for its workers)
    threads = o.set_threads(len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity")
                            else os.cpu_count())
    m = OracleModel(o, None, LAYERS, CTX + 8, random_seed=7)
    rng = np.random.default_rng(7)
    for layer in range(LAYERS):
        m.k_cache(layer)[: CTX - 1] = rng.standard_normal((CTX - 1, 256)).astype(np.float16)
        m.v_cache(layer)[: CTX - 1] = rng.standard_normal((CTX - 1, 256)).astype(np.float16)
    tok = 100
    for _ in range(warmup):
        m.forward(tok, CTX - 1)
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        lg = m.forward(tok, CTX - 1)
        tok = int(np.argmax(lg[:151666]))
    dt = time.perf_counter() - t0
    m.close()
    return {"value": n_tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n_tokens} decode tokens (after {warmup} warm-up) of the 28-layer model "
                      f"at ctx {CTX}, random-init weights and KV cache, oracle/liboracle.so"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    # one step = one decode token of the CPU port (~0.2-0.4 s on the host cores):
    # the requested warm-up (at most 5) and at most 50 timed steps keep the run
    # well under a minute
    steps = max(1, min(args.steps, 50))
    warm = max(0, min(args.warmup, 5))
    cb = cpu_baseline(n_tokens=steps, warmup=warm)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": steps, "warmup": warm,
            "ms_per_step": 1000.0 / cb["value"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 (fp32 accumulate), int4 weights",
            "data": "synthetic",
            "config": {"workload": "Qwen2.5-1.5B Q4 block-32 decode, batch 1, ctx 512 (28 layers)",
                       "batch": 1, "ctx": CTX, "layers": LAYERS,
                       "note": "the reference runs on Metal only; this arm times the oracle port of "
                               "its arithmetic on the host cores (rank 0)"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


BATCH = 64          # sequences per GPU, batched replicated decode
BATCH_PROMPT = 1024
BATCH_CTX = 2048


def run_batched(args, rank, world, local, barrier, max_over_ranks):
    """Batched replicated decode: 64 independent sequences per GPU on the
    tensor-core step (every projection one tcgen05 GEMM over the batch), each
    with a 1024-token random prompt seeded by its global sequence index, then
    top-p 0.9 / T 0.7 decode steps with per-sequence seeded uniforms.  Timed
    over decode steps only (the prompt is prefilled first); whole-job tokens/s."""
    import torch

    from qweninferenceengine_b200 import QwenConfig, QwenEngine

    cfg = QwenConfig(max_context_window=BATCH_CTX, temperature=0.7, top_p=0.9, seed=rank,
                     batch=BATCH, device=local, kernels="tc", stop_on_eos=False)
    eng = QwenEngine(config=cfg, random_seed=1234 + rank)
    prompts = np.stack([np.random.default_rng(rank * BATCH + i).integers(0, VOCAB, size=BATCH_PROMPT)
                        for i in range(BATCH)]).astype(np.int32)
    eng.prefill(prompts)
    eng.decode(args.warmup, record=False)
    stream = torch.cuda.ExternalStream(eng.stream())
    steps = max(5, min(args.steps, 100))
    pos0 = eng.position(0)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    start.record(stream)
    eng.decode(steps, record=False)
    end.record(stream)
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    ms_step_prof, ms_model = eng.time_steps(5)
    launches = eng.kernels_per_step()
    eng.close()
    ctx_avg = pos0 + (steps + 1) / 2.0
    step_bytes = (LAYERS * LAYER_BYTES + LM_BYTES + BATCH * (KV_BYTES_PER_POS * ctx_avg + EMBED_ROW))
    peak, peak_kind = peak_gbs()
    achieved = step_bytes / (ms_model * 1e-3) / 1e9
    return {
        "metric": "decode tokens/s (bs64 per GPU, replicas)",
        "value": replica_tokens_per_s(world, BATCH * steps, ms),
        "unit": "tokens/s", "n_gpus": world, "steps": steps, "ms_per_step": ms / steps,
        "config": {"workload": "Qwen2.5-1.5B Q4 block-32 decode, 64 sequences per GPU, 1024-token "
                               "prompts, top-p 0.9 T 0.7 (28 layers)",
                   "batch_per_gpu": BATCH, "ctx_start": pos0, "ctx_avg": ctx_avg, "kernels": "tc"},
        "roofline": {"bound": "hbm", "kernel": "model kernels of the batched step",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} hbm_gbs", "algorithmic_bytes": step_bytes,
                     "ms_model": ms_model},
        "gpu_launches_per_step": launches,
    }


def run_ours(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    from qweninferenceengine_b200 import QwenConfig, QwenEngine

    cfg = QwenConfig(max_context_window=1024, temperature=0.7, top_p=0.8, seed=rank,
                     device=local, kernels=args.kernels, stop_on_eos=False)
    eng = QwenEngine(config=cfg, random_seed=1234 + rank)
    rng = np.random.default_rng(rank)
    prompt = rng.integers(0, VOCAB, size=CTX - 1).astype(np.int32)
    eng.prefill(prompt)                   # positions 0..510
    eng.decode(args.warmup, record=False)  # warm-up decode steps
    stream = torch.cuda.ExternalStream(eng.stream())

    def barrier():
        replica_barrier(world)

    def max_over_ranks(x: float) -> float:
        return replica_max(x, world)

    # ---- device-timed decode: K graph replays, inputs resident in HBM.
    pos0 = eng.position()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clk:
        start.record(stream)
        eng.decode(args.steps, record=False)
        end.record(stream)
        barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    ctx_avg = pos0 + (args.steps + 1) / 2.0

    # ---- dominant kernel timing (model kernels only, CUDA events), roofline.
    n_prof = max(3, min(20, args.steps))
    ms_step_prof, ms_model = eng.time_steps(n_prof)
    ctx_prof = eng.position() - n_prof / 2.0
    algo = bytes_per_token(ctx_prof)
    peak, peak_kind = peak_gbs()
    achieved = algo / (ms_model * 1e-3) / 1e9

    # ---- end to end through the public API: forward(token, position) per step,
    # token in from pinned host memory, next token back to the host each step.
    n_e2e = max(3, min(args.steps, 50))
    tok = 17
    pos = eng.position()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for i in range(n_e2e):
        tok = eng.forward(tok, pos + i)
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))

    launches = eng.kernels_per_step() * args.steps
    eng.close()

    batched = None if args.no_batched else run_batched(args, rank, world, local, barrier,
                                                       max_over_ranks)
    if rank == 0:
        tok_s = replica_tokens_per_s(world, args.steps, ms)
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 (fp32 accumulate), int4 weights", "data": "synthetic",
            "config": {"workload": "Qwen2.5-1.5B Q4 block-32 decode, batch 1, ctx 512 (28 layers)",
                       "batch_per_gpu": 1, "ctx_start": pos0, "ctx_avg": ctx_avg, "layers": LAYERS,
                       "kernels": args.kernels, "temperature": 0.7, "top_p": 0.8,
                       "parallelism": f"replicas x{world}",
                       "l2": "weights 1.2 GB per token >> 126 MB L2; no flush"},
            "roofline": {"bound": "hbm", "kernel": "model kernels of the step (all layers + LM head)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": fused_traffic(ctx_prof) if args.kernels == "fused" else None,
                         "traffic_source": "ncu dram bytes of one 28-layer launch at context 6, "
                                           "plus the KV bytes of the extra positions",
                         "algorithmic_bytes": algo,
                         "ms_model": ms_model, "ms_step_unfused_launch": ms_step_prof},
            "e2e": {"value": world * n_e2e / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 + 32, "d2h_bytes_per_step": 4 + 4,
                    "steps": n_e2e, "api": "QwenEngine.forward(token, position)"},
            "clocks": clk.summary(),
            "gpu_launches": launches,
        }
        if batched is not None:
            line["batched"] = batched
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--kernels", choices=["fused", "ops"], default="fused")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true",
                    help="skip the batched (64 sequences per GPU) measurement")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
