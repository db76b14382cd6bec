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


def headline_config(world: int) -> dict:
    """The workload of the headline line, shared by both arms."""
    return {"workload": "Qwen2.5-1.5B Q4 block-32 decode, batch 1, ctx 512 (28 layers)",
            "batch_per_gpu": 1, "ctx": CTX, "layers": LAYERS, "temperature": 0.7, "top_p": 0.8,
            "parallelism": f"replicas x{world}",
            "l2": "weights 1.2 GB per token >> 126 MB L2; no flush"}


# DRAM traffic of one launch of the fused step kernel (dram__bytes_read.sum +
# dram__bytes_write.sum from one ncu capture of the 28-layer model at context 8:
# 1.004 x the algorithmic bytes there).  Weights and LM head are read once per
# launch, so the traffic at another context adds the KV bytes of the extra
# positions.
FUSED_TRAFFIC_CTX8 = 1_209_005_312


def fused_traffic(ctx: float) -> float:
    return FUSED_TRAFFIC_CTX8 + KV_BYTES_PER_POS * (ctx - 8)


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
    return cpu_decode(CTX, n_tokens, warmup)


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
            "config": headline_config(args.gpus),
            "note": "the reference runs on Metal only; this arm times the oracle port of its "
                    "arithmetic on the host cores (rank 0)",
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


BATCH = 64          # sequences per GPU, batched replicated decode
BATCH_PROMPT = 1024
BATCH_CTX = 2048


def run_batched(args, rank, world, local, barrier, max_over_ranks):
    """Batched replicated decode, the whole stated workload: 64 independent
    sequences per GPU on the tensor-core step (every projection one tcgen05 GEMM
    over the batch), each a 1024-token random prompt seeded by its global
    sequence index, prefilled on the tensor cores, then 1024 sampled tokens
    (top-p 0.9 / T 0.7, per-sequence seeded uniforms) at context 1025..2048.
    A warm-up prefill + W decode steps come first; then the prefill and the
    1024 decode steps are timed separately; whole-job tokens/s over the decode."""
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
    steps = BATCH_CTX - BATCH_PROMPT
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    barrier()
    ev[0].record(stream)
    eng.prefill(prompts)                  # positions 0..1023 again, timed
    ev[1].record(stream)
    eng.decode(steps, record=False)       # positions 1024..2047
    ev[2].record(stream)
    barrier()
    ms_prefill = max_over_ranks(ev[0].elapsed_time(ev[1]))
    ms = max_over_ranks(ev[1].elapsed_time(ev[2]))
    assert eng.position(0) == BATCH_CTX
    launches = eng.kernels_per_step()
    eng.close()
    ctx_avg = BATCH_PROMPT + (steps + 1) / 2.0
    step_bytes = (LAYERS * LAYER_BYTES + LM_BYTES + BATCH * (KV_BYTES_PER_POS * ctx_avg + EMBED_ROW))
    peak, peak_kind = peak_gbs()
    achieved = step_bytes / (ms / steps * 1e-3) / 1e9
    return {
        "metric": "decode tokens/s (bs64 per GPU, replicas)",
        "value": replica_tokens_per_s(world, BATCH * steps, ms),
        "unit": "tokens/s", "n_gpus": world, "steps": steps, "ms_per_step": ms / steps,
        "prefill_s": ms_prefill * 1e-3,
        "prefill_tokens_per_s": world * BATCH * BATCH_PROMPT / (ms_prefill * 1e-3),
        "config": {"workload": "Qwen2.5-1.5B Q4 block-32 decode, 64 sequences per GPU, 1024-token "
                               "prompts + 1024 sampled tokens, top-p 0.9 T 0.7 (28 layers)",
                   "batch_per_gpu": BATCH, "ctx_range": [BATCH_PROMPT + 1, BATCH_CTX],
                   "kernels": "tc", "prefill": "chunked tensor-core"},
        "roofline": {"bound": "hbm", "kernel": "whole batched step (model kernels + sampler)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} hbm_gbs", "algorithmic_bytes": step_bytes},
        "gpu_launches_per_step": launches,
    }


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracle_lib import Oracle, OracleModel

    o = Oracle()
    threads = o.set_threads(len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity")
                            else os.cpu_count())
    return o, OracleModel, threads


def cpu_decode(ctx: int, n_tokens: int, warmup: int = 1):
    """Oracle port decoding at context `ctx` (random-init 28-layer model, random
    KV cache of ctx - 1 positions): tokens/s over a bounded sample."""
    o, OracleModel, threads = _oracle()
    m = OracleModel(o, None, LAYERS, ctx + 8, random_seed=7)
    rng = np.random.default_rng(7)
    for layer in range(LAYERS):
        m.k_cache(layer)[: ctx - 1] = rng.standard_normal((ctx - 1, 256)).astype(np.float16)
        m.v_cache(layer)[: ctx - 1] = rng.standard_normal((ctx - 1, 256)).astype(np.float16)
    tok = 100
    for _ in range(warmup):
        m.forward(tok, ctx - 1)
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        lg = m.forward(tok, ctx - 1)
        tok = int(np.argmax(lg[:151666]))
    dt = time.perf_counter() - t0
    m.close()
    return {"value": n_tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n_tokens} decode tokens (after {warmup} warm-up) of the 28-layer model at "
                      f"ctx {ctx}, random-init weights and KV cache, oracle/liboracle.so"}


def gemv_inputs(seed: int):
    """The single-GEMV workload: W [8960 x 1536] int4, q uniform in [-8, 7]
    stored as q + 8 (low nibble first), fp16 scales |N(0, 0.02)| / 7 per
    32-block, x ~ N(0, 1) fp16, bias ~ N(0, 0.01) fp16."""
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, GEMV_N * GEMV_K // 2, dtype=np.uint8)
    scales = (np.abs(rng.standard_normal(GEMV_N * GEMV_K // 32)) * 0.02 / 7).astype(np.float16)
    x = rng.standard_normal(GEMV_K).astype(np.float16)
    bias = (rng.standard_normal(GEMV_N) * 0.01).astype(np.float16)
    return packed, scales, x, bias


GEMV_N, GEMV_K = 8960, 1536
GEMV_BYTES = GEMV_N * GEMV_K // 2 + GEMV_N * GEMV_K // 32 * 2 + GEMV_N * 2 + GEMV_K * 2 + GEMV_N * 2


def config_gemv(peak, peak_kind):
    """Config 1: qwen_gemv_q4_0 (the drop-in gemv_q4_0, matmul.metal:9-73) on
    8960 x 1536.  Enough distinct weight copies to cover 4x the L2 are called
    in rotation, so every call reads its weights from HBM.  Timed over back-to-
    back calls as a caller makes them (eager) and as a CUDA graph of one
    rotation (no host launch gaps)."""
    import torch

    from qweninferenceengine_b200 import ops

    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    copies = max(8, -(-4 * l2 // GEMV_BYTES))
    packed = torch.empty((copies, GEMV_N * GEMV_K // 2), dtype=torch.uint8, device="cuda")
    scales = torch.empty((copies, GEMV_N * GEMV_K // 32), dtype=torch.float16, device="cuda")
    bias = torch.empty((copies, GEMV_N), dtype=torch.float16, device="cuda")
    for c in range(copies):
        p_, s_, x_, b_ = gemv_inputs(c)       # copy 0 is the seed-0 case
        packed[c] = torch.from_numpy(p_)
        scales[c] = torch.from_numpy(s_)
        bias[c] = torch.from_numpy(b_)
        if c == 0:
            x = torch.from_numpy(x_).cuda()
    ys = torch.empty((copies, GEMV_N), dtype=torch.float16, device="cuda")

    def rotation():
        for c in range(copies):
            ops.gemv_q4_0(packed[c], scales[c], x, bias[c], out=ys[c])

    for _ in range(3):
        rotation()
    torch.cuda.synchronize()
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        rotation()
    e1.record()
    torch.cuda.synchronize()
    eager_us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        rotation()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    del packed, scales, bias, ys
    achieved = GEMV_BYTES / (us * 1e-6) / 1e9
    return {"metric": "Q4 GEMV 8960x1536 (qwen_gemv_q4_0)", "value": us, "unit": "us/call",
            "higher_is_better": False, "eager_us_per_call": eager_us,
            "config": {"workload": "y = W_deq x + b, W 8960x1536 Q4 block-32, seed 0",
                       "weight_copies": copies, "l2": f"{copies} copies = "
                       f"{copies * GEMV_BYTES / 1e6:.0f} MB rotated (>= 4x L2)"},
            "roofline": {"bound": "hbm", "kernel": "k_gemv_q4_rowmajor", "achieved": achieved,
                         "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} hbm_gbs", "algorithmic_bytes": GEMV_BYTES}}


def cpu_gemv():
    o, _, threads = _oracle()
    packed, scales, x, bias = gemv_inputs(0)
    o.gemv_q4_0(packed, scales, x, bias)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 1.0:
        o.gemv_q4_0(packed, scales, x, bias)
        n += 1
    us = (time.perf_counter() - t0) / n * 1e6
    return {"value": us, "unit": "us/call", "cores": threads, "kind": "port",
            "gbs": GEMV_BYTES / (us * 1e-6) / 1e9,
            "sample": f"{n} calls of the oracle's gemv_q4_0 on the seed-0 8960x1536 case"}


def layer_weights(rng):
    """One layer's Q4 weights and fp16 vectors with the workload's
    distributions (random nibbles and |N(0,0.02)|/7 scales stand in for
    quantised N(0,0.02) weights: same bytes, same arithmetic)."""
    def q4(rows, k):
        return (rng.integers(0, 256, rows * k // 2, dtype=np.uint8),
                (np.abs(rng.standard_normal(rows * k // 32)) * 0.02 / 7).astype(np.float16))
    w = {"q": q4(1536, 1536), "k": q4(256, 1536), "v": q4(256, 1536), "o": q4(1536, 1536),
         "gate": q4(8960, 1536), "up": q4(8960, 1536), "down": q4(1536, 8960)}
    w["in_norm"] = (1 + rng.standard_normal(1536) * 0.02).astype(np.float16)
    w["post_norm"] = (1 + rng.standard_normal(1536) * 0.02).astype(np.float16)
    w["qkv_bias"] = (rng.standard_normal(2048) * 0.02).astype(np.float16)
    return w


def config_layer(peak, peak_kind, local, seed_base):
    """Config 2: one decoder layer's decode step at position 511 (511 cached
    positions).  Two numbers: (a) the fused engine's time per layer in its step,
    (T28 - T1) / 27 from the model-kernel times of a 28-layer and a 1-layer
    engine decoding at positions 511..518; (b) the layer as the chain of
    drop-in operator launches in the reference's dispatch order
    (InferenceEngine.swift:103-253), over 8 distinct layer copies (> L2) in one
    CUDA graph."""
    import torch

    from qweninferenceengine_b200 import QwenConfig, QwenEngine, ops

    model_ms = {}
    for nl in (28, 1):
        eng = QwenEngine(config=QwenConfig(num_layers=nl, max_context_window=1024, temperature=0.7,
                                           top_p=0.8, device=local, stop_on_eos=False),
                         random_seed=seed_base + nl)
        eng.prefill(np.random.default_rng(nl).integers(0, VOCAB, size=CTX - 1).astype(np.int32))
        eng.time_steps(3)
        eng.reset()
        eng.prefill(np.random.default_rng(nl).integers(0, VOCAB, size=CTX - 1).astype(np.int32))
        model_ms[nl] = eng.time_steps(8)[1]
        eng.close()
    fused_us = (model_ms[28] - model_ms[1]) / 27 * 1e3

    copies = 8
    rng = np.random.default_rng(511)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    layers = []
    for _ in range(copies):
        w = layer_weights(rng)
        layers.append({k: (tuple(dev(a) for a in v) if isinstance(v, tuple) else dev(v))
                       for k, v in w.items()})
    kc = [dev(rng.standard_normal((CTX, 256)).astype(np.float16)) for _ in range(copies)]
    vc = [dev(rng.standard_normal((CTX, 256)).astype(np.float16)) for _ in range(copies)]
    x = dev(rng.standard_normal(1536).astype(np.float16))
    sl = torch.tensor([CTX], dtype=torch.int32, device="cuda")
    zero = torch.zeros(8960, dtype=torch.float16, device="cuda")
    scores = torch.empty(12 * CTX, dtype=torch.float32, device="cuda")
    h = torch.empty(1536, dtype=torch.float16, device="cuda")
    q = torch.empty(1536, dtype=torch.float16, device="cuda")
    k = torch.empty(256, dtype=torch.float16, device="cuda")
    v = torch.empty(256, dtype=torch.float16, device="cuda")
    att = torch.empty(1536, dtype=torch.float16, device="cuda")
    o = torch.empty(1536, dtype=torch.float16, device="cuda")
    g = torch.empty(8960, dtype=torch.float16, device="cuda")
    u = torch.empty(8960, dtype=torch.float16, device="cuda")
    dn = torch.empty(1536, dtype=torch.float16, device="cuda")

    def chain():
        for i, L in enumerate(layers):
            xn = ops.rms_norm_q4(x, L["in_norm"])
            ops.gemv_q4_0(*L["q"], xn, L["qkv_bias"][:1536], out=q)
            ops.gemv_q4_0(*L["k"], xn, L["qkv_bias"][1536:1792], out=k)
            ops.gemv_q4_0(*L["v"], xn, L["qkv_bias"][1792:], out=v)
            ops.apply_rope_q4(q, 12, sl)
            ops.apply_rope_q4(k, 2, sl)
            ops.write_kv_cache(k, v, kc[i], vc[i], sl, CTX)
            ops.attention_scores(q, kc[i], scores, sl, CTX)
            ops.softmax(scores, sl)
            ops.attn_weighted_sum(scores, vc[i], att, sl)
            ops.gemv_q4_0(*L["o"], att, None, out=o)
            ops.residual_add(x, o, out=h)
            xn2 = ops.rms_norm_q4(h, L["post_norm"])
            ops.gemv_q4_0(*L["gate"], xn2, zero, out=g)
            ops.gemv_q4_0(*L["up"], xn2, zero, out=u)
            ops.swiglu(g, u)
            ops.gemv_q4_0(*L["down"], g, None, out=dn)
            ops.residual_add(h, dn, out=h)

    chain()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ops_us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    unit = LAYER_BYTES + CTX * 1024 + 1024
    achieved = unit / (fused_us * 1e-6) / 1e9
    return {"metric": "one decoder layer at position 511", "value": fused_us, "unit": "us/layer",
            "higher_is_better": False, "ops_chain_us_per_layer": ops_us,
            "ops_chain_gbs": unit / (ops_us * 1e-6) / 1e9,
            "config": {"workload": "Qwen2.5-1.5B decoder layer, decode step at position 511 "
                                   "(511 cached positions)",
                       "fused": "(T28 - T1) / 27 of the fused step's model-kernel time, positions "
                                "511..518",
                       "ops_chain": "18 drop-in operator launches per layer, 8 layer copies "
                                    "(210 MB > L2) in one CUDA graph"},
            "roofline": {"bound": "hbm", "kernel": "k_decode_fused (per layer)", "achieved": achieved,
                         "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} hbm_gbs", "algorithmic_bytes": unit}}


def cpu_layer():
    """The oracle's chain of the reference kernels for one layer at position 511."""
    o, _, threads = _oracle()
    rng = np.random.default_rng(511)
    w = layer_weights(rng)
    kc = np.zeros((CTX, 256), np.float16)
    vc = np.zeros((CTX, 256), np.float16)
    kc[: CTX - 1] = rng.standard_normal((CTX - 1, 256)).astype(np.float16)
    vc[: CTX - 1] = rng.standard_normal((CTX - 1, 256)).astype(np.float16)
    x = rng.standard_normal(1536).astype(np.float16)

    def layer():
        xn = o.rms_norm(x, w["in_norm"])
        q = o.gemv_q4_0(*w["q"], xn, w["qkv_bias"][:1536])
        k = o.gemv_q4_0(*w["k"], xn, w["qkv_bias"][1536:1792])
        v = o.gemv_q4_0(*w["v"], xn, w["qkv_bias"][1792:])
        q = o.rope(q, 12, CTX)
        k = o.rope(k, 2, CTX)
        o.write_kv_cache(k, v, kc, vc, CTX)
        att = o.attention(q, kc, vc, CTX)
        h = o.residual_add(x, o.gemv_q4_0(*w["o"], att, None))
        xn2 = o.rms_norm(h, w["post_norm"])
        g = o.gemv_q4_0(*w["gate"], xn2, None)
        u = o.gemv_q4_0(*w["up"], xn2, None)
        g = o.swiglu(g, u)
        return o.residual_add(h, o.gemv_q4_0(*w["down"], g, None))

    layer()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 1.0:
        layer()
        n += 1
    us = (time.perf_counter() - t0) / n * 1e6
    return {"value": us, "unit": "us/layer", "cores": threads, "kind": "port",
            "sample": f"{n} layers through the oracle's restated reference kernels at position 511"}


def config_decode(name, peak, peak_kind, local, seed_base, n_prompt, n_decode, max_ctx, temperature,
                  top_p, prompt_seed, seed):
    """A batch-1 prefill + decode run of the 28-layer model on the fused step:
    the prefill (chunked on the tensor cores) and the decode steps are timed
    separately with CUDA events on the engine's stream."""
    import torch

    from qweninferenceengine_b200 import QwenConfig, QwenEngine

    eng = QwenEngine(config=QwenConfig(max_context_window=max_ctx, temperature=temperature,
                                       top_p=top_p, seed=seed, device=local, stop_on_eos=False),
                     random_seed=seed_base)
    prompt = np.random.default_rng(prompt_seed).integers(0, VOCAB, size=n_prompt).astype(np.int32)
    eng.prefill(prompt)                    # warm-up: graphs, module loads
    eng.decode(3, record=False)
    stream = torch.cuda.ExternalStream(eng.stream())
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record(stream)
    eng.prefill(prompt)
    ev[1].record(stream)
    out = eng.decode(n_decode)
    ev[2].record(stream)
    torch.cuda.synchronize()
    ms_prefill = ev[0].elapsed_time(ev[1])
    ms = ev[1].elapsed_time(ev[2])
    eng.close()
    assert out.shape == (1, n_decode)
    ctx_avg = n_prompt + (n_decode + 1) / 2.0
    achieved = bytes_per_token(ctx_avg) / (ms / n_decode * 1e-3) / 1e9
    return {"metric": f"{name} decode tokens/s", "value": n_decode / (ms * 1e-3), "unit": "tokens/s",
            "ms_per_step": ms / n_decode, "prefill_s": ms_prefill * 1e-3,
            "prefill_tokens_per_s": n_prompt / (ms_prefill * 1e-3),
            "config": {"workload": f"28 layers, batch 1, {n_prompt}-token prompt (seed {prompt_seed}) "
                                   f"then {n_decode} decode steps, "
                                   + ("greedy" if temperature <= 0 else
                                      f"top-p {top_p} T {temperature}"),
                       "ctx_range": [n_prompt + 1, n_prompt + n_decode], "max_ctx": max_ctx,
                       "kernels": "fused", "prefill": "chunked tensor-core"},
            "roofline": {"bound": "hbm", "kernel": "whole decode step", "achieved": achieved,
                         "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes": bytes_per_token(ctx_avg)}}


def run_configs(args, local, seed_base):
    """The other workloads, one object each with its own CPU baseline (rank 0,
    one GPU)."""
    peak, peak_kind = peak_gbs()
    out = {}
    c1 = config_gemv(peak, peak_kind)
    if not args.no_cpu_baseline:
        c1["cpu_baseline"] = cpu_gemv()
    out["gemv_q4_8960x1536"] = c1
    c2 = config_layer(peak, peak_kind, local, seed_base)
    if not args.no_cpu_baseline:
        c2["cpu_baseline"] = cpu_layer()
    out["layer_pos511"] = c2
    c3 = config_decode("greedy 256", peak, peak_kind, local, seed_base, 128, 256, 512, 0.0, 1.0, 1, 0)
    if not args.no_cpu_baseline:
        c3["cpu_baseline"] = cpu_decode(256, 3)
    out["greedy_256"] = c3
    c4 = config_decode("long context", peak, peak_kind, local, seed_base, 8192, 512, 8704, 0.7, 0.9,
                       2, 3)
    if not args.no_cpu_baseline:
        c4["cpu_baseline"] = cpu_decode(8448, 2)
    out["long_context_8192"] = c4
    return out


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
    configs = None
    if world == 1 and not args.no_configs:
        configs = run_configs(args, local, 1234 + rank)
    if rank == 0:
        tok_s = replica_tokens_per_s(world, args.steps, ms)
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 (fp32 accumulate), int4 weights", "data": "synthetic",
            "config": headline_config(world),
            "run": {"ctx_start": pos0, "ctx_avg": ctx_avg, "kernels": args.kernels},
            "roofline": {"bound": "hbm", "kernel": "model kernels of the step (all layers + LM head)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": fused_traffic(ctx_prof) if args.kernels == "fused" else None,
                         "traffic_source": "ncu dram bytes of one 28-layer launch at context 8, "
                                           "plus the KV bytes of the extra positions",
                         "algorithmic_bytes": algo,
                         "ms_model": ms_model, "ms_step_unfused_launch": ms_step_prof},
            "e2e": {"value": world * n_e2e / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 32, "d2h_bytes_per_step": 8,
                    "steps": n_e2e, "api": "QwenEngine.forward(token, position)"},
            "clocks": clk.summary(),
            "gpu_launches": launches,
        }
        if batched is not None:
            line["batched"] = batched
            if world == 1 and not args.no_cpu_baseline:
                batched["cpu_baseline"] = dict(
                    cpu_decode(BATCH_PROMPT + 512, 2),
                    note="one sequence at a time: the port decodes the 64 sequences one after "
                         "another at this rate")
        if configs is not None:
            line["configs"] = configs
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
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the single-GEMV, one-layer, greedy-256 and long-context workloads")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
