"""Golden tokens for the full-model greedy decode (28 layers, 128 random prompt
ids from seed 1, 256 greedy tokens), produced by the CPU oracle through the
reference's generate loop (InferenceEngine.swift:29-52): every prompt token is
forwarded, the last prompt forward's sample is the first generated token, and
each generated token is fed back.

Weights: tests/model_fixture.make_weight_dir(oracle, 28, WEIGHT_SEED) -- numpy
N(0, 0.02) quantised by the oracle's packAndSave4Bit restatement, so the GPU
test can rebuild the identical directory.  Also records, per generated token,
the oracle's top-2 logit margin (a near tie can flip under the fp16 tolerance).

    python tests/golden/make_config3.py      # several minutes of CPU
"""
from __future__ import annotations

import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle_lib import Oracle, OracleModel  # noqa: E402
from model_fixture import make_weight_dir  # noqa: E402

WEIGHT_SEED = 3
PROMPT_SEED = 1
N_PROMPT = 128
N_GEN = 256
MAX_CTX = 512


def prompt_ids():
    return np.random.default_rng(PROMPT_SEED).integers(0, 151936, size=N_PROMPT).astype(np.int32)


def main() -> None:
    o = Oracle()
    t0 = time.time()
    d = make_weight_dir(o, 28, WEIGHT_SEED)
    print(f"weights in {d} ({time.time() - t0:.0f} s)", flush=True)
    m = OracleModel(o, d, 28, MAX_CTX)
    prompt = prompt_ids().tolist()
    for i, t in enumerate(prompt[:-1]):
        m.forward(t, i, want_logits=False)
    lg = m.forward(prompt[-1], N_PROMPT - 1)
    toks, margins = [], []
    for j in range(N_GEN):
        r = lg[:151666].astype(np.float32)
        top = np.argsort(r)[-2:]
        margins.append(float(r[top[1]] - r[top[0]]))
        cur = o.sample_greedy(lg)
        toks.append(int(cur))
        if j + 1 < N_GEN:
            lg = m.forward(cur, N_PROMPT + j)
        if j % 32 == 0:
            print(f"token {j}: {cur} margin {margins[-1]:.4f} ({time.time() - t0:.0f} s)", flush=True)
    out = {"weight_seed": WEIGHT_SEED, "prompt_seed": PROMPT_SEED, "n_prompt": N_PROMPT,
           "tokens": toks, "top2_margin": margins}
    with open(os.path.join(HERE, "config3_greedy256.json"), "w") as f:
        json.dump(out, f)
    print("done", time.time() - t0)


if __name__ == "__main__":
    main()
