"""The sampler kernel's selection steps, restated in numpy, against the rule
they implement (CPU only).

k_sample draws a token from fixed-point weights E (InferenceEngine.swift:317-367
restated exactly): order by (E desc, id asc), keep the shortest prefix whose sum
reaches thr = floor(S * p24 / 2^24), draw R = floor(K * u24 / 2^24) over the kept
sum K and return the first kept id whose running sum exceeds R.  The kernel finds
the cutoff and the draw with two 4-pass weighted radix selects (8-bit digits).
It builds the first pass of the cutoff select while it computes the weights (S
is the sum of that pass's totals), and it derives the draw's digit totals from
the cutoff select's while the draw's prefix equals the cutoff value's, scanning
the weights only after the prefixes part.  This file checks that restatement,
pass for pass as the kernel runs it, against a plain sort over many weight
distributions (ties at the cutoff, all-equal weights, one dominant weight, zero
weights, u24 and top-p at their ends).
"""
import numpy as np
import pytest


def mul_shift24(a: int, b: int) -> int:
    return (a >> 24) * b + (((a & 0xFFFFFF) * b) >> 24)


def rule(E: np.ndarray, p24: int, u24: int) -> int:
    """The reference's steps on fixed-point weights: stable order, prefix, draw."""
    order = np.lexsort((np.arange(E.size), -E.astype(np.int64)))
    w = E[order].astype(object)
    S = int(E.astype(np.int64).sum())
    thr = max(mul_shift24(S, p24), 1)
    run, n_keep = 0, 0
    for n_keep, v in enumerate(w, 1):
        run += int(v)
        if run >= thr:
            break
    K = run
    R = mul_shift24(K, u24)
    run = 0
    for i in range(n_keep):
        run += int(w[i])
        if run > R:
            return int(order[i])
    raise AssertionError("no id drawn")


def totals(E, member, shift):
    t = np.zeros(256, np.int64)
    np.add.at(t, (E[member] >> shift) & 255, E[member].astype(np.int64))
    return t


def pick(tot, above, target):
    """Largest digit d with above + sum(tot[d:]) >= target (0 when short) and the
    weight above it, as the kernel's pick_digit."""
    run = above
    for d in range(255, -1, -1):
        if run + int(tot[d]) >= target or d == 0:
            return d, run
        run += int(tot[d])


def kernel(E: np.ndarray, p24: int, u24: int, scans: list) -> int:
    E = E.astype(np.uint32)
    nz = E != 0
    # cutoff select; pass 0 comes with the weights, S from its totals
    tot1, above1 = [], []
    prefix = mask = above = 0
    thr = None
    for p in range(4):
        shift = 24 - 8 * p
        tot = totals(E, nz & ((E & mask) == prefix), shift)
        if p == 0:
            thr = max(mul_shift24(int(tot.sum()), p24), 1)
        tot1.append(tot)
        d, above = pick(tot, above, thr)
        prefix |= d << shift
        mask |= 255 << shift
        above1.append(above)
    e_star, above_star = prefix, above
    k_tie = (thr - above_star + e_star - 1) // e_star
    kept = above_star + k_tie * e_star
    R = mul_shift24(kept, u24)
    # draw: derived totals while on e_star's prefix, scans after
    prefix = mask = above = 0
    on_star, n_scans = True, 0
    for p in range(4):
        shift = 24 - 8 * p
        ds = (e_star >> shift) & 255
        if on_star:
            tot = np.zeros(256, np.int64)
            tot[ds + 1:] = tot1[p][ds + 1:]
            tot[ds] = (above_star - above1[p]) + k_tie * e_star
        else:
            tot = totals(E, (E > e_star) & ((E & mask) == prefix), shift)
            n_scans += 1
        d, above = pick(tot, above, R + 1)
        on_star = on_star and d == ds
        prefix |= d << shift
        mask |= 255 << shift
    scans.append(n_scans)
    e2 = prefix
    j = (R - above) // e2
    ids = np.flatnonzero(E == e2)
    return int(ids[j])


def weights(rng, kind, n):
    if kind == "flat":
        x = rng.standard_normal(n) * rng.uniform(0.05, 0.5)
    elif kind == "peaked":
        x = rng.standard_normal(n) * rng.uniform(2, 8)
    elif kind == "ties":
        x = rng.integers(0, 6, size=n) * 0.25
    elif kind == "equal":
        x = np.zeros(n)
    elif kind == "dominant":
        x = rng.standard_normal(n) * 0.3
        x[rng.integers(n)] = 40.0
    else:  # underflow: most weights truncate to zero
        x = rng.standard_normal(n) * 30
    e = np.exp(np.minimum(x - x.max(), 0.0))
    return np.floor(e * 2.0 ** 31).astype(np.uint64).clip(0, 2 ** 31).astype(np.uint32)


@pytest.mark.parametrize("kind", ["flat", "peaked", "ties", "equal", "dominant", "underflow"])
def test_select_matches_rule(kind):
    rng = np.random.default_rng(len(kind))
    scans = []
    for trial in range(12):
        n = int(rng.integers(1, 4000))
        E = weights(rng, kind, n)
        for p24 in (0, 1, int(0.8 * 2 ** 24), int(0.9 * 2 ** 24), 2 ** 24, int(rng.integers(1, 2 ** 24))):
            for u24 in (0, 2 ** 24 - 1, int(rng.integers(0, 2 ** 24))):
                assert kernel(E, p24, u24, scans) == rule(E, p24, u24), (kind, trial, p24, u24)
    assert len(scans) == 12 * 18


def test_draw_scans_only_after_the_prefixes_part():
    """A draw inside the cutoff's tie group scans nothing; one at the top of a
    flat distribution parts from the cutoff's prefix in the first pass."""
    E = np.full(1000, 1 << 30, np.uint32)
    scans = []
    assert kernel(E, int(0.5 * 2 ** 24), 12345, scans) == rule(E, int(0.5 * 2 ** 24), 12345)
    assert scans == [0]
    rng = np.random.default_rng(3)
    E = weights(rng, "flat", 3000)
    scans = []
    assert kernel(E, int(0.9 * 2 ** 24), 0, scans) == rule(E, int(0.9 * 2 ** 24), 0)
    assert scans[0] == 3
