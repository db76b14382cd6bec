"""The sampler kernel's selection steps, restated in numpy, against the rule
they implement (CPU only).

k_sample draws a token from fixed-point weights E (InferenceEngine.swift:317-367
restated exactly): order by (E desc, id asc), keep the shortest prefix whose sum
reaches thr = floor(S * p24 / 2^24), draw R = floor(K * u24 / 2^24) over the kept
sum K and return the first kept id whose running sum exceeds R.  The kernel finds
the cutoff and the draw with two 4-pass weighted radix selects (8-bit digits).
It builds the first pass of the cutoff select while it computes the weights (S
is the sum of that pass's totals), and it derives the draw's digit totals from
the cutoff select's while the draw's prefix equals the cutoff value's.  The
kernels run the draw beside the cutoff select: after each pass R is
bounded (the kept sum lies in [thr, thr + e_star - 1] and the cutoff's prefix
bounds e_star), and while both ends of that range pick the same digit the next
pass histograms the draw's members beside the cutoff's; otherwise the draw
resumes after the cutoff select, scanning the weights
only after the prefixes part.  The final id is located from the per-rank
weights of the last exchange (the grid kernel's count of the drawn value from that exchange's totals, or
the cutoff's pass-3 totals when the draw ended without a scan).  This file checks that restatement,
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


def kernel(E: np.ndarray, p24: int, u24: int, scans: list, spec: bool = False, C: int = 4,
           fails: list | None = None) -> int:
    """k_sample's select on C ranks' chunks of E.  spec: the draw select runs
    beside the cutoff select (the kernels' mode) while both ends of R's range
    pick the same digit; without it, or from the pass at which the ends part,
    the draw runs after the cutoff select."""
    E = E.astype(np.uint32)
    n = E.size
    chunk = -(-n // C)
    ranks = [slice(r * chunk, min(n, (r + 1) * chunk)) for r in range(C)]
    nz = E != 0
    last = None   # per-rank bins of the last exchange

    def exchange(mn, md, shift):
        per = np.zeros((C, 512 if md is not None else 256), np.int64)
        for r, sl in enumerate(ranks):
            en = E[sl][mn[sl]]
            np.add.at(per[r], (en >> shift) & 255, en.astype(np.int64))
            if md is not None:
                ed = E[sl][md[sl]]
                np.add.at(per[r], 256 + ((ed >> shift) & 255), ed.astype(np.int64))
        return per

    def mask_of(p):
        return 0 if p == 0 else (0xFFFFFFFF << (24 - 8 * p + 8)) & 0xFFFFFFFF

    an = pn = ad = pd = 0
    dmode, dfail, don, dhi = (0 if spec else 2), 0, True, 0
    tot1, above1 = [], []
    thr = R = None
    for p in range(4):
        shift, mask = 24 - 8 * p, mask_of(p)
        dact = dmode == 1
        mn = nz & ((E & mask) == pn)
        md = ((E & mask) == pd) if dact else None
        if md is not None:
            assert not np.any(mn & md)
        last = exchange(mn, md, shift)
        tot = last.sum(0)
        tot1.append(tot[:256].copy())
        if p == 0:
            thr = max(mul_shift24(int(tot[:256].sum()), p24), 1)
        seln, aboven = pick(tot[:256], an, thr)
        pn_new = pn | (seln << shift)
        if p == 3:
            k_tie = -(-(thr - aboven) // pn_new)
            R = mul_shift24(aboven + k_tie * pn_new, u24)
            tl = th = R + 1
        else:
            e_hi = pn_new | ((1 << shift) - 1)
            tl, th = mul_shift24(thr, u24) + 1, mul_shift24(thr + e_hi - 1, u24) + 1
        ndmode, npd, nad, ndhi = dmode, pd, ad, 0
        if dmode == 0:
            if tl > aboven:
                npd, nad = pn_new, aboven
            elif th <= aboven:
                sl_, al = pick(tot[:256], ad, tl)
                sh_, _ = pick(tot[:256], ad, th)
                if sl_ == sh_:
                    ndmode, npd, nad = 1, pd | (sl_ << shift), al
                else:
                    ndmode = 2
            else:
                ndmode = 2
        elif dmode == 1:
            sl_, al = pick(tot[256:], ad, tl)
            sh_, _ = pick(tot[256:], ad, th)
            if sl_ == sh_:
                npd, nad, ndhi = pd | (sl_ << shift), al, 1
            else:
                ndmode = 2
        an, pn = aboven, pn_new
        above1.append(aboven)
        if dmode != 2:
            if ndmode == 2:
                dfail, don = p, dmode == 0
            else:
                pd, ad, dhi = npd, nad, ndhi
            dmode = ndmode
    e_star, above_star = pn, an
    n_scans = 0
    if dmode != 2:
        e2, above, bin3 = pd, ad, (pd & 255) | (256 if dhi else 0)
        tot_real = True
    else:
        if fails is not None and spec:
            fails.append(dfail)
        # draw: derived totals while on e_star's prefix, scans after
        k_tie = (thr - above_star + e_star - 1) // e_star
        prefix, above, on_star = pd, ad, don
        tot_real = False
        for p in range(dfail, 4):
            shift, mask = 24 - 8 * p, mask_of(p)
            ds = (e_star >> shift) & 255
            if on_star:
                tot = np.zeros(256, np.int64)
                tot[ds + 1:] = tot1[p][ds + 1:]
                tot[ds] = (above_star - above1[p]) + k_tie * e_star
            else:
                last = exchange((E > e_star) & ((E & mask) == prefix), None, shift)
                tot = last.sum(0)
                n_scans += 1
                tot_real = p == 3
            d, above = pick(tot, above, R + 1)
            on_star = on_star and d == ds
            prefix |= d << shift
        e2, bin3 = prefix, prefix & 255
    scans.append(n_scans)
    j = (R - above) // e2
    # the grid kernel's count of the drawn value: the last exchange's total at
    # its bin, or the cutoff's pass-3 total when the draw ended without a scan
    total = int(last.sum(0)[bin3]) if tot_real else int(tot1[3][bin3])
    assert total == int(np.count_nonzero(E == e2)) * int(e2)
    # the owning rank from the last exchange's per-rank weights at e2
    w = last[:, bin3]
    assert np.all(w % e2 == 0)
    cnt = w // e2
    before = np.cumsum(cnt) - cnt
    r = int(np.flatnonzero((before <= j) & (j < before + cnt))[0])
    local = np.flatnonzero(E[ranks[r]] == e2)
    return int(local[j - before[r]]) + r * chunk


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


@pytest.mark.parametrize("spec,C", [(False, 4), (True, 4), (True, 8), (True, 16)])
@pytest.mark.parametrize("kind", ["flat", "peaked", "ties", "equal", "dominant", "underflow"])
def test_select_matches_rule(kind, spec, C):
    rng = np.random.default_rng(len(kind))
    scans = []
    for trial in range(12):
        n = int(rng.integers(1, 4000))
        E = weights(rng, kind, n)
        for p24 in (0, 1, int(0.8 * 2 ** 24), int(0.9 * 2 ** 24), 2 ** 24, int(rng.integers(1, 2 ** 24))):
            for u24 in (0, 2 ** 24 - 1, int(rng.integers(0, 2 ** 24))):
                assert kernel(E, p24, u24, scans, spec, C) == rule(E, p24, u24), (kind, trial, p24, u24)
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


def test_speculative_draw_resolves_beside_the_cutoff():
    """With the draw beside the cutoff select, a flat vocabulary-sized
    distribution resolves the draw's first digit beside the cutoff's for every
    u24 (and the second for nearly every); at the third digit a bin holds about one weight and R's range
    (as wide as e_star) straddles a bin edge for a fraction of the draws, which
    take the exact path from there and still match the rule."""
    rng = np.random.default_rng(11)
    E = weights(rng, "flat", 151936)
    scans, fails = [], []
    n = 60
    for t in range(n):
        u24 = int(rng.integers(0, 2 ** 24))
        assert kernel(E, int(0.8 * 2 ** 24), u24, scans, True, 16, fails) == rule(E, int(0.8 * 2 ** 24), u24)
    assert len(fails) <= n // 2, fails
    assert all(f >= 1 for f in fails), fails
    assert sum(scans) <= 3 * len(fails)


def test_speculation_fallback_paths():
    """Weights chosen so that R's range straddles a digit boundary at the first
    pass: the draw leaves the speculation there and resumes exactly, both from
    on e_star and from a parted prefix."""
    found = {"from_star": 0, "from_parted": 0}
    rng = np.random.default_rng(5)
    for trial in range(400):
        n = int(rng.integers(2, 64))
        E = rng.integers(1, 1 << 31, size=n, dtype=np.int64).astype(np.uint32)
        E[rng.integers(n)] = np.uint32(1 << 31)
        for p24 in (int(0.5 * 2 ** 24), int(0.95 * 2 ** 24)):
            u24 = int(rng.integers(0, 2 ** 24))
            scans, fails = [], []
            got = kernel(E, p24, u24, scans, True, 8, fails)
            assert got == rule(E, p24, u24), (trial, p24, u24)
            if fails:
                found["from_star" if scans[0] == 0 or fails[0] == 0 else "from_parted"] += 1
    assert found["from_star"] + found["from_parted"] > 0, found
