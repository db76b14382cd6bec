"""The batched tensor-core GEMM's launch plans and its barrier protocol, on the
CPU.

`qwen_tc_gemm_plan` (a test hook of libqwen_b200.so) returns the plan
launch_tc_gemm uses for a shape: unit (64-k chunks per pipeline unit), A
stages, activation stages, raw Q4 stages, MMA warps, dequantising groups and
shared memory.  The kernel's mbarrier waits are parity waits, which cannot tell
a phase from the one two fills earlier; the plan must therefore keep every
waiter at most one phase behind.  These tests check the plan's invariants for
many shapes, then run a model of the kernel's roles (producer, copy engine,
dequantising warps, MMA warps) with the product's plans under random schedules:
every wait must see exactly the fill it expects, no slot may be overwritten
before it was read, and every schedule must finish.
"""
import ctypes
import random

import pytest

from qweninferenceengine_b200 import _lib

SMEM_BUDGET = 227 * 1024
TMEM_COLS = 512


def plan(nb, q4, cps):
    lib = ctypes.CDLL(_lib.LIB_PATH)
    f = lib.qwen_tc_gemm_plan
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_longlong)]
    f.restype = ctypes.c_int
    out = (ctypes.c_longlong * 7)()
    rc = f(nb, 1 if q4 else 0, cps, out)
    unit, st, xs, rs, mw, ng, smem = list(out)
    return rc, dict(unit=unit, stages=st, xstages=xs, raw=rs, mma_warps=mw, groups=ng, smem=smem)


SHAPES = [(nb, q4, cps) for nb in (16, 32, 48, 64, 128, 256) for q4 in (True, False)
          for cps in list(range(1, 41)) + [70, 140]]


@pytest.mark.parametrize("nb,q4,cps", SHAPES)
def test_plan_invariants(nb, q4, cps):
    rc, p = plan(nb, q4, cps)
    assert rc == 0 and p["smem"] <= SMEM_BUDGET
    nu = cps // p["unit"]
    assert cps % p["unit"] == 0
    acc = 32 if nb <= 32 else 64 if nb <= 64 else 128 if nb <= 128 else 256
    a_cols = p["stages"] * p["unit"] * 32 if q4 else 0
    assert acc * p["mma_warps"] + a_cols <= TMEM_COLS
    # activation ring: at least min(nu, A stages); even when refilled with two MMA warps
    assert p["xstages"] >= min(nu, p["stages"])
    if p["xstages"] < nu and p["mma_warps"] == 2:
        assert p["xstages"] % 2 == 0
    if q4:
        # one A stage per dequantising group or more: a group's wait for unit i - S
        # must imply unit i - 2S (its previous unit is i - groups)
        assert p["stages"] >= p["groups"]
        # a refilled raw ring is reused by the same group
        assert p["raw"] >= 1
        if p["raw"] < nu:
            assert p["raw"] % p["groups"] == 0
    else:
        assert p["raw"] == 0


# ------------------------------------------------------------------ model --
class Bar:
    """mbarrier: `count` arrivals plus pending transaction bytes complete a phase;
    try_wait(parity) succeeds when the phase of that parity is not the current one."""

    def __init__(self, count):
        self.count, self.pending, self.phase, self.tx = count, count, 0, 0

    def arrive(self):
        self.pending -= 1
        self._check()

    def expect(self):
        self.tx += 1
        self.pending -= 1
        self._check()

    def complete_tx(self):
        self.tx -= 1
        self._check()

    def _check(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, parity):
        return (self.phase & 1) != parity


def simulate(nu, S, XS, RS, q4, groups, mma_warps, seed):
    rnd = random.Random(seed)
    NW = RS if q4 else S
    wfull = [Bar(1) for _ in range(NW)]
    rempty = [Bar(4) for _ in range(RS)]
    xfull = [Bar(1) for _ in range(XS)]
    xempty = [Bar(1) for _ in range(XS)]
    deq = [Bar(4) for _ in range(S)]
    aempty = [Bar(1) for _ in range(S)]
    inflight, done = [], []
    slot_a, slot_r, slot_x = [None] * S, [None] * max(RS, 1), [None] * XS
    reads = {}

    def producer():
        def load_w(i):
            wfull[i % NW].expect()
            inflight.append(("w", i, i % NW))

        def load_x(i):
            xfull[i % XS].expect()
            inflight.append(("x", i, i % XS))

        nw, nx = min(nu, NW), min(nu, XS)
        for i in range(nw):
            load_w(i)
        for i in range(nx):
            load_x(i)
        t = 0
        while nw < nu or nx < nu:
            if nw < nu:
                bar, par = (rempty[t % RS], (t // RS) & 1) if q4 else (aempty[t % S], (t // S) & 1)
                while not bar.done(par):
                    yield
                load_w(nw)
                nw += 1
            if nx < nu:
                while not xempty[t % XS].done((t // XS) & 1):
                    yield
                load_x(nx)
                nx += 1
            t += 1

    def copy_engine():
        while True:
            if inflight and rnd.random() < 0.5:
                kind, i, s = inflight.pop(rnd.randrange(len(inflight)))
                if kind == "w":
                    if q4:
                        assert slot_r[s] in (None, "read"), ("raw slot overwritten", i)
                        slot_r[s] = ("w", i)
                    else:
                        assert slot_a[s] in (None, "used"), ("A slot overwritten", i)
                        slot_a[s] = ("w", i)
                    wfull[s].complete_tx()
                else:
                    assert slot_x[s] in (None, "used"), ("activation slot overwritten", i)
                    slot_x[s] = ("x", i)
                    xfull[s].complete_tx()
            yield

    def dequant_warp(g, w):
        for i in range(g, nu, groups):
            s, rs = i % S, i % RS
            while not wfull[rs].done((i // RS) & 1):
                yield
            assert slot_r[rs] == ("w", i), ("raw wait passed early", i, slot_r[rs])
            yield
            reads[i] = reads.get(i, 0) + 1
            if reads[i] == 4:
                slot_r[rs] = "read"
            rempty[rs].arrive()
            if i >= S:
                while not aempty[s].done(((i // S) - 1) & 1):
                    yield
            assert slot_a[s] in (None, "used", ("d", i)), ("A stage busy", i, slot_a[s])
            slot_a[s] = ("d", i)
            if w == 0:  # one warp of the group also waits for the unit's activations
                while not xfull[i % XS].done((i // XS) & 1):
                    yield
                assert slot_x[i % XS] == ("x", i), ("activation wait passed early", i)
            deq[s].arrive()

    def mma_warp(m):
        for i in range(m, nu, mma_warps):
            s, xs = i % S, i % XS
            if q4:
                while not deq[s].done((i // S) & 1):
                    yield
            else:
                while not wfull[s].done((i // S) & 1):
                    yield
                while not xfull[xs].done((i // XS) & 1):
                    yield
            assert slot_a[s] == (("d", i) if q4 else ("w", i)), ("MMA read a stale A stage", i)
            assert slot_x[xs] == ("x", i), ("MMA read stale activations", i)
            yield
            slot_a[s], slot_x[xs] = "used", "used"
            aempty[s].arrive()
            xempty[xs].arrive()
            done.append(i)

    actors = [producer(), copy_engine()] + [mma_warp(m) for m in range(mma_warps)]
    if q4:
        actors += [dequant_warp(g, w) for g in range(groups) for w in range(4)]
    alive, steps = list(actors), 0
    while len(done) < nu:
        a = rnd.choice(alive)
        try:
            next(a)
        except StopIteration:
            alive.remove(a)
        steps += 1
        assert steps < 2_000_000, "no progress: a wait never completes"


# the launches the engine makes (64 sequences, 128-row prefill, 256 rows), and more
PROTOCOL_SHAPES = [(64, True, 24), (64, True, 14), (64, True, 3), (64, True, 2), (128, True, 24),
                   (256, True, 24), (64, False, 24), (256, False, 24), (16, True, 40),
                   (48, True, 9), (128, True, 70), (32, False, 7)]


@pytest.mark.parametrize("nb,q4,cps", PROTOCOL_SHAPES)
def test_protocol_model(nb, q4, cps):
    rc, p = plan(nb, q4, cps)
    assert rc == 0
    nu = cps // p["unit"]
    for seed in range(2):
        simulate(nu, p["stages"], p["xstages"], p["raw"], q4, p["groups"], p["mma_warps"], seed)


def test_model_catches_unsafe_plans():
    """The model is sensitive: a raw ring that is not a multiple of the group
    count, or an activation ring shallower than the A stages, fails."""
    for bad in ((24, 4, 6, 6, True, 4, 2), (24, 4, 3, 8, True, 4, 2)):
        caught = 0
        for seed in range(10):
            try:
                simulate(*bad, seed)
            except AssertionError:
                caught += 1
        assert caught > 0, bad
