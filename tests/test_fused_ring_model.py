"""The fused decode step's weight ring, modelled on the CPU.

k_decode_fused streams each CTA's weight items through kNS = 14 shared-memory
slots.  Item i lives in slot i % 14.  The first 14 items are issued at start;
after that, item i + 14 is issued by the warp whose release completes item i's
eight release shares.  A per-slot counter collects the shares, and a per-slot
tag (slot_item) names the item issued into the slot.  A warp waits for
slot_item == i before its parity wait on the slot's full barrier, which keeps
a warp that runs ahead from taking the previous ring lap's phase for its own.

Release shares per phase, as the kernel gives them:
  * k-split tiles (QKV, O): all 8 warps read every chunk, one share each;
  * the MLP unit's gate/up tiles: one warp per tile (item j of the phase ->
    warp j), 8 shares;
  * the unit's down strip (4 items of 24 row tiles): warps 2j and 2j+1 read
    item j, 12 row tiles and 4 shares each;
  * LM head: tile t's chunks belong to warp t % 8, 8 shares each.
All warps meet at a barrier between phases.

The model runs the warps, the copy engine (bytes land in any order) and the
refills under random schedules, with the full barrier's parity semantics: a
wait for parity P passes when the slot's completed-phase count has the other
parity, so the phase two laps back would also pass it.  It checks that no slot
is rewritten before its eight shares are in, that every wait sees the item it
expects, and that every schedule finishes.
"""
import random

import pytest

KNS = 14
WARPS = 8
DOWN_ITEMS = 4


def layer_items(n_gu):
    """(phase, tile, chunk) items of one layer for one CTA, in stream order
    (n_gu = 8 for a CTA that owns an MLP unit, 0 for one that does not)."""
    items = [("qkv", 0, 0), ("o", 0, 0)]
    items += [("gu", t, 0) for t in range(n_gu)]
    if n_gu:
        items += [("down", 0, c) for c in range(DOWN_ITEMS)]
    return items


def plan(n_layers, n_gu, n_lm_tiles, lm_chunks=4):
    """Per item: its phase index and {warp: shares}; per warp: its item order."""
    items, shares, phase_of = [], [], []
    ph = 0
    for _ in range(n_layers):
        lay = layer_items(n_gu)
        for kind in ("qkv", "o", "gu", "down"):
            for (k, t, c) in lay:
                if k != kind:
                    continue
                if k in ("qkv", "o"):
                    sh = {w: 1 for w in range(WARPS)}
                elif k == "down":
                    sh = {2 * c: WARPS // 2, 2 * c + 1: WARPS // 2}
                else:
                    sh = {t % WARPS: WARPS}
                items.append((k, t, c))
                shares.append(sh)
                phase_of.append(ph)
            ph += 1
    for t in range(n_lm_tiles):
        for c in range(lm_chunks):
            items.append(("lm", t, c))
            shares.append({t % WARPS: WARPS})
            phase_of.append(ph)
    ph += 1
    for sh in shares:
        assert sum(sh.values()) == WARPS
    return items, shares, phase_of, ph


def simulate(n_layers, n_gu, n_lm_tiles, seed):
    rnd = random.Random(seed)
    items, shares, phase_of, n_phases = plan(n_layers, n_gu, n_lm_tiles)
    n = len(items)
    slot_item = [-1] * KNS
    rel_cnt = [0] * KNS
    landed = [None] * KNS      # item whose bytes are in the slot
    completed = [0] * KNS      # phases of the slot's full barrier completed
    reads_left = [0] * n       # shares still to come for item i
    inflight = []
    at_barrier = [0] * n_phases

    def issue(i):
        s = i % KNS
        if slot_item[s] >= 0:
            j = slot_item[s]
            assert reads_left[j] == 0, ("slot rewritten before item %d was released" % j, i)
        slot_item[s] = i
        landed[s] = None
        reads_left[i] = WARPS
        inflight.append(i)

    for i in range(min(KNS, n)):
        issue(i)

    def warp(w):
        for ph in range(n_phases):
            for i in range(n):
                if phase_of[i] != ph or w not in shares[i]:
                    continue
                while slot_item[i % KNS] != i:
                    yield
                parity = (i // KNS) & 1
                while (completed[i % KNS] & 1) == parity:   # try_wait.parity
                    yield
                assert landed[i % KNS] == i, ("parity wait passed on another lap's phase", i)
                yield  # reading the slot
                assert landed[i % KNS] == i, ("slot changed under a reader", i)
                sh = shares[i][w]
                reads_left[i] -= sh
                s = i % KNS
                rel_cnt[s] += sh
                if rel_cnt[s] == WARPS:
                    rel_cnt[s] = 0
                    if i + KNS < n:
                        issue(i + KNS)
            at_barrier[ph] += 1
            while at_barrier[ph] < WARPS:
                yield

    def copy_engine():
        while True:
            if inflight and rnd.random() < 0.4:
                i = inflight.pop(rnd.randrange(len(inflight)))
                landed[i % KNS] = i
                completed[i % KNS] += 1
            yield

    actors = [warp(w) for w in range(WARPS)] + [copy_engine()]
    alive = list(actors[:WARPS])
    steps = 0
    while alive:
        a = rnd.choice(alive + [actors[WARPS]])
        try:
            next(a)
        except StopIteration:
            alive.remove(a)
        steps += 1
        assert steps < 3_000_000, "no progress: a wait never completes"
    assert all(r == 0 for r in reads_left), "an item was not fully released"
    assert not inflight


@pytest.mark.parametrize("n_gu", [0, 8])
@pytest.mark.parametrize("seed", range(4))
def test_ring_protocol(n_gu, seed):
    simulate(n_layers=2, n_gu=n_gu, n_lm_tiles=20, seed=seed)


def test_model_catches_a_missing_slot_tag_check():
    """Without the slot tag a warp that runs ahead can pass its parity wait on
    the phase two laps back: the model must see it (it is why the kernel keeps
    the tag)."""
    src = open(__file__).read()
    bad = src.replace("                while slot_item[i % KNS] != i:\n                    yield\n", "", 1)
    assert bad != src
    ns = {"__name__": "bad_model", "__file__": __file__}
    exec(compile(bad, "bad_model", "exec"), ns)
    caught = 0
    for seed in range(20):
        try:
            ns["simulate"](n_layers=1, n_gu=8, n_lm_tiles=30, seed=seed)
        except AssertionError:
            caught += 1
    assert caught > 0


def simulate_abort(n_layers, n_gu, n_lm_tiles, seed, propagate=True, drain_by_count=True):
    """The ring when another CTA gives up part way (the global error word is set
    at a random moment).  From then on a warp's wait returns false as soon as it
    looks (skipping the read) and the warp still releases its share, as the
    kernel does.  With `propagate` the warp that sees the error raises the
    CTA's own abort flag first, and a completed release refills only while that
    flag is clear; without it (the kernel before the fix) only the CTA that timed
    out stops refilling.  At exit thread 0 drains: per slot it waits (bounded)
    on the phase of the slot's last copy -- by the count of copies issued into
    the slot, or (the old way) by the last item's index.  Returns the problems
    seen: a second copy put in flight into a slot, or a copy still in flight
    when the CTA exits."""
    rnd = random.Random(seed)
    items, shares, phase_of, n_phases = plan(n_layers, n_gu, n_lm_tiles)
    n = len(items)
    slot_item = [-1] * KNS
    issued = [0] * KNS
    rel_cnt = [0] * KNS
    completed = [0] * KNS
    inflight = []
    problems = []
    err = [False]
    local_abort = [False]
    strike = rnd.randrange(50, 4000)
    at_barrier = [0] * n_phases

    def issue(i):
        s = i % KNS
        if any(j % KNS == s for j in inflight):
            problems.append(("second copy in flight", s))
        slot_item[s] = i
        issued[s] += 1
        inflight.append(i)

    for i in range(min(KNS, n)):
        issue(i)

    def aborted():
        if local_abort[0]:
            return True
        if err[0]:
            if propagate:
                local_abort[0] = True
            return True
        return False

    def warp(w):
        for ph in range(n_phases):
            for i in range(n):
                if phase_of[i] != ph or w not in shares[i]:
                    continue
                ok = True
                while slot_item[i % KNS] != i:
                    if aborted():
                        ok = False
                        break
                    yield
                if ok:
                    parity = (i // KNS) & 1
                    while (completed[i % KNS] & 1) == parity:
                        if aborted():
                            ok = False
                            break
                        yield
                yield
                s = i % KNS
                rel_cnt[s] += shares[i][w]
                if rel_cnt[s] == WARPS:
                    rel_cnt[s] = 0
                    if i + KNS < n and not local_abort[0]:
                        issue(i + KNS)
            at_barrier[ph] += 1
            while at_barrier[ph] < WARPS:
                yield

    def copy_engine():
        while True:
            if inflight and rnd.random() < 0.4:
                i = inflight.pop(rnd.randrange(len(inflight)))
                completed[i % KNS] += 1
            yield

    eng = copy_engine()
    alive = [warp(w) for w in range(WARPS)]
    steps = 0
    while alive:
        steps += 1
        if steps == strike:
            err[0] = True
        a = rnd.choice(alive + [eng])
        try:
            next(a)
        except StopIteration:
            alive.remove(a)
        assert steps < 3_000_000
    for s in range(KNS):                       # the drain, a bounded wait per slot
        if issued[s] == 0:
            continue
        parity = (issued[s] - 1) & 1 if drain_by_count else (slot_item[s] // KNS) & 1
        for _ in range(2000):
            if (completed[s] & 1) != parity:
                break
            next(eng)
    if inflight:
        problems.append(("copy in flight at exit", len(inflight)))
    return problems


@pytest.mark.parametrize("seed", range(40))
def test_abort_path_leaves_no_copy_in_flight(seed):
    assert simulate_abort(n_layers=1, n_gu=8, n_lm_tiles=30, seed=seed) == []


def test_model_catches_the_unpropagated_abort():
    """The kernel before the fix (a CTA kept refilling after another CTA's
    timeout, and drained by item index) could exit with a copy in flight --
    the model must show it."""
    bad = sum(bool(simulate_abort(n_layers=1, n_gu=8, n_lm_tiles=30, seed=s, propagate=False,
                                  drain_by_count=False)) for s in range(40))
    assert bad > 0
