"""The fused decode step's per-CTA work schedule, checked on the CPU.

`qwen_fused_schedule` (a test hook of libqwen_b200.so) returns the schedule
build_fused_weights uploads: each CTA's weight items in stream order, packed as
fused.h describes (phase, tile, k0, nk, last, seq).  k_decode_fused relies on
these properties of it:

  * every tile of every matrix is covered over its whole K exactly once; the
    down projection is streamed by MLP unit: unit u's item covers block pair
    u of all 96 row tiles, in 4 chunks of 24 row tiles (k0 / nk count row
    tiles there);
  * a CTA's items are in stream order (phases ascending, a tile's chunks
    consecutive and ascending, `last` on its final chunk);
  * QKV tiles sit on the first 128 CTAs, one each (the attention units use
    the last CTAs); a CTA holds at most one O tile per layer; a QKV or O tile
    is one item over its whole K (warp w takes block pairs w, w+8, w+16);
  * CTA u < 140 owns MLP unit u: gate/up tiles 8u .. 8u+7 (seq 0..7, one item
    each, warp w takes item cur + w) and the down strip of unit u; the other
    CTAs own none;
  * `seq` numbers a CTA's tiles within a phase 0, 1, 2, ...;
  * an LM-head tile's chunks are 24 k16 steps (4 per tile), and tile ownership
    (seq % 8) gives every warp whole tiles;
  * no CTA exceeds the shared-memory item table (768 items) or is empty.
"""
import ctypes

import numpy as np
import pytest

from qweninferenceengine_b200 import _lib

PH_QKV, PH_ATTN, PH_O, PH_GU, PH_DOWN = range(5)
TILES = {PH_QKV: 128, PH_O: 96, PH_GU: 1120, PH_DOWN: 140}   # down: MLP units
KSTEPS = {PH_QKV: 24, PH_O: 24, PH_GU: 24, PH_DOWN: 96}   # block pairs (down: row tiles; LM: k16 steps)
MLP_UNITS, DOWN_CHUNK = 140, 24
LM_TILES, LM_STEPS, LM_CHUNK = 151936 // 16, 96, 24
MAX_ITEMS = 768


def schedule(n_layers, grid):
    lib = ctypes.CDLL(_lib.LIB_PATH)
    f = lib.qwen_fused_schedule
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p]
    f.restype = ctypes.c_longlong
    cap = 200_000
    items = np.zeros(cap, np.uint64)
    begin = np.zeros(grid + 1, np.uint32)
    n = f(n_layers, grid, items.ctypes.data, cap, begin.ctypes.data)
    assert n > 0
    return items[:n], begin


def unpack(w):
    w = int(w)
    return (w & 0xFF, (w >> 8) & 0x3FFF, (w >> 22) & 0xFF, (w >> 30) & 0xFF, (w >> 38) & 1,
            (w >> 39) & 0xFF)


def test_hook_rejects_bad_arguments():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    f = lib.qwen_fused_schedule
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p]
    f.restype = ctypes.c_longlong
    items = np.zeros(16, np.uint64)
    begin = np.zeros(200, np.uint32)
    assert f(0, 148, items.ctypes.data, 16, begin.ctypes.data) == -1
    assert f(28, 148, items.ctypes.data, 16, begin.ctypes.data) == -1     # capacity too small
    assert f(28, 148, None, 16, begin.ctypes.data) == -1
    big = np.zeros(200_000, np.uint64)
    assert f(28, 132, big.ctypes.data, big.size, begin.ctypes.data) == -1   # fewer CTAs than MLP units


@pytest.mark.parametrize("n_layers,grid", [(28, 148), (4, 148), (1, 148), (28, 140), (2, 160)])
def test_schedule_invariants(n_layers, grid):
    items, begin = schedule(n_layers, grid)
    lm_phase = n_layers * 5
    assert begin[0] == 0 and begin[grid] == len(items)
    assert np.all(np.diff(begin.astype(np.int64)) >= 1), "a CTA has no work (or overflowed its table)"
    assert int(np.max(np.diff(begin.astype(np.int64)))) <= MAX_ITEMS
    cover = {}
    for c in range(grid):
        its = [unpack(w) for w in items[begin[c]:begin[c + 1]]]
        phases = [it[0] for it in its]
        assert phases == sorted(phases), "items out of stream order"
        per_phase = {}
        prev = None
        for (ph, tile, k0, nk, last, seq) in its:
            assert nk >= 1
            if ph == lm_phase:
                assert nk == LM_CHUNK and k0 % LM_CHUNK == 0 and k0 + nk <= LM_STEPS
                assert last == (k0 + nk == LM_STEPS)
            else:
                kind = ph % 5
                assert kind in TILES and tile < TILES[kind]
                assert k0 + nk <= KSTEPS[kind]
                assert last == (k0 + nk == KSTEPS[kind])
                if kind in (PH_QKV, PH_O):
                    assert k0 == 0 and nk == KSTEPS[kind], "a QKV / O tile must be one item"
                if kind == PH_GU:
                    assert k0 == 0 and nk == KSTEPS[PH_GU], "a gate/up tile must be one item"
                    assert tile // 8 == c and seq == tile % 8, "unit c's tiles 8c .. 8c+7 on CTA c"
                if kind == PH_DOWN:
                    assert tile == c and nk == DOWN_CHUNK and k0 % DOWN_CHUNK == 0
            # a tile's chunks are consecutive and ascending
            if prev is not None and (prev[0], prev[1]) == (ph, tile):
                assert k0 == prev[2] + prev[3]
            else:
                assert k0 == 0, "a tile starts at k0 = 0"
                tiles = per_phase.setdefault(ph, [])
                assert seq == len(tiles), "seq numbers a CTA's tiles of a phase 0, 1, 2, ..."
                tiles.append(tile)
            assert seq == len(per_phase[ph]) - 1
            key = (ph, tile)
            cover.setdefault(key, []).append((k0, nk))
            prev = (ph, tile, k0, nk)
        for ph, tiles in per_phase.items():
            if ph == lm_phase:
                continue
            kind = ph % 5
            if kind == PH_QKV:
                assert c < 128 and len(tiles) == 1
            elif kind in (PH_O, PH_DOWN):
                assert len(tiles) <= 1
            elif kind == PH_GU:
                assert c < MLP_UNITS and len(tiles) == 8
    # every tile covered over its whole K exactly once
    for layer in range(n_layers):
        for kind, n in TILES.items():
            for t in range(n):
                ranges = sorted(cover.get((layer * 5 + kind, t), []))
                assert ranges, ("tile missing", layer, kind, t)
                pos = 0
                for k0, nk in ranges:
                    assert k0 == pos, ("gap or overlap", layer, kind, t)
                    pos += nk
                assert pos == KSTEPS[kind]
    for t in range(LM_TILES):
        ranges = sorted(cover.get((lm_phase, t), []))
        assert [k0 for k0, _ in ranges] == list(range(0, LM_STEPS, LM_CHUNK)), ("LM tile", t)
    assert len(cover) == n_layers * sum(TILES.values()) + LM_TILES
