"""Multi-GPU is replicas only: every rank decodes its own sequences and the
ranks meet only on the host (a start/stop barrier and the max-over-ranks time,
over gloo).  These tests run that host-side plumbing of bench.py with two gloo
ranks on CPU (127.0.0.1) -- no GPU, no data-path collective."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _rank(rank: int, world: int, port: int, out):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from datetime import timedelta

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    r, w, local = bench.dist_env()
    bench.replica_barrier(w)
    ms = 100.0 + 50.0 * r                       # rank 1 is the slow one
    ms_max = bench.replica_max(ms, w)
    tok_s = bench.replica_tokens_per_s(w, 64 * 10, ms_max)
    bench.replica_barrier(w)
    dist.destroy_process_group()
    out.put((r, w, local, ms_max, tok_s))


def test_two_replicas_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(i, 2, port, q)) for i in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[0] for r in res] == [0, 1] and all(r[1] == 2 for r in res)
    assert [r[2] for r in res] == [0, 1]
    # every rank sees the slowest rank's time and the same whole-job throughput
    assert all(r[3] == pytest.approx(150.0) for r in res)
    assert all(r[4] == pytest.approx(2 * 640 / 0.150) for r in res)


def test_single_replica_needs_no_process_group():
    sys.path.insert(0, ROOT)
    import bench

    assert bench.replica_max(3.5, 1) == 3.5
    assert bench.replica_tokens_per_s(1, 200, 100.0) == pytest.approx(2000.0)
