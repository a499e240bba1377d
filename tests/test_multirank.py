"""Multi-rank host logic on CPU (gloo, world_size 2): the head partition that
shards a call over GPUs, the post-run gather of per-rank timings and
checksums that bench.py does over NCCL, and a rank that fails before the
gather surfacing as an error on the other rank (no hang)."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import time

import pytest

from conftest import PKG, ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, mode, q):
    sys.path[:0] = [ROOT, PKG]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    import torch.distributed as dist

    import workloads

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=8))
        total = 40  # the video workload's head count
        h0, h1 = workloads.head_range(total, rank, world)
        # stand-in per-rank work: a checksum over the heads this rank owns
        checksum = float(sum(range(h0, h1)))
        ms = 10.0 + 5.0 * rank
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 failed before the gather")
        t0 = time.monotonic()
        stats = workloads.gather_rank_stats(dist, [ms, checksum, h0, h1], "cpu")
        q.put((rank, "ok", stats.tolist(), time.monotonic() - t0))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which asserts on it
        q.put((rank, "error", repr(e), 0.0))


def _run(mode, world=2, limit=60.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.monotonic() + limit
    while len(results) < world and time.monotonic() < deadline:
        try:
            r, status, payload, dt = q.get(timeout=1.0)
            results[r] = (status, payload, dt)
        except Exception:
            pass
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.monotonic()))
        if p.is_alive():
            p.kill()
            p.join()
    return results


def test_head_partition_covers_every_head_once():
    import workloads

    for total in (1, 7, 24, 40, 48, 128):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                h0, h1 = workloads.head_range(total, r, world)
                assert 0 <= h0 <= h1 <= total
                seen.extend(range(h0, h1))
            assert seen == list(range(total))


def test_gather_of_timings_and_checksums_gloo():
    res = _run("ok")
    assert set(res) == {0, 1}, res
    for r in (0, 1):
        status, stats, _ = res[r]
        assert status == "ok", stats
        assert len(stats) == 2
        ms = [row[0] for row in stats]
        assert max(ms) == 15.0  # the job time is the slowest rank's
        heads = [h for row in stats for h in range(int(row[2]), int(row[3]))]
        assert heads == list(range(40))
        assert sum(row[1] for row in stats) == float(sum(range(40)))


def test_failed_rank_surfaces_as_error_not_hang():
    t0 = time.monotonic()
    res = _run("fail", limit=60.0)
    assert time.monotonic() - t0 < 60.0
    assert res[1][0] == "error" and "rank 1 failed" in res[1][1]
    assert res[0][0] == "error", res[0]
