"""Multi-process host logic of the request-sharded multi-GPU path, on CPU.

Two gloo ranks (spawned processes, rendezvous on 127.0.0.1) exercise what a
torchrun launch of ``bench.py --gpus N`` relies on: every rank computes the
same longest-processing-time partition of the requests, the end-of-run
statistics reduce (SUM of counters, MAX of elapsed time), and -- the failure
case -- a rank that dies before the reduce makes the surviving rank's
collective fail within the process group's timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
import traceback

import pytest
import torch.multiprocessing as mp

from microserve_b200 import distributed


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    distributed.init("gloo", timeout_s=timeout_s)


def _worker_reduce(rank: int, world: int, port: int, out) -> None:
    try:
        _init(rank, world, port, 30.0)
        costs = [float((7 * i) % 13 + 1) for i in range(21)]
        mine = distributed.shard_requests(costs, world, rank)
        counters = {"emitted": 10 * (rank + 1), "accepted": rank + 3}
        tot, t = distributed.reduce_stats(counters, 0.5 + rank)
        distributed.barrier()
        out.put((rank, mine, tot, t))
        distributed.shutdown()
    except Exception:  # report instead of dying silently
        out.put((rank, "error", traceback.format_exc(), None))


def _worker_dies(rank: int, world: int, port: int, out) -> None:
    try:
        _init(rank, world, port, 5.0)
        distributed.barrier()  # both ranks are up
        if rank == 1:
            os._exit(3)  # leaves between steps, nothing in flight
        try:
            distributed.reduce_stats({"emitted": 1}, 1.0)
            out.put((rank, "no error"))
        except Exception as e:  # the expected outcome
            out.put((rank, type(e).__name__))
    except Exception:
        out.put((rank, "setup: " + traceback.format_exc()))


def _run(target, world: int, timeout_s: float):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for p in procs:
        p.join(timeout_s)
    while not out.empty():
        results.append(out.get())
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return results, procs


def test_shard_requests_is_a_deterministic_balanced_partition() -> None:
    costs = [float((7 * i) % 13 + 1) for i in range(101)]
    parts = [distributed.shard_requests(costs, 4, r) for r in range(4)]
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(len(costs)))
    loads = [sum(costs[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(costs)  # LPT bound
    assert parts == [distributed.shard_requests(costs, 4, r) for r in range(4)]
    assert distributed.shard_requests(costs, 1, 0) == list(range(len(costs)))


def test_two_gloo_ranks_shard_and_reduce() -> None:
    results, procs = _run(_worker_reduce, 2, 120.0)
    assert all(p.exitcode == 0 for p in procs), results
    by_rank = {r[0]: r for r in results}
    assert sorted(by_rank) == [0, 1], results
    for r in (0, 1):
        assert by_rank[r][1] != "error", by_rank[r][2]
    costs = [float((7 * i) % 13 + 1) for i in range(21)]
    assert sorted(by_rank[0][1] + by_rank[1][1]) == list(range(21))
    assert by_rank[0][1] == distributed.shard_requests(costs, 2, 0)
    for r in (0, 1):
        _, _, tot, t = by_rank[r]
        assert tot == {"emitted": 30, "accepted": 7}
        assert t == pytest.approx(1.5)


def test_a_rank_that_dies_fails_the_survivors_collective() -> None:
    results, procs = _run(_worker_dies, 2, 120.0)
    assert not any(p.is_alive() for p in procs)
    assert procs[1].exitcode == 3
    survivor = [r for r in results if r[0] == 0]
    assert survivor, results
    assert survivor[0][1] not in ("no error",) and not survivor[0][1].startswith("setup"), survivor


def test_strong_scaling_request_sets_do_not_depend_on_the_gpu_count() -> None:
    """bench.py --total-requests: every request lands on exactly one rank for
    any world size, and its token ids, context and generator seed depend
    only on its global id -- the premise of identical streams at any N."""
    import argparse
    import sys

    import numpy as np

    from .conftest import ROOT

    sys.path.insert(0, str(ROOT))
    import bench

    args = argparse.Namespace(total_requests=96, requests=256, ctx_min=8, ctx_max=300, seed=3,
                              steps=4)
    want = {}
    for world in (1, 2, 4, 8):
        seen = {}
        for rank in range(world):
            rs = bench.RequestSet(args, rank, world, 500)
            for k, gid in enumerate(rs.ids.tolist()):
                assert gid not in seen
                seen[gid] = (rs.prompt(k), rs.seed(k), int(rs.ctx[k]))
        assert sorted(seen) == list(range(96))
        if not want:
            want = seen
        assert seen == want
        loads = [sum(len(seen[g][0]) for g in bench.RequestSet(args, r, world, 500).ids.tolist())
                 for r in range(world)]
        assert max(loads) <= 1.25 * np.mean(loads) + 300  # LPT keeps the ranks balanced


def test_waves_cover_every_request_once_within_the_cache() -> None:
    import sys

    import numpy as np

    from .conftest import ROOT

    sys.path.insert(0, str(ROOT))
    import bench

    rng = np.random.default_rng(0)
    blocks = rng.integers(1, 40, 300)
    waves = bench.plan_waves(np.zeros(300), blocks, cap_blocks=500, max_batch=64)
    assert np.concatenate(waves).tolist() == list(range(300))
    for w in waves:
        assert blocks[w].sum() <= 500 and len(w) <= 64
