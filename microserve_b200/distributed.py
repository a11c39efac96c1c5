"""Multi-GPU plumbing: shard requests by id, reduce run statistics once at the end.

Requests are independent, so the engine scales by request: each rank (one
process per GPU, launched by torchrun) serves its own subset with a full
replica of the target and draft weights and its own caches.  There is no
collective in the decode loop.  The only exchange is the end-of-run
statistics reduce (SUM of token counters, MAX of elapsed time) over NCCL,
bounded by the process group's timeout.

The reference is single-process; this module has no counterpart there.
"""

from __future__ import annotations

import datetime
import heapq
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class RankInfo:
    rank: int
    world_size: int
    local_rank: int


def rank_info() -> RankInfo:
    return RankInfo(
        rank=int(os.environ.get("RANK", "0")),
        world_size=int(os.environ.get("WORLD_SIZE", "1")),
        local_rank=int(os.environ.get("LOCAL_RANK", "0")),
    )


def init(backend: str = "nccl", timeout_s: float = 120.0) -> RankInfo:
    """Initialise the default process group from torchrun's environment (world > 1)."""
    info = rank_info()
    if info.world_size > 1 and not dist.is_initialized():
        kwargs = {}
        if backend == "nccl":
            torch.cuda.set_device(info.local_rank)
            kwargs["device_id"] = torch.device("cuda", info.local_rank)
        dist.init_process_group(
            backend=backend,
            timeout=datetime.timedelta(seconds=timeout_s),
            **kwargs,
        )
    return info


def shard_requests(costs: list[float], world_size: int, rank: int) -> list[int]:
    """Deterministic longest-processing-time partition of request indices.

    ``costs[i]`` is request i's expected work (prompt + budget tokens).  Every
    rank computes the same partition and keeps its own part, sorted.
    """
    if world_size <= 1:
        return list(range(len(costs)))
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(world_size)]
    owner = [0] * len(costs)
    for i in order:
        load, r = heapq.heappop(heap)
        owner[i] = r
        heapq.heappush(heap, (load + costs[i], r))
    return [i for i in range(len(costs)) if owner[i] == rank]


def reduce_stats(counters: dict[str, int], elapsed_s: float, device: torch.device | None = None
                 ) -> tuple[dict[str, int], float]:
    """SUM the counters and MAX the elapsed time over all ranks (identity at world 1)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return dict(counters), elapsed_s
    keys = sorted(counters)
    dev = device or (torch.device("cuda", torch.cuda.current_device())
                     if dist.get_backend() == "nccl" else torch.device("cpu"))
    vals = torch.tensor([counters[k] for k in keys], dtype=torch.int64, device=dev)
    dist.all_reduce(vals, op=dist.ReduceOp.SUM)
    t = torch.tensor([elapsed_s], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return dict(zip(keys, vals.cpu().tolist(), strict=True)), float(t.item())


def barrier() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def shutdown() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
