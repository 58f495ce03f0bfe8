"""Replicas over the GPUs of one box.

A julia-cuda request does not shard (one sequence runs through the whole encoder on one GPU; the
reference serves one engine on GPU 0, src/engine.rs), so N GPUs serve N independent request
streams: one process and one engine per GPU, requests partitioned across the ranks, and no
collective on the data path. The process group carries only what a measurement or a serving
front-end needs across ranks: barriers and the maximum over ranks of a timed region, so the
whole-job rate is (units done on all ranks) / (slowest rank's time).

The functions take `world` explicitly and do nothing collective when it is 1, so the single-GPU
path never touches torch.distributed.
"""
from __future__ import annotations

import os
from datetime import timedelta


def rank_env() -> tuple[int, int, int]:
    """(rank, world size, local rank) from the launcher's environment (torchrun sets them)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(world: int, backend: str, device=None, timeout_s: float = 120.0) -> bool:
    """Joins the process group when world > 1 (rendezvous on 127.0.0.1 unless MASTER_ADDR says
    otherwise; a short timeout so ranks waiting on a missing one end with an error). `device` (a
    torch.device) binds an NCCL group to this rank's GPU. Returns whether a group was created."""
    if world <= 1:
        return False
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kw = {"device_id": device} if device is not None else {}
    dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s), **kw)
    return True


def shard(items: list, rank: int, world: int) -> list:
    """This rank's share of a request list: every world-th item from position rank, so every
    request is served by exactly one rank and the ranks' shares differ by at most one."""
    return items[rank::world]


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value: float, world: int, device="cpu") -> float:
    """The maximum of `value` over all ranks (every rank gets it)."""
    if world <= 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_rate(units_per_rank: float, slowest_seconds: float, world: int) -> float:
    """Whole-job throughput: units done by all ranks (each did units_per_rank) over the slowest
    rank's time."""
    return world * units_per_rank / slowest_seconds


def finalize(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()
