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


def request_cost(n: int) -> float:
    """Device time of one request of n tokens, in microseconds, as measured for this engine on a
    B200 at hidden 768 (per-step kernels: 586 / 661 / 1190 us at 72 / 293 / 1024 tokens): a fixed
    part (125 dependent kernel launches) plus GEMM work linear in n and attention work in n^2."""
    return 550.0 + 0.3 * n + 0.0003 * n * n


def shard_lpt(lengths: list, world: int) -> list:
    """Greedy longest-processing-time partition of requests (by token count) over `world` ranks:
    requests in decreasing cost order, each to the rank with the least work so far (ties to the
    lower rank). Returns one list of request indices per rank, each in arrival order."""
    order = sorted(range(len(lengths)), key=lambda i: (-request_cost(lengths[i]), i))
    load = [0.0] * world
    parts = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        parts[r].append(i)
        load[r] += request_cost(lengths[i])
    return [sorted(p) for p in parts]


def serving_requests(count: int, seed: int, vocab: int, markers: int = 4, mean: float = 293.0,
                     sigma: float = 0.5, lo: int = 32, hi: int = 1024) -> list:
    """A seeded serving workload: `count` requests whose lengths are log-normal (sigma, with the
    mean `mean`: mu = ln(mean) - sigma^2 / 2), rounded and clipped to [lo, hi]; token ids uniform
    over the vocabulary; `markers` distinct marker positions in [0, n); question type 0. Returns
    a list of (ids uint32, markers uint32 sorted, qtype)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    mu = float(np.log(mean) - sigma * sigma / 2)
    lens = np.clip(np.rint(rng.lognormal(mu, sigma, count)), lo, hi).astype(np.int64)
    out = []
    for n in lens:
        ids = rng.integers(0, vocab, int(n)).astype(np.uint32)
        mk = np.sort(rng.choice(int(n), min(markers, int(n)), replace=False)).astype(np.uint32)
        out.append((ids, mk, 0))
    return out


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


def all_over_ranks(value: float, world: int, device="cpu") -> list:
    """`value` of every rank, in rank order (every rank gets the list)."""
    if world <= 1:
        return [float(value)]
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def job_rate(units_per_rank: float, slowest_seconds: float, world: int) -> float:
    """Whole-job throughput: units done by all ranks (each did units_per_rank) over the slowest
    rank's time."""
    return world * units_per_rank / slowest_seconds


def finalize(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()
