"""The N > 1 host path (replicas: one engine per GPU, requests partitioned, the slowest rank's time
sets the whole-job rate) on CPU: two `gloo` ranks in child processes, rendezvous on 127.0.0.1.
No GPU is involved; the GPU run (bench.py under torchrun) uses the same functions over NCCL."""
import importlib
import json
import os
import socket
import sys

import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, fail_rank):
    sys.path.insert(0, ROOT)
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    rep = importlib.import_module("julia-cuda_b200.replicas")
    r, w, local = rep.rank_env()
    res = {"rank_env": [r, w, local]}
    try:
        res["joined"] = rep.init(w, "gloo", timeout_s=10.0)
        if rank == fail_rank:
            # This rank leaves between steps without taking part in the next collective.
            raise SystemExit(0)
        requests = list(range(7))
        res["share"] = rep.shard(requests, r, w)
        # Rank r pretends its timed region took r + 1 seconds for 5 requests.
        slowest = rep.max_over_ranks(r + 1.0, w)
        res["slowest"] = slowest
        res["rate"] = rep.job_rate(5, slowest, w)
        res["all"] = rep.all_over_ranks(10.0 * r + 0.5, w)
        rep.barrier(w)
        res["ok"] = True
    except RuntimeError as e:
        res["error"] = str(e)[:200]
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(res, f)
        rep.finalize(w)


def run_ranks(tmp_path, world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, str(tmp_path), fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        assert not p.is_alive(), "a rank did not finish"
    return [json.load(open(tmp_path / f"rank{r}.json")) for r in range(world)]


def test_two_gloo_ranks_partition_requests_and_agree_on_the_slowest_time(tmp_path):
    res = run_ranks(tmp_path, 2)
    for r, x in enumerate(res):
        assert x["rank_env"] == [r, 2, r] and x["joined"] and x.get("ok"), x
        assert x["slowest"] == 2.0          # max over ranks, the same on every rank
        assert x["rate"] == 2 * 5 / 2.0     # all ranks' requests over the slowest time
        assert x["all"] == [0.5, 10.5]      # every rank's value, in rank order
    # every request is served by exactly one rank
    assert sorted(res[0]["share"] + res[1]["share"]) == list(range(7))
    assert not set(res[0]["share"]) & set(res[1]["share"])


def test_a_rank_that_leaves_ends_the_others_collective_with_an_error(tmp_path):
    """Failure detection on the host: rank 1 leaves before the max-reduction; rank 0's collective
    ends with an error (gloo sees the peer gone, or the short group timeout) instead of waiting
    for good."""
    res = run_ranks(tmp_path, 2, fail_rank=1)
    assert "error" in res[0] and not res[0].get("ok"), res[0]


def test_single_process_needs_no_process_group():
    rep = importlib.import_module("julia-cuda_b200.replicas")
    assert rep.init(1, "gloo") is False
    assert rep.max_over_ranks(3.5, 1) == 3.5
    assert rep.all_over_ranks(3.5, 1) == [3.5]
    assert rep.shard([1, 2, 3], 0, 1) == [1, 2, 3]
    assert rep.job_rate(10, 2.0, 1) == 5.0


def test_reference_arm_runs_on_rank_zero_only(capsys):
    """Under torchrun the reference arm (CPU) is run and printed by rank 0 alone."""
    sys.path.insert(0, ROOT)
    bench = importlib.import_module("bench")

    class Args:
        steps, warmup, seq, head_length = 1, 0, 293, 0
    bench.reference_arm(Args, 1, 2)
    assert capsys.readouterr().out == ""


def test_lpt_partition_balances_request_costs():
    rep = importlib.import_module("julia-cuda_b200.replicas")
    import random
    rng = random.Random(0)
    lengths = [max(32, min(1024, int(rng.lognormvariate(5.55, 0.5)))) for _ in range(500)]
    for world in (1, 2, 4, 8):
        parts = rep.shard_lpt(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(len(lengths)))
        loads = [sum(rep.request_cost(lengths[i]) for i in p) for p in parts]
        # LPT: no rank exceeds the mean by more than the largest single request
        assert max(loads) - sum(loads) / world <= max(rep.request_cost(n) for n in lengths)
    assert rep.shard_lpt([10, 300, 20], 2) == [[1], [0, 2]]
