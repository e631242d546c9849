"""The N > 1 bench path on CPU: two gloo ranks (127.0.0.1) run the bench's sharding
and timing helpers -- disjoint utterance blocks covering 0 .. 2*per_rank, and every
rank seeing the slowest rank's step time -- and a rank that raises ends the job
with an error instead of a hang (short process-group timeout)."""

import datetime
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, fail_rank):
    sys.path.insert(0, REPO)
    import torch.distributed as dist
    import bench
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        if rank == fail_rank:
            raise RuntimeError("rank failed before its first collective")
        seeds = list(bench.rank_seeds(rank))
        step_ms = 100.0 + 37.0 * rank                      # rank-dependent step time
        worst = bench.max_over_ranks(step_ms, world, device="cpu")
        q.put((rank, seeds, worst))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    return sorted(out, key=lambda t: t[0])


def test_two_ranks_shard_utterances_and_agree_on_the_slowest_time():
    import bench
    out = _run(2)
    assert [o[0] for o in out] == [0, 1]
    s0, s1 = out[0][1], out[1][1]
    assert len(s0) == len(s1) == bench.UTTS and not set(s0) & set(s1)
    assert sorted(s0 + s1) == list(range(2 * bench.UTTS))
    assert out[0][2] == out[1][2] == 137.0


def test_a_failing_rank_ends_the_job_with_an_error():
    out = _run(2, fail_rank=1)
    assert out[1][1] == "error"
    assert out[0][1] == "error"   # rank 0's collective fails (peer gone / timeout), no hang
