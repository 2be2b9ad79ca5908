"""World-size-2 gloo run of the multi-GPU harness's host logic on CPU: every rank derives
the same seeded agent lengths, takes its LPT share, the shares are disjoint and cover all
agents, and the step time reported is the max over ranks (no collective on the data
path, only this timing reduction).  Under weak scaling the job is 256 agents per rank;
under strong scaling 256 agents in total."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, scaling):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    from __graft_entry__ import load_package

    am = load_package()
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import argparse

        job = bench.job_agents(argparse.Namespace(agents=256, scaling=scaling), world)
        lens = bench.agent_lengths(job, 1024, 32768, 0)
        mine = sorted(am.lpt_partition(lens, world)[rank])
        got = [None] * world
        dist.all_gather_object(got, mine)
        t = torch.tensor([float(10 + rank)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, got, float(t.item()), sum(lens[i] for i in mine)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("scaling,job", [("weak", 512), ("strong", 256)])
def test_two_rank_partition_and_max_timing(scaling, job):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, scaling)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    shares = res[0][1]
    assert res[1][1] == shares
    flat = sorted(i for s in shares for i in s)
    assert flat == list(range(job)) and not set(shares[0]) & set(shares[1])
    assert res[0][2] == res[1][2] == 11.0
    loads = [r[3] for r in res]
    assert max(loads) / min(loads) < 1.01
