"""Host logic of the multi-GPU (replicas) path on CPU: stream placement and
the max-over-ranks job time, exercised with world_size-2 gloo process
groups."""
import os
import socket

import pytest

from conftest import load_package

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_assign_streams_balances_cost():
    sh = load_package().sharding
    costs = [sh.stream_cost(p, 256, cfg=True) for p in (100, 400, 250, 380, 120, 300, 200, 150)]
    owned = sh.assign_streams(costs, 2)
    assert sorted(i for o in owned for i in o) == list(range(8))
    loads = [sum(costs[i] for i in o) for o in owned]
    assert max(loads) / min(loads) < 1.2
    # one stream per rank when there are as many ranks as streams
    assert sorted(len(o) for o in sh.assign_streams(costs, 8)) == [1] * 8


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sh = load_package().sharding
    costs = [sh.stream_cost(100 + 37 * i, 256) for i in range(10)]
    mine = sh.assign_streams(costs, world)[rank]
    # every rank computes the same placement without communication
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    # rank r "ran" for 10 + r ms on its streams
    value, ms = sh.job_throughput(dist, 10.0 + rank, len(mine) * 256, world)
    q.put((rank, gathered, value, ms))
    dist.destroy_process_group()


def test_two_rank_placement_and_job_time():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    owned = res[0][1]
    assert res[1][1] == owned                          # identical placement on both ranks
    assert sorted(i for o in owned for i in o) == list(range(10))
    assert all(len(o) > 0 for o in owned)
    for _, _, value, ms in res:
        assert ms == 11.0                              # max over ranks
        assert abs(value - 10 * 256 / 0.011) < 1e-6    # all units / slowest rank
