"""The multi-GPU host path on CPU: world_size-2 ``gloo`` ranks exercise the
request sharding, the max-over-ranks step time and the host-side gather that
bench.py uses around the (collective-free) draft step."""
import importlib
import os
import socket

import pytest
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    shard = importlib.import_module("mirror-sd_b200.shard")
    lens = [4096, 17, 2048, 2048, 900, 3000, 5, 64]
    mine = shard.shard_requests(lens, world, rank, block=16)
    t = shard.max_over_ranks(1.5 + rank)          # rank 1 is the slow one
    got = shard.gather_to_rank0({"rank": rank, "mine": mine, "acc": [rank * 10 + i for i in range(2)]})
    dist.barrier()
    dist.destroy_process_group()
    out.put((rank, mine, t, got))


def _run(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(res, key=lambda r: r[0])


def test_gloo_two_ranks_shard_time_gather(pkg):
    shard = importlib.import_module("mirror-sd_b200.shard")
    res = _run(2)
    lens = [4096, 17, 2048, 2048, 900, 3000, 5, 64]
    # every request on exactly one rank, and the plan is what a single process computes
    all_idx = sorted(i for _, mine, _, _ in res for i in mine)
    assert all_idx == list(range(len(lens)))
    for rank, mine, _, _ in res:
        assert mine == shard.shard_requests(lens, 2, rank, block=16)
    loads = [sum(lens[i] + 16 for i in mine) for _, mine, _, _ in res]
    assert max(loads) - min(loads) <= max(lens) + 16
    # the job's step time is the slowest rank's
    assert [t for _, _, t, _ in res] == [2.5, 2.5]
    # rank 0 holds every rank's stats in rank order; the others hold nothing
    assert res[0][3] == [{"rank": 0, "mine": res[0][1], "acc": [0, 1]},
                         {"rank": 1, "mine": res[1][1], "acc": [10, 11]}]
    assert res[1][3] is None


def test_single_process_fallbacks(pkg):
    shard = importlib.import_module("mirror-sd_b200.shard")
    assert shard.max_over_ranks(3.25) == 3.25
    assert shard.gather_to_rank0(7) == [7]
    assert shard.shard_requests([1, 2, 3], 1, 0) == [0, 1, 2]
    assert shard.job_throughput([31, 31], 2.0) == pytest.approx(31000.0)
    with pytest.raises(ValueError):
        shard.shard_requests([1], 2, 2)


def test_uniform_requests_split_evenly(pkg):
    shard = importlib.import_module("mirror-sd_b200.shard")
    for world in (2, 4, 8):
        parts = [shard.shard_requests([4096] * (world * 3), world, r, 32) for r in range(world)]
        assert all(len(p) == 3 for p in parts)
        assert sorted(i for p in parts for i in p) == list(range(world * 3))
