"""The multi-rank logic of bench.py and the host side of the path, on two gloo ranks (CPU).

On the GPU box the same code runs one process per GPU over NCCL; the request-parallel
path has no data-path collective, so what needs checking across ranks is the partition
of the work, the reductions that turn per-rank numbers into job numbers (max of times,
sum of work), and that every rank's host bookkeeping stands alone.
"""

from __future__ import annotations

import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "hayate-exp_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        from hayate_b200 import PagedKVCacheManager

        result = {}
        # job time = the slowest rank, job work = the sum over ranks
        result["max"] = bench.max_over_ranks(1.5 + rank, world)
        result["sum"] = bench.sum_over_ranks(10.0 * (rank + 1), world)
        # per-rank output checksums gathered in rank order
        result["gather"] = bench.gather_over_ranks(100.0 + rank, world)
        # config 5: whole prefix groups per rank
        groups = bench.long_groups(rank, world)
        result["groups"] = groups
        # each rank's own pool: a group's requests alias the group's prefix pages
        manager = PagedKVCacheManager(1, 1, 4, 64 * 128, 128, 1 + 4 * len(groups), torch.float32, "cpu")
        refs = []
        for _ in groups:
            prefix = manager.allocate()
            manager.reserve(prefix, 256)
            prefix.length = 256
            reqs = [manager.share(prefix, 256) for _ in range(3)]
            refs.append(manager.page_refcount(prefix.pages[0]))
            batch = manager.begin_batch(reqs, 1)   # appends land in private pages
            manager.commit_batch(reqs, 1)
            refs.append(int(batch.page_table.shape[1]))
            for h in reqs + [prefix]:
                manager.release(h)
        result["refs"] = refs
        result["free"] = len(manager._free_pages) == manager.num_pages
        # the same seeds give every rank its own requests
        result["lengths"] = bench.decode_lengths(1000 + rank)[:4]
        dist.barrier()
        out[rank] = result
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_two_gloo_ranks(world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        mp.start_processes(_worker, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
        res = dict(out)
    assert sorted(res) == list(range(world))
    for r in range(world):
        assert res[r]["max"] == 1.5 + world - 1
        assert res[r]["sum"] == sum(10.0 * (k + 1) for k in range(world))
        assert res[r]["gather"] == [100.0 + k for k in range(world)]
        assert res[r]["free"]
        assert all(x == 4 for x in res[r]["refs"][0::2])   # prefix page held by 1 + 3 requests
        assert all(x == 3 for x in res[r]["refs"][1::2])   # 2 prefix pages + 1 private page
    covered = sorted(g for r in range(world) for g in res[r]["groups"])
    import bench  # noqa: E402  (ROOT is on sys.path via conftest)
    assert covered == list(range(bench.LONG_GROUPS))
    assert res[0]["lengths"] != res[1]["lengths"]
