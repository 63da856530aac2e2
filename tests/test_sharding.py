"""Multi-rank host logic of the end-to-end run on CPU (gloo, world size 2 and
4): the page shards of all ranks are disjoint and cover the job exactly, a
rank's work needs no data from another rank, and the step time a rank
reports is the maximum over ranks (what bench.py prints)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from turboocr_b200.pipeline import shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, total, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    first, n = shard(total, world, rank)
    got = [None] * world
    dist.all_gather_object(got, (first, n))
    t = torch.tensor([10.0 + rank], dtype=torch.float64)   # this rank's step time
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        q.put((got, float(t)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,total", [(2, 4096), (4, 4096), (2, 100)])
def test_shards_cover_job(world, total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    got, tmax = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    covered = []
    for first, n in got:
        covered.extend(range(first, first + n))
    assert covered == list(range(total))
    assert tmax == 10.0 + world - 1


def test_shard_micro_batch_rounding():
    assert shard(4096, 8, 7) == (3584, 512)
    assert shard(4096, 3, 2) == (2752, 1344)
    assert shard(10, 4, 3) == (10, 0)
