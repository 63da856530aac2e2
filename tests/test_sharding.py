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


# ---- per-page results through the host-side gather ---------------------------
PAGES, H, W = 6, 192, 256


def _page_records(first, n):
    """The oracle's DB boxes of pages first..first+n-1 (small synthetic pages)."""
    from oracle import db_oracle as do
    from oracle import synth_host as sh
    out = []
    for p in range(first, first + n):
        prob = sh.ink_map(sh.make_page(H, W, 0x7EC00005, p))
        out.append([b for b, _ in do.db_postprocess(prob)])
    return out


def _gather_worker(rank, world, port, mode, q):
    import datetime
    import time
    from turboocr_b200.sharding import RankFailure, run_sharded
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))

    def work(first, n):
        if mode == "raise" and rank == 1:
            raise ValueError("injected failure on rank 1")
        if mode == "stall" and rank == 1:
            time.sleep(20)   # never reaches the gather within the group timeout
        return _page_records(first, n)

    try:
        res = run_sharded(PAGES, work, micro_batch=1)
        q.put((rank, "ok", res))
    except RankFailure as e:
        q.put((rank, "failure", (e.errors, e.results)))
    if mode != "stall":
        dist.destroy_process_group()


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world if mode != "stall" else 1):
        r, kind, payload = q.get(timeout=180)
        out[r] = (kind, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_gather_matches_single_rank_run():
    single = _page_records(0, PAGES)
    assert sum(len(b) for b in single) > 10
    out = _run(2, "ok")
    for r in (0, 1):
        kind, res = out[r]
        assert kind == "ok" and res == single


def test_failing_rank_is_reported_while_the_other_finishes():
    single = _page_records(0, PAGES)
    out = _run(2, "raise")
    for r in (0, 1):
        kind, (errors, results) = out[r]
        assert kind == "failure" and list(errors) == [1]
        assert "injected failure on rank 1" in errors[1]
        assert results[:3] == single[:3] and results[3:] == [None] * 3   # rank 0's shard done


def test_stalled_rank_is_reported_by_the_timeout():
    out = _run(2, "stall")
    kind, (errors, results) = out[0]
    assert kind == "failure" and -1 in errors and "did not report" in errors[-1]
    assert results[:3] == _page_records(0, 3)
