"""Data-parallel runs over ranks (one process per GPU): contiguous page
shards, no collective on the data path, and the host-side gather of the
per-page results in page order. Pages are independent, so the only
cross-rank traffic is this gather of small per-page records (quads, scores,
tokens: ~KB per page) and the timing reduction of the benchmark.

A rank whose work raises reports its error through the same gather, so the
other ranks still finish their shards and every rank raises the same
RankFailure afterwards; a rank that never reaches the gather is reported
when the process group's timeout ends the others' wait."""
from __future__ import annotations

from typing import Any, Callable, Sequence

import torch.distributed as dist

from .pipeline import shard


class RankFailure(RuntimeError):
    """Raised on every rank when one or more ranks failed; .errors maps rank
    -> message, .results holds the page-ordered records of the ranks that
    finished (None for the pages of failed ranks)."""

    def __init__(self, errors: dict[int, str], results: list[Any]):
        super().__init__("; ".join(f"rank {r}: {m}" for r, m in sorted(errors.items())))
        self.errors = errors
        self.results = results


def run_sharded(total_pages: int, work: Callable[[int, int], Sequence[Any]],
                micro_batch: int = 32, group=None) -> list[Any]:
    """Runs work(first_page, n_pages) on this rank's shard and gathers every
    rank's per-page records, concatenated in page order (the same list on
    every rank). work must return exactly n_pages records."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    first, n = shard(total_pages, world, rank, micro_batch)
    try:
        recs = list(work(first, n))
        if len(recs) != n:
            raise ValueError(f"work returned {len(recs)} records for {n} pages")
        status: tuple = ("ok", recs)
    except Exception as e:  # reported to every rank, raised after the gather
        status = ("error", f"{type(e).__name__}: {e}")
    if world == 1:
        gathered = [(rank, first, n, status)]
    else:
        gathered = [None] * world
        try:
            dist.all_gather_object(gathered, (rank, first, n, status), group=group)
        except Exception as e:  # a rank that never arrived: the group timed out
            mine = [None] * total_pages
            if status[0] == "ok":
                mine[first:first + n] = status[1]
            raise RankFailure({-1: f"gather failed (a rank did not report): {e}"}, mine) from e
    results: list[Any] = [None] * total_pages
    errors: dict[int, str] = {}
    for r, f, cnt, (kind, payload) in gathered:
        if kind == "ok":
            results[f:f + cnt] = payload
        else:
            errors[r] = payload
    if errors:
        raise RankFailure(errors, results)
    return results
