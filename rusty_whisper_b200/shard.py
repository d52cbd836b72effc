"""Window sharding across GPUs (one process per GPU).

Independent 30 s windows are the unit of parallelism (the reference's
``transcribe_parallel`` splits audio into chunks processed by worker
threads and ``merge_parallel_results`` concatenates them in order,
transcribe.rs:1528-1586).  Here each rank owns a contiguous range of
windows, holds a full weight replica and computes with no collective on
the data path; every rank reports its results through the process
group's key-value store and rank 0 assembles them in window order.

Failure handling (the reference has none: a failed worker thread panics
the whole call at ``join().unwrap()``): a rank whose share raises, or that
has not reported within ``timeout_s`` (a rank that died), is treated as
failed; its windows are split again over the ranks that succeeded, which
run them and report once more.  Rank 0 gathers, so rank 0 itself must stay
up.  No collective runs after the first report, so a dead peer cannot
block the survivors.
"""
from __future__ import annotations

import datetime
import pickle
from typing import Callable, List, Sequence


def window_range(n_windows: int, world: int, rank: int) -> range:
    """Contiguous, balanced share of ``n_windows`` for ``rank`` (sizes
    differ by at most one; earlier ranks take the extra windows)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of world {world}")
    if n_windows < 0:
        raise ValueError("n_windows must be >= 0")
    base, extra = divmod(n_windows, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def merge_in_order(per_rank: Sequence[Sequence], n_windows: int) -> list:
    """Concatenate per-rank results (rank order == window order)."""
    out = [x for part in per_rank for x in part]
    if len(out) != n_windows:
        raise RuntimeError(f"gathered {len(out)} results for {n_windows} windows")
    return out


_CALLS = [0]


def _run(fn: Callable, items: list, index: list):
    """fn over a list of windows -> ("ok", index, results) or ("err", ...)."""
    if not index:
        return ("ok", [], [])
    try:
        res = list(fn(items))
        if len(res) != len(index):
            raise RuntimeError(f"{len(res)} results for {len(index)} windows")
        return ("ok", index, res)
    except Exception as e:   # reported to the other ranks, whose survivors re-run the windows
        return ("err", index, repr(e))


def _read(store, key: str, timeout_s: float):
    try:
        store.wait([key], datetime.timedelta(seconds=timeout_s))
        return pickle.loads(store.get(key))
    except Exception:
        return None


def run_sharded(windows: Sequence, fn: Callable, group=None, store=None, timeout_s: float = 600.0,
                requeue: bool = True) -> List | None:
    """Run ``fn`` on this rank's windows: ``fn(list_of_windows)`` returns one
    result per window.  Rank 0 returns every result in window order, other
    ranks return None.  Without an initialised process group everything
    runs locally.  Windows of a rank that fails or does not report within
    ``timeout_s`` are re-run on the ranks that succeeded (``requeue``);
    a window that still has no result raises RuntimeError on rank 0."""
    import torch.distributed as dist
    windows = list(windows)
    n = len(windows)
    if not (dist.is_available() and dist.is_initialized()):
        return list(fn(windows)) if n else []
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if store is None:
        store = dist.distributed_c10d._get_default_store()
    _CALLS[0] += 1
    tag = f"rwq_shard/{_CALLS[0]}"

    mine = list(window_range(n, world, rank))
    store.set(f"{tag}/r{rank}", pickle.dumps(_run(fn, [windows[i] for i in mine], mine)))
    reports = {}
    for r in range(world):
        rep = _read(store, f"{tag}/r{r}", timeout_s)
        reports[r] = rep if rep is not None else ("lost", list(window_range(n, world, r)), None)
    ok = [r for r in range(world) if reports[r][0] == "ok"]
    missing = sorted(i for r in range(world) if reports[r][0] != "ok" for i in reports[r][1])
    retry = {}
    if missing and requeue and ok:
        if rank in ok:
            share = [missing[i] for i in window_range(len(missing), len(ok), ok.index(rank))]
            store.set(f"{tag}/retry/r{rank}", pickle.dumps(_run(fn, [windows[i] for i in share], share)))
        if rank == 0:
            for r in ok:
                rep = _read(store, f"{tag}/retry/r{r}", timeout_s)
                if rep is not None and rep[0] == "ok":
                    retry[r] = rep
    if rank != 0:
        return None
    out = [None] * n
    have = [False] * n
    for rep in list(reports.values()) + list(retry.values()):
        if rep[0] == "ok":
            for i, v in zip(rep[1], rep[2]):
                out[i] = v
                have[i] = True
    if not all(have):
        lost = [r for r in range(world) if reports[r][0] != "ok"]
        raise RuntimeError(f"windows {[i for i in range(n) if not have[i]]} have no result "
                           f"(ranks {lost} failed: {[reports[r][2] for r in lost]})")
    return out
