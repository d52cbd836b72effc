"""Window sharding across GPUs (one process per GPU).

Independent 30 s windows are the unit of parallelism (the reference's
``transcribe_parallel`` splits audio into chunks processed by worker
threads and ``merge_parallel_results`` concatenates them in order,
transcribe.rs:1528-1586).  Here each rank owns a contiguous range of
windows, holds a full weight replica and computes with no collective on
the data path; results are gathered on the host of rank 0 in window order.
"""
from __future__ import annotations

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


def run_sharded(windows: Sequence, fn: Callable, group=None) -> List | None:
    """Apply ``fn`` to this rank's windows; rank 0 returns every result in
    window order, other ranks return None.  Without an initialised
    process group this runs everything locally."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return [fn(w) for w in windows]
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    mine = [fn(windows[i]) for i in window_range(len(windows), world, rank)]
    gathered = [None] * world if rank == 0 else None
    dist.gather_object(mine, gathered, dst=0, group=group)
    if rank != 0:
        return None
    return merge_in_order(gathered, len(windows))
