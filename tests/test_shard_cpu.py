"""Multi-process window sharding on CPU (gloo ranks standing in for GPUs).

Each rank runs its windows through the CPU oracle (standing in for a GPU
replica) and reports through the process group's store; rank 0 assembles
the results in window order, which must equal the single-process result.
Failures are made on the host: a rank whose share raises, and a rank that
exits without reporting; their windows are re-run on the survivors.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from rusty_whisper_b200.shard import merge_in_order, window_range

N_WIN = 11


def test_window_range_balanced():
    for n in (0, 1, 7, 256):
        for world in (1, 2, 4, 8):
            parts = [window_range(n, world, r) for r in range(world)]
            assert sum(len(p) for p in parts) == n
            assert [i for p in parts for i in p] == list(range(n))
            assert max(map(len, parts)) - min(map(len, parts)) <= 1
    with pytest.raises(ValueError):
        window_range(4, 2, 2)
    with pytest.raises(RuntimeError):
        merge_in_order([[1], [2]], 3)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _one_window(seed):
    import oracle
    from rusty_whisper_b200 import synth
    a = synth.normal(seed, 3 * 64).reshape(3, 64)
    raw = synth.random_blocks(7, 16, 64, 5)
    return oracle.matmul_t_q(a, 7, raw, 16, tier=2, threads=1)


def _worker(rank, world, port, out_path, mode):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from rusty_whisper_b200.shard import run_sharded

    def fn(batch):
        if (mode == "raise" and rank == 1) or mode == "all_raise":
            raise RuntimeError(f"injected failure on rank {rank}")
        if mode == "die" and rank == world - 1:
            os._exit(0)     # leaves without reporting, between steps
        return [_one_window(w) for w in batch]

    try:
        res = run_sharded(list(range(N_WIN)), fn, timeout_s=5.0)
        if rank == 0:
            np.save(out_path, np.stack(res))
    except RuntimeError as e:
        if rank == 0:
            with open(out_path + ".err", "w") as f:
                f.write(str(e))
    finally:
        if mode != "die":
            dist.destroy_process_group()


def _run(world, mode, tmp_path):
    out = str(tmp_path / "res.npy")
    mp.start_processes(_worker, args=(world, _free_port(), out, mode), nprocs=world, join=True, start_method="spawn")
    return out


def _serial():
    return np.stack([_one_window(i) for i in range(N_WIN)])


def test_two_rank_gather_matches_serial(tmp_path):
    out = _run(2, "ok", tmp_path)
    assert np.array_equal(np.load(out), _serial())


def test_failed_rank_windows_requeued(tmp_path):
    """Rank 1's share raises: ranks 0 and 2 re-run its windows and rank 0
    still returns every window's result, in order."""
    out = _run(3, "raise", tmp_path)
    assert np.array_equal(np.load(out), _serial())


def test_dead_rank_windows_requeued(tmp_path):
    """The last rank exits without reporting: after the timeout the
    survivors re-run its windows (no collective waits on it)."""
    out = _run(3, "die", tmp_path)
    assert np.array_equal(np.load(out), _serial())


def test_every_rank_failing_is_an_error(tmp_path):
    """No rank succeeds: rank 0 raises (listing the windows and the ranks'
    errors) instead of hanging or returning a partial result."""
    out = _run(2, "all_raise", tmp_path)
    assert not os.path.exists(out)
    msg = open(out + ".err").read()
    assert "have no result" in msg and "injected failure" in msg
