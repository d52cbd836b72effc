"""Multi-process window sharding on CPU (gloo, world size 2).

Each rank quantizes and multiplies its own windows with the CPU oracle
(standing in for a GPU replica), and rank 0 gathers results in window
order; the result must equal the single-process computation.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from rusty_whisper_b200.shard import merge_in_order, window_range


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


def _window_fn(seed):
    import oracle
    from rusty_whisper_b200 import synth
    a = synth.normal(seed, 3 * 64).reshape(3, 64)
    raw = synth.random_blocks(7, 16, 64, 5)
    return oracle.matmul_t_q(a, 7, raw, 16, tier=2, threads=1)


def _worker(rank, world, port, out_path, fail_rank):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from rusty_whisper_b200.shard import run_sharded
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure")
        res = run_sharded(list(range(11)), _window_fn)
        if rank == 0:
            np.save(out_path, np.stack(res))
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_matches_serial(tmp_path):
    out = str(tmp_path / "res.npy")
    mp.start_processes(_worker, args=(2, _free_port(), out, -1), nprocs=2, join=True, start_method="spawn")
    got = np.load(out)
    ref = np.stack([_window_fn(i) for i in range(11)])
    assert np.array_equal(got, ref)


def test_rank_failure_surfaces_as_error(tmp_path):
    """A rank that raises before the gather: the job ends with an error
    (the other rank's gather times out or sees the peer gone), no hang."""
    out = str(tmp_path / "res.npy")
    with pytest.raises(Exception):
        mp.start_processes(_worker, args=(2, _free_port(), out, 1), nprocs=2, join=True, start_method="spawn")
    assert not os.path.exists(out)
