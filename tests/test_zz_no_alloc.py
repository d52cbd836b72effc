"""The allocation-free decoder matmul, rwq_matmul_t_q_noalloc (marked gpu).

It exists for callers that may not allocate GPU memory — a live-microphone
decode loop on a latency-critical thread, or an embedder whose GPU memory
belongs to another allocator.  This file is collected last so that a run
stopping at its first failure has already run every other test.  The
entry point is called through the C ABI and checked against
rwq_matmul_t_q_dev (the same kernels with library-owned scratch) with the
tolerance the other GPU tests use, on two calls in a row; it must not move
the device's free memory, and must reject sizes beyond its fixed scratch.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _close(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float((np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)).max())


def test_noalloc_matches_device_entry_point():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rusty_whisper_b200 import _lib, quant, synth
    quant.init(0)
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    m, k, n, dtype = 5, 1024, 777, 6
    w = quant.QTensor([n, k], dtype, synth.random_blocks(dtype, n, k, 91))
    bias = torch.from_numpy(synth.normal(92, n)).cuda()
    out = torch.empty((m, n), device="cuda")
    free_after = []
    for call in range(2):
        a = torch.from_numpy(synth.normal(93 + call, m * k).reshape(m, k)).cuda()
        ref = quant.matmul_t_q(a, w, bias=bias)
        rc = L.rwq_matmul_t_q_noalloc(ctypes.c_void_p(a.data_ptr()), m, k, w.handle,
                                      ctypes.c_void_p(bias.data_ptr()), ctypes.c_void_p(out.data_ptr()), stream)
        assert rc == _lib.RWQ_OK, L.rwq_last_error()
        torch.cuda.synchronize()
        assert _close(out.cpu().numpy(), ref.cpu().numpy()) < TOL
        free_after.append(torch.cuda.mem_get_info()[0])
    assert free_after[0] == free_after[1]

    # sizes beyond the fixed scratch are refused with a clear message
    big = torch.zeros((9, k), device="cuda")
    rc = L.rwq_matmul_t_q_noalloc(ctypes.c_void_p(big.data_ptr()), 9, k, w.handle, None,
                                  ctypes.c_void_p(out.data_ptr()), stream)
    assert rc == _lib.RWQ_ERR_ARG and b"0..8 rows" in L.rwq_last_error()
    wk = quant.QTensor([4, 8224], 8, synth.random_blocks(8, 4, 8224, 94))
    ak = torch.zeros((1, 8224), device="cuda")
    rc = L.rwq_matmul_t_q_noalloc(ctypes.c_void_p(ak.data_ptr()), 1, 8224, wk.handle, None,
                                  ctypes.c_void_p(out.data_ptr()), stream)
    assert rc == _lib.RWQ_ERR_ARG and b"up to 8192" in L.rwq_last_error()
