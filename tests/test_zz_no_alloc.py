"""The allocation-free decoder matmul, rwq_matmul_t_q_noalloc (marked gpu).

It exists for callers that may not allocate GPU memory: a live-microphone
decode loop on a latency-critical thread (cudaMalloc/cudaFree can stall on
an implicit device synchronization), or an embedder whose GPU memory belongs
to another allocator.  This file is collected last, so a run that stops at
its first failure has already run every other test.

The entry point is called through the C ABI.  One warm-up call comes first:
the first call on a device looks up the scratch array's device address,
which may make the CUDA driver load the library's module on that device (a
driver-side allocation).  The two calls after it are each checked for:
  * unchanged free device memory around the call (synchronized readings);
  * the same bits as rwq_matmul_t_q_dev (the same quantizer and GEMV
    kernels with library-owned scratch);
  * the tolerance the other GPU tests use against the scalar int8 oracle.
The largest accepted shape (8 rows, k = 8192, which fills the whole fixed
array) is run the same way, and sizes beyond it must be refused.
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


def _run_case(L, _lib, quant, synth, orc, stream, m, k, n, dtype, seed):
    import torch
    raw = synth.random_blocks(dtype, n, k, seed)
    w = quant.QTensor([n, k], dtype, raw)
    bias_np = synth.normal(seed + 1, n)
    bias = torch.from_numpy(bias_np).cuda()
    out = torch.empty((m, n), device="cuda")

    def call(a):
        return L.rwq_matmul_t_q_noalloc(ctypes.c_void_p(a.data_ptr()), m, k, w.handle,
                                        ctypes.c_void_p(bias.data_ptr()), ctypes.c_void_p(out.data_ptr()), stream)

    warm = torch.from_numpy(synth.normal(seed + 2, m * k).reshape(m, k)).cuda()
    assert call(warm) == _lib.RWQ_OK, L.rwq_last_error()
    torch.cuda.synchronize()
    for c in range(2):
        a_np = synth.normal(seed + 3 + c, m * k).reshape(m, k)
        a = torch.from_numpy(a_np).cuda()
        ref_dev = quant.matmul_t_q(a, w, bias=bias)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        rc = call(a)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        assert rc == _lib.RWQ_OK, L.rwq_last_error()
        assert free0 == free1, (c, free0, free1)
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), ref_dev.cpu().numpy().view(np.uint32)), c
        ref = orc.int8_scalar_matmul(a_np, dtype, raw, n) + bias_np[None, :]
        assert _close(got, ref) < TOL, c
    return w, out


def test_noalloc_matches_device_entry_point_and_oracle(orc):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rusty_whisper_b200 import _lib, quant, synth
    quant.init(0)
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    w, out = _run_case(L, _lib, quant, synth, orc, stream, 5, 1024, 777, 6, 91)
    _run_case(L, _lib, quant, synth, orc, stream, 8, 8192, 300, 8, 191)   # the whole fixed array

    # sizes beyond the fixed scratch are refused with a clear message
    k = 1024
    big = torch.zeros((9, k), device="cuda")
    rc = L.rwq_matmul_t_q_noalloc(ctypes.c_void_p(big.data_ptr()), 9, k, w.handle, None,
                                  ctypes.c_void_p(out.data_ptr()), stream)
    assert rc == _lib.RWQ_ERR_ARG and b"0..8 rows" in L.rwq_last_error()
    wk = quant.QTensor([4, 8224], 8, synth.random_blocks(8, 4, 8224, 94))
    ak = torch.zeros((1, 8224), device="cuda")
    rc = L.rwq_matmul_t_q_noalloc(ctypes.c_void_p(ak.data_ptr()), 1, 8224, wk.handle, None,
                                  ctypes.c_void_p(out.data_ptr()), stream)
    assert rc == _lib.RWQ_ERR_ARG and b"up to 8192" in L.rwq_last_error()
