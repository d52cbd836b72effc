"""CPU-only checks of the C ABI library and the host logic (no GPU calls).

* librwq.so loads and exports every function include/rwq.h declares;
* argument validation answers with status codes before touching CUDA;
* the golden fixtures still match the oracle (regression of the checker);
* the seeded generators are deterministic and follow the stated ranges.
"""
import ctypes
import glob
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "rwq.h")).read()
    return sorted(set(re.findall(r"\b(rwq_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    from rusty_whisper_b200 import _lib
    L = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(L, s), s
    # and the ctypes table covers exactly the header
    assert sorted(_lib.SIGNATURES) == syms


def test_block_bytes_and_status_codes():
    from rusty_whisper_b200 import _lib
    L = _lib.lib()
    assert [L.rwq_block_bytes(t) for t in (2, 3, 6, 7, 8)] == [18, 20, 22, 24, 34]
    assert L.rwq_block_bytes(1) == _lib.RWQ_ERR_DTYPE
    assert b"unsupported" in L.rwq_last_error()
    h = ctypes.c_void_p()
    raw = (ctypes.c_uint8 * 34)()
    # bad dtype, k % 32, wrong raw length: rejected before any CUDA call
    assert L.rwq_qtensor_new(raw, 34, 5, 1, 32, ctypes.byref(h)) == _lib.RWQ_ERR_DTYPE
    assert L.rwq_qtensor_new(raw, 34, 8, 1, 33, ctypes.byref(h)) == _lib.RWQ_ERR_ARG
    assert L.rwq_qtensor_new(raw, 33, 8, 1, 32, ctypes.byref(h)) == _lib.RWQ_ERR_ARG
    assert L.rwq_matmul_t_q(None, 1, 32, None, None, None, 0) == _lib.RWQ_ERR_ARG
    assert L.rwq_set_gemm_path(7) == _lib.RWQ_ERR_ARG
    assert L.rwq_set_gemm_path(0) == _lib.RWQ_OK


def test_python_mirror_errors_without_gpu():
    from rusty_whisper_b200 import formats
    with pytest.raises(ValueError):
        formats.block_bytes(4)
    assert formats.row_bytes(formats.Q5_0, 768) == 24 * 22


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "*.npz"))))
def test_golden_fixture_matches_oracle(orc, path):
    fx = np.load(path)
    dtype, n, k = int(fx["dtype"]), int(fx["n"]), int(fx["k"])
    a, raw = fx["a"], fx["raw"]
    assert np.array_equal(orc.to_dense(dtype, raw, n, k).view(np.uint32), fx["dense"].view(np.uint32))
    q, d, s = orc.quantize_acts_i8(a)
    assert np.array_equal(q, fx["qa"]) and np.array_equal(d, fx["da"]) and np.array_equal(s, fx["sa"])
    assert np.array_equal(orc.block_dots(q, dtype, raw, n), fx["S"])
    assert np.array_equal(orc.int8_scalar_matmul(a, dtype, raw, n), fx["y_int8_scalar"])
    assert np.array_equal(orc.matmul_t_q(a, dtype, raw, n, tier=2), fx["y_avx2"])
    assert np.array_equal(orc.matmul_t_q(a, dtype, raw, n, tier=3), fx["y_f32"])
    if "y_vnni" in fx.files and orc.lib().orc_has_vnni():
        assert np.array_equal(orc.matmul_t_q(a, dtype, raw, n, tier=1), fx["y_vnni"])


def test_synth_deterministic_and_ranged(orc):
    from rusty_whisper_b200 import synth
    a = synth.normal(7, 10001)
    assert np.array_equal(a, synth.normal(7, 10001))
    assert abs(float(a.mean())) < 0.05 and abs(float(a.std()) - 1) < 0.05
    u = synth.uniform(3, 5000, 0.001, 0.02)
    assert u.min() >= 0.001 and u.max() < 0.02
    for dt in (2, 3, 6, 7, 8):
        raw = synth.random_blocks(dt, 16, 64, 5)
        bb = orc.block_bytes(dt)
        assert raw.size == 16 * 2 * bb
        dense = orc.to_dense(dt, raw, 16, 64)
        assert np.all(np.isfinite(dense))
        dh = raw.reshape(-1, bb)[:, :2].copy().view(np.uint16).ravel()
        dv = np.array([orc.f16_to_f32(int(h)) for h in dh])
        assert dv.min() >= 0.00099 and dv.max() <= 0.0201
    q8 = synth.random_blocks(8, 64, 64, 9).reshape(-1, 34)[:, 2:].view(np.int8)
    assert q8.min() >= -127 and q8.max() == 127
