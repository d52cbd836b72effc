"""GPU parity of the B200 kernels against the CPU oracle (marked gpu).

Bars (rusty_whisper's own rules, quant.rs:1125-1160, 1336-1384):
  * dequant: bit-identical to the reference's scalar dequant;
  * activation quantizer: bit-identical q, d, sum(q);
  * per-block integer dots S[i,j,kb]: bit-identical, both kernel families;
  * int8-path f32 outputs: |y - ref| <= 1e-3 * max(|ref|, 1) against the
    scalar int8 oracle and the reference tier that runs on this host;
  * dequant-then-f32 outputs: same rule against the oracle's f32 tier;
  * batch invariance: a row's result does not depend on M.
"""
import glob
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FORMATS = (2, 3, 6, 7, 8)
TOL = 1e-3  # quant.rs:1365


@pytest.fixture(scope="module")
def rq():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rusty_whisper_b200 import quant
    quant.init(0)
    return quant


def close(got, ref, tol=TOL):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)
    return float(err.max()) if err.size else 0.0


def cuda(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "*.npz"))))
def test_golden_fixture_on_gpu(rq, path):
    fx = np.load(path)
    dtype, m, n, k = int(fx["dtype"]), int(fx["m"]), int(fx["n"]), int(fx["k"])
    w = rq.QTensor([n, k], dtype, fx["raw"])
    a = cuda(fx["a"])
    assert np.array_equal(host(w.to_dense()).view(np.uint32), fx["dense"].view(np.uint32))
    q, d, s = rq.quantize_acts_i8(a)
    assert np.array_equal(host(q), fx["qa"])
    assert np.array_equal(host(d).view(np.uint32), fx["da"].view(np.uint32))
    assert np.array_equal(host(s), fx["sa"])
    assert np.array_equal(host(rq.block_dots(a, w, path=0)), fx["S"])
    y = host(rq.matmul_t_q(a, w))
    assert close(y, fx["y_int8_scalar"]) < TOL
    assert close(y, fx["y_avx2"]) < TOL
    if "y_vnni" in fx.files:
        assert close(y, fx["y_vnni"]) < TOL
    yf = host(rq.matmul_t_q(a, w, mode="f32"))
    assert close(yf, fx["y_f32"]) < TOL


def exact_int8(orc, a, dtype, raw, n):
    """The reference's int8 formula sum_kb d_a*(d_b*S + m_b*sum(q_a))
    (quant.rs:349-354, 452-454) evaluated in float64: the activations are
    quantized by the oracle (bit-exact), the weights dequantized by it
    (bit-exact f32 x = d*q + m), then one f64 product."""
    m, k = a.shape
    qa, da, _ = orc.quantize_acts_i8(a)
    deq = qa.astype(np.float64).reshape(m, k // 32, 32) * da.astype(np.float64).reshape(m, k // 32, 1)
    x = orc.to_dense(dtype, raw, n, k).astype(np.float64)
    return deq.reshape(m, k) @ x.T


def _case(dtype, m, k, n, seed):
    from rusty_whisper_b200 import synth
    a = synth.normal(seed, m * k).reshape(m, k)
    raw = synth.random_blocks(dtype, n, k, seed + 1)
    return a, raw


@pytest.mark.parametrize("dtype", FORMATS)
@pytest.mark.parametrize("m,k,n", [(129, 96, 41), (200, 256, 130), (300, 768, 257)])
def test_gemm_tensor_core_block_dots_bit_exact(rq, orc, dtype, m, k, n):
    a, raw = _case(dtype, m, k, n, 7 * dtype + m)
    w = rq.QTensor([n, k], dtype, raw)
    qa, _, _ = orc.quantize_acts_i8(a)
    S_ref = orc.block_dots(qa, dtype, raw, n)
    S_tc = host(rq.block_dots(cuda(a), w, path=1))
    assert np.array_equal(S_tc, S_ref)
    S_cc = host(rq.block_dots(cuda(a), w, path=0))
    assert np.array_equal(S_cc, S_ref)


@pytest.mark.parametrize("dtype", FORMATS)
@pytest.mark.parametrize("m,k,n", [(1, 768, 768), (5, 768, 3072), (8, 3072, 768), (9, 128, 200),
                                   (37, 96, 41), (1500, 384, 1536), (333, 1024, 520)])
def test_matmul_int8_matches_oracle(rq, orc, dtype, m, k, n):
    a, raw = _case(dtype, m, k, n, 11 * dtype + m + k)
    w = rq.QTensor([n, k], dtype, raw)
    y = host(rq.matmul_t_q(cuda(a), w))
    rq.stream_check()
    ref = orc.matmul_t_q(a, dtype, raw, n)          # tier dispatched on this host
    assert close(y, ref) < TOL
    if m * n * k <= 50_000_000:
        assert close(y, orc.int8_scalar_matmul(a, dtype, raw, n)) < TOL


@pytest.mark.parametrize("kind", [1, 2, 3])
@pytest.mark.parametrize("dtype", FORMATS)
@pytest.mark.parametrize("m,k,n", [(1, 1024, 1000), (2, 96, 41), (5, 768, 3072), (7, 160, 333), (8, 3072, 768),
                                   (3, 1280, 5120), (5, 4096, 257), (6, 8192, 40), (13, 1024, 700), (40, 256, 300),
                                   (64, 1280, 1280), (80, 1024, 1024), (200, 5120, 256)])
def test_gemv_kernels_match_oracle(rq, orc, kind, dtype, m, k, n):
    """The GEMV kernels (dp4a, integer MMA, tiled integer MMA) at every
    K-split and tail, one to several launches of rows."""
    if m * n * k > 100_000_000 and kind == 1:
        pytest.skip("dp4a at this size is covered by the smaller cases")
    a, raw = _case(dtype, m, k, n, 17 * dtype + m + k + kind)
    w = rq.QTensor([n, k], dtype, raw)
    rq.set_gemv_kernel(kind)
    try:
        y = host(rq.matmul_t_q(cuda(a), w))
        rq.stream_check()
    finally:
        rq.set_gemv_kernel(0)
    assert close(y, orc.int8_scalar_matmul(a, dtype, raw, n)) < TOL
    if k <= 4096:
        # The reference's x86 tier rounds its per-block f32 terms (the
        # +128 offset correction and the min term, quant.rs:452-454) on
        # its own: at k = 8192 the tier alone is ~1e-3 away from the exact
        # block dots for Q4_1/Q5_1, so the long row is held to the scalar
        # int8 oracle only.
        assert close(y, orc.matmul_t_q(a, dtype, raw, n)) < TOL


@pytest.mark.parametrize("kind", [1, 2, 3])
def test_gemv_batch_invariance_per_kernel(rq, kind):
    """Within each GEMV kernel a row's result is the same for M = 1..8."""
    import torch
    from rusty_whisper_b200 import synth
    rq.set_gemv_kernel(kind)
    try:
        for dtype in FORMATS:
            for k, n in ((1024, 3000), (768, 200)):
                w = rq.QTensor([n, k], dtype, synth.random_blocks(dtype, n, k, 31 + k))
                a = cuda(synth.normal(32, 8 * k).reshape(8, k))
                y8 = rq.matmul_t_q(a, w)
                for mm in (1, 2, 5, 7):
                    assert torch.equal(rq.matmul_t_q(a[:mm], w), y8[:mm])
    finally:
        rq.set_gemv_kernel(0)


@pytest.mark.parametrize("dtype", FORMATS)
@pytest.mark.parametrize("k,n", [(1280, 1280), (1280, 5120), (5120, 1280), (160, 333), (96, 41),
                                 (1280, 20000), (224, 19000)])
def test_gemv_tile_bit_identical_to_mma(rq, dtype, k, n):
    """The tiled kernel reproduces the integer-MMA GEMV's summation order
    (its K slices for KS > 1, the head/tail split of tiles shared by two
    warps for KS == 1, pad blocks when K/32 is not a multiple of 4), so the
    two give identical bits at every m and the switch between them keeps
    a row's result independent of m."""
    import torch
    from rusty_whisper_b200 import synth
    w = rq.QTensor([n, k], dtype, synth.random_blocks(dtype, n, k, 5 * dtype + n))
    bias = torch.from_numpy(synth.normal(3, n)).cuda()
    a = cuda(synth.normal(40 + k, 256 * k).reshape(256, k))
    try:
        for m in (1, 5, 16, 31, 32, 33, 63, 64, 80, 128, 200, 256):
            outs = []
            for kind in (2, 3, 0):
                rq.set_gemv_kernel(kind)
                outs.append(rq.matmul_t_q(a[:m], w, bias=bias if m % 2 else None))
            rq.stream_check()
            assert torch.equal(outs[0].view(torch.int32), outs[1].view(torch.int32)), (m, "mma vs tile")
            assert torch.equal(outs[0].view(torch.int32), outs[2].view(torch.int32)), (m, "mma vs auto")
    finally:
        rq.set_gemv_kernel(0)


@pytest.mark.parametrize("dtype", FORMATS)
@pytest.mark.parametrize("k,n", [(1024, 51865), (1280, 19000), (256, 20001), (224, 19000), (5120, 19200)])
def test_gemv_rows_bit_identical_to_mma(rq, orc, dtype, k, n):
    """The row-per-lane GEMV (one weight row per lane, dp4a block dots, the
    planes staged by TMA) reproduces the integer-MMA GEMV's summation order
    -- blocks in kb order, and the head/tail split of the 16-row tiles that
    two of its warps share -- so at one and two rows the two kernels give
    identical bits; it is the automatic choice there on wide weights
    (ragged N, pad blocks when K/32 is not a multiple of 4)."""
    import torch
    from rusty_whisper_b200 import synth
    raw = synth.random_blocks(dtype, n, k, 7 * dtype + n + k)
    w = rq.QTensor([n, k], dtype, raw)
    bias = torch.from_numpy(synth.normal(5, n)).cuda()
    a_np = synth.normal(60 + k, 2 * k).reshape(2, k)
    a = cuda(a_np)
    assert rq.gemv_kernel_for(w, 1) == 4 and rq.gemv_kernel_for(w, 2) == 4
    assert rq.gemv_kernel_for(w, 3) == 2
    try:
        for m in (1, 2):
            outs = []
            for kind in (2, 4, 0):
                rq.set_gemv_kernel(kind)
                outs.append(rq.matmul_t_q(a[:m], w, bias=bias if m == 1 else None))
            rq.stream_check()
            assert torch.equal(outs[0].view(torch.int32), outs[1].view(torch.int32)), (m, "mma vs rows")
            assert torch.equal(outs[0].view(torch.int32), outs[2].view(torch.int32)), (m, "mma vs auto")
    finally:
        rq.set_gemv_kernel(0)
    y = host(outs[2])
    assert close(y, orc.int8_scalar_matmul(a_np, dtype, raw, n)) < TOL


@pytest.mark.parametrize("dtype", FORMATS)
@pytest.mark.parametrize("m,k,n", [(1, 768, 768), (5, 256, 300), (20, 96, 41)])
def test_matmul_f32_mode_matches_dequant_then_fp(rq, orc, dtype, m, k, n):
    a, raw = _case(dtype, m, k, n, 13 * dtype + m)
    w = rq.QTensor([n, k], dtype, raw)
    y = host(rq.matmul_t_q(cuda(a), w, mode="f32"))
    ref = orc.matmul_t(a, orc.to_dense(dtype, raw, n, k))
    assert close(y, ref) < TOL


@pytest.mark.parametrize("dtype", FORMATS)
def test_dequant_rows_bit_exact(rq, orc, dtype):
    n, k = 77, 160
    _, raw = _case(dtype, 1, k, n, 3 * dtype)
    w = rq.QTensor([n, k], dtype, raw)
    dense = orc.to_dense(dtype, raw, n, k)
    assert np.array_equal(host(w.to_dense()).view(np.uint32), dense.view(np.uint32))
    rows = [76, 0, 13, 13]
    assert np.array_equal(host(w.rows_f32(rows)).view(np.uint32), dense[rows].view(np.uint32))
    assert np.array_equal(host(w.row_f32(5)).view(np.uint32), dense[5].view(np.uint32))


def test_batch_invariance(rq):
    """Row results do not depend on M (quant.rs:1372-1384), within each
    kernel family: the GEMV family (M <= 256, integer-MMA launches of up to
    64 rows) and the tensor-core GEMM (M > 256)."""
    import torch
    from rusty_whisper_b200 import synth
    for dtype in FORMATS:
        k, n = 512, 1200
        w = rq.QTensor([n, k], dtype, synth.random_blocks(dtype, n, k, 21))
        a = cuda(synth.normal(22, 700 * k).reshape(700, k))
        y256 = rq.matmul_t_q(a[:256], w)
        for mm in (1, 3, 8, 9, 17, 64, 65, 200):
            assert torch.equal(rq.matmul_t_q(a[:mm], w), y256[:mm])
        y700 = rq.matmul_t_q(a, w)
        for mm in (257, 300, 640):
            assert torch.equal(rq.matmul_t_q(a[:mm], w), y700[:mm])


def test_bias_and_host_path(rq, orc):
    from rusty_whisper_b200 import synth
    dtype, m, k, n = 7, 150, 256, 96
    a, raw = _case(dtype, m, k, n, 5)
    b = synth.normal(6, n)
    w = rq.QTensor([n, k], dtype, raw)
    y_dev = host(rq.linear_w(cuda(a), w, cuda(b)))
    y_host = rq.linear_w(a, w, b)                   # host buffers in, host out
    assert np.array_equal(y_dev, y_host)
    ref = orc.matmul_t_q(a, dtype, raw, n) + b[None, :]
    assert close(y_host, ref) < TOL
    for mm in (1, 5):                               # GEMV with bias
        y = rq.linear_w(a[:mm], w, b)
        assert close(y, ref[:mm]) < TOL


@pytest.mark.parametrize("m", [514, 1030, 1500])
def test_host_path_chunks_match_device_path(rq, orc, m):
    """Host-buffer calls of the GEMM family run in overlapped row chunks of
    more than 256 rows (1030 rows: four chunks of 257-258); the result is
    bit-identical to one device call, and pinned host buffers give the
    same as pageable ones."""
    import torch
    from rusty_whisper_b200 import synth
    dtype, k, n = 6, 768, 640
    a, raw = _case(dtype, m, k, n, 9 + m)
    b = synth.normal(8, n)
    w = rq.QTensor([n, k], dtype, raw)
    y_dev = host(rq.linear_w(cuda(a), w, cuda(b)))
    y_host = rq.linear_w(a, w, b)
    assert np.array_equal(y_dev.view(np.uint32), np.asarray(y_host).view(np.uint32))
    a_pin = torch.from_numpy(a).pin_memory()
    y_pin = rq.linear_w(a_pin.numpy(), w, b)
    assert np.array_equal(y_dev.view(np.uint32), np.asarray(y_pin).view(np.uint32))
    if m == 514:
        assert close(y_host, orc.matmul_t_q(a, dtype, raw, n) + b[None, :]) < TOL


def test_errors_and_edges(rq):
    import torch
    from rusty_whisper_b200 import synth
    w = rq.QTensor([40, 64], 8, synth.random_blocks(8, 40, 64, 1))
    with pytest.raises(ValueError):
        rq.matmul_t_q(torch.zeros((3, 96), device="cuda"), w)        # inner dims
    with pytest.raises(ValueError):
        rq.QTensor([4, 48], 8, bytes(4 * 34))                        # k % 32
    with pytest.raises(ValueError):
        rq.QTensor([4, 32], 4, bytes(4 * 18))                        # dtype
    with pytest.raises(ValueError):
        rq.QTensor([4, 32], 8, bytes(3 * 34))                        # raw length
    y = rq.matmul_t_q(torch.zeros((0, 64), device="cuda"), w)        # empty batch
    assert y.shape == (0, 40)
    z = rq.matmul_t_q(torch.zeros((20, 64), device="cuda"), w)      # zero blocks: d = 0
    assert torch.count_nonzero(z) == 0
    empty = rq.QTensor([0, 64], 8, b"")
    assert rq.matmul_t_q(torch.ones((3, 64), device="cuda"), empty).shape == (3, 0)
    with pytest.raises(ValueError):
        w.rows_f32([40])


@pytest.mark.parametrize("dtype", FORMATS)
def test_config2_full_shapes(rq, orc, dtype):
    """BASELINE config 2 at full size: M=1500 GEMMs and M in {1,5} GEMVs."""
    from rusty_whisper_b200 import synth
    for (k, n) in synth.SWEEP_SHAPES:
        raw = synth.sweep_weight(dtype, k, n)
        w = rq.QTensor([n, k], dtype, raw)
        for m in (synth.ENCODER_M,) + synth.SWEEP_GEMV_M:
            a = synth.sweep_acts(m, k)
            y = host(rq.matmul_t_q(cuda(a), w))
            ref = orc.matmul_t_q(a, dtype, raw, n)
            assert close(y, ref) < TOL, (k, n, m)


def test_qacts_reuse_matches_matmul(rq):
    """One quantization reused against several weights gives the same bits
    as separate matmul_t_q calls (GEMV and GEMM sizes)."""
    import torch
    from rusty_whisper_b200 import synth
    k = 256
    ws = [rq.QTensor([n, k], dt, synth.random_blocks(dt, n, k, 40 + dt)) for dt, n in ((2, 130), (7, 64), (8, 300))]
    qa = rq.QActs(400, k)
    for m in (1, 5, 8, 9, 400):
        a = cuda(synth.normal(50 + m, m * k).reshape(m, k))
        qa.quantize(a)
        for w in ws:
            assert torch.equal(qa.matmul(w), rq.matmul_t_q(a, w))
    with pytest.raises(ValueError):
        qa.quantize(torch.zeros((401, k), device="cuda"))


@pytest.mark.parametrize("dtype", FORMATS)
def test_exact_integer_gemm_path_matches_oracle(rq, orc, dtype):
    """Path 3: the tensor-core GEMM that forms every block's integer dot
    exactly and scales it on the CUDA cores."""
    m, k, n = 300, 768, 520
    a, raw = _case(dtype, m, k, n, 17 * dtype)
    w = rq.QTensor([n, k], dtype, raw)
    rq.set_gemm_path(3)
    try:
        y3 = host(rq.matmul_t_q(cuda(a), w))
    finally:
        rq.set_gemm_path(0)
    y2 = host(rq.matmul_t_q(cuda(a), w))
    ref = orc.matmul_t_q(a, dtype, raw, n)
    assert close(y3, ref) < TOL
    assert close(y2, ref) < TOL


@pytest.mark.parametrize("dtype", FORMATS)
def test_extreme_block_scales(rq, orc, dtype):
    """Rows whose f16 scales span huge, tiny and subnormal values: the
    folded-scale GEMM normalises each row by a power of two."""
    m, k, n = 150, 256, 64
    a, raw = _case(dtype, m, k, n, 23 * dtype)
    bb = orc.block_bytes(dtype)
    blocks = raw.reshape(-1, bb).copy()
    nb = k // 32
    for j in range(n):
        h = [0x6400, 0x5BFF, 0x0400, 0x0010, 0x3C00, 0x1400][j % 6]   # 1024, 255.9, 6.1e-5, 9.5e-7 (subnormal), 1, 2^-6
        for bl in range(nb):
            blocks[j * nb + bl, 0] = h & 0xFF
            blocks[j * nb + bl, 1] = h >> 8
    raw = blocks.reshape(-1)
    w = rq.QTensor([n, k], dtype, raw)
    y = host(rq.matmul_t_q(cuda(a), w))
    # The scalar int8 oracle is the reference's own tight check
    # (quant.rs:1336-1370).  At these magnitudes the VNNI tier's -128*sum(q_b)
    # offset loses f32 digits by cancellation, so it is not used here.
    assert close(y, orc.int8_scalar_matmul(a, dtype, raw, n)) < TOL


def test_unaligned_device_pointers(rq, orc):
    """Bias and output buffers offset by one float (4-byte aligned only)."""
    import torch
    from rusty_whisper_b200 import synth
    for m in (5, 200):
        dtype, k, n = 6, 256, 384
        a, raw = _case(dtype, m, k, n, 31 + m)
        w = rq.QTensor([n, k], dtype, raw)
        bias_buf = torch.from_numpy(synth.normal(9, n + 1)).cuda()
        bias = bias_buf[1:]
        out_buf = torch.empty(m * n + 1, device="cuda")
        out = out_buf[1:].view(m, n)
        rq.matmul_t_q(cuda(a), w, out=out, bias=bias)
        ref = orc.matmul_t_q(a, dtype, raw, n) + bias.cpu().numpy()[None, :]
        assert close(host(out), ref) < TOL
    rq.set_gemm_path(3)
    try:
        out_buf = torch.empty(200 * n + 1, device="cuda")
        out = out_buf[1:].view(200, n)
        a, raw = _case(6, 200, 256, n, 77)
        w = rq.QTensor([n, 256], 6, raw)
        rq.matmul_t_q(cuda(a), w, out=out, bias=bias)
        assert close(host(out), orc.matmul_t_q(a, 6, raw, n) + bias.cpu().numpy()[None, :]) < TOL
    finally:
        rq.set_gemm_path(0)


def test_quantizer_unaligned_and_nan(rq, orc):
    """Activations at a 4-byte (not 16-byte) offset, with NaN and inf."""
    import torch
    from rusty_whisper_b200 import synth
    m, k = 7, 96
    a = synth.normal(3, m * k).reshape(m, k)
    a[1, 5] = np.nan
    a[2, 40] = np.inf
    a[3, 64:96] = 0.0
    buf = torch.zeros(m * k + 1, device="cuda")
    buf[1:] = torch.from_numpy(a.ravel()).cuda()
    av = buf[1:].view(m, k)
    q, d, s = rq.quantize_acts_i8(av)
    qr, dr, sr = orc.quantize_acts_i8(a)
    assert np.array_equal(host(q), qr)
    assert np.array_equal(host(d).view(np.uint32), dr.view(np.uint32))
    assert np.array_equal(host(s), sr)


@pytest.mark.parametrize("dtype", FORMATS)
@pytest.mark.parametrize("m,k,n", [(257, 96, 41), (300, 768, 257), (640, 256, 64), (700, 1024, 130),
                                   (1500, 768, 768), (1500, 3072, 768), (1100, 5120, 1280)])
def test_hl_gemm_both_modes_match_oracle(rq, orc, dtype, m, k, n):
    """The hi|lo tensor-core GEMM in both tiers (forced for int8, the f32
    tier's kernel from 257 rows): int8 activation semantics against the
    exact int8 sum and the oracle's dispatched tier, and dequant-then-f32
    against the oracle's f32 `matmul_t(a, to_dense)` (quant.rs:1194), at
    every K split (1, 2, 4), tile width (64, 128, 256) and ragged M / N
    edge."""
    a, raw = _case(dtype, m, k, n, 19 * dtype + m + k)
    w = rq.QTensor([n, k], dtype, raw)
    rq.set_gemm_path(4)
    try:
        y = host(rq.matmul_t_q(cuda(a), w))
        rq.stream_check()
    finally:
        rq.set_gemm_path(0)
    assert close(y, exact_int8(orc, a, dtype, raw, n)) < TOL
    if k <= 4096:
        # Beyond k = 4096 the reference's x86 tier itself drifts ~1e-3 from
        # the exact block dots for the min formats (its per-block f32
        # terms, quant.rs:452-454), so long rows are held to the exact sum.
        assert close(y, orc.matmul_t_q(a, dtype, raw, n)) < TOL
    yf = host(rq.matmul_t_q(cuda(a), w, mode="f32"))
    rq.stream_check()
    assert close(yf, orc.matmul_t(a, orc.to_dense(dtype, raw, n, k))) < TOL


@pytest.mark.parametrize("path", [2, 3, 4])
def test_gemm_paths_agree_with_oracle(rq, orc, path):
    """Each tensor-core GEMM path, forced, on the config-2 shapes of one
    format (Q5_1: scales and minimums on both sides)."""
    from rusty_whisper_b200 import synth
    rq.set_gemm_path(path)
    try:
        for (k, n) in synth.SWEEP_SHAPES:
            raw = synth.sweep_weight(7, k, n)
            w = rq.QTensor([n, k], 7, raw)
            a = synth.sweep_acts(synth.ENCODER_M, k)
            y = host(rq.matmul_t_q(cuda(a), w))
            rq.stream_check()
            assert close(y, orc.matmul_t_q(a, 7, raw, n)) < TOL, (path, k, n)
    finally:
        rq.set_gemm_path(0)


def test_hl_gemm_row_scales_span_f32_range(rq, orc):
    """Activation rows of magnitude 1e-30 .. 1e30 and rows of zeros: each
    row is normalised by its own power of two before the f16 split."""
    from rusty_whisper_b200 import synth
    dtype, m, k, n = 6, 300, 256, 200
    a, raw = _case(dtype, m, k, n, 91)
    scales = np.array([1e-30, 1e-12, 1e-3, 1.0, 37.0, 1e6, 1e20, 1e30, 0.0], np.float32)
    a = (a * scales[np.arange(m) % scales.size][:, None]).astype(np.float32)
    w = rq.QTensor([n, k], dtype, raw)
    rq.set_gemm_path(4)
    try:
        y = host(rq.matmul_t_q(cuda(a), w))
    finally:
        rq.set_gemm_path(0)
    ref = orc.int8_scalar_matmul(a, dtype, raw, n)
    # The 1e-3 rule relative to max(|ref|, 1) is not scale-free (vacuous for
    # tiny rows, elementwise-relative for huge ones, where outputs near
    # zero come from cancellation), so every row is held to 1e-3 of its own
    # largest output instead.
    for i in range(m):
        s = max(float(np.abs(ref[i]).max()), 1e-37)
        assert float(np.abs(y[i] - ref[i]).max()) <= 1e-3 * s, i
    yf = host(rq.matmul_t_q(cuda(a), w, mode="f32"))
    reff = orc.matmul_t(a, orc.to_dense(dtype, raw, n, k))
    for i in range(m):
        s = max(float(np.abs(reff[i]).max()), 1e-37)
        assert float(np.abs(yf[i] - reff[i]).max()) <= 1e-3 * s, i


def test_hl_gemm_unaligned_and_host_f32(rq, orc):
    """Activations, bias and output at 4-byte offsets on the hi|lo GEMM, and
    the f32 tier through the host-buffer entry point (chunked)."""
    import torch
    from rusty_whisper_b200 import synth
    dtype, m, k, n = 3, 600, 384, 258
    a, raw = _case(dtype, m, k, n, 5)
    w = rq.QTensor([n, k], dtype, raw)
    abuf = torch.zeros(m * k + 1, device="cuda")
    abuf[1:] = torch.from_numpy(a.ravel()).cuda()
    bias_buf = torch.from_numpy(synth.normal(9, n + 1)).cuda()
    out_buf = torch.empty(m * n + 1, device="cuda")
    out = out_buf[1:].view(m, n)
    rq.set_gemm_path(4)
    try:
        rq.matmul_t_q(abuf[1:].view(m, k), w, out=out, bias=bias_buf[1:])
    finally:
        rq.set_gemm_path(0)
    ref = orc.matmul_t_q(a, dtype, raw, n) + bias_buf[1:].cpu().numpy()[None, :]
    assert close(host(out), ref) < TOL
    yh = rq.matmul_t_q(a, w, mode="f32")           # host buffers, row chunks
    yd = host(rq.matmul_t_q(cuda(a), w, mode="f32"))
    assert np.array_equal(np.asarray(yh).view(np.uint32), yd.view(np.uint32))
    assert close(yh, orc.matmul_t(a, orc.to_dense(dtype, raw, n, k))) < TOL
