"""Pin the CPU oracle to rusty_whisper's own tests for the quant path.

Each test restates one reference test (file:line in the reference's
``src/``) with its exact inputs and assertions, run against the oracle.
The reference itself is Rust and cannot be built in this image, so these
known answers are the parity anchor.
"""
import math

import numpy as np
import pytest

QK = 32
FORMATS = (2, 3, 6, 7, 8)


def f16le(h):
    return bytes([h & 0xFF, h >> 8])


# model.rs:282-291
def test_f16_conversion_reference_values(orc):
    assert orc.f16_to_f32(0x0000) == 0.0
    assert orc.f16_to_f32(0x3C00) == 1.0
    assert orc.f16_to_f32(0xC000) == -2.0
    assert orc.f16_to_f32(0x3555) == np.float32(0.33325195)
    assert abs(orc.f16_to_f32(0x0001) - 5.9604645e-8) < 1e-12
    assert math.isinf(orc.f16_to_f32(0x7C00))
    assert math.isnan(orc.f16_to_f32(0x7E00))


# model.rs:383-390
def test_f16_round_trip(orc):
    for v in [0.0, 1.0, -2.0, 0.333251953125, 65504.0, 6.1035156e-5]:
        v32 = float(np.float32(v))
        assert orc.f16_to_f32(orc.f32_to_f16(v32)) == v32
    assert math.isinf(orc.f16_to_f32(orc.f32_to_f16(1e20)))


# model.rs:90-115: half-up rounding on bit 12, not round-to-nearest-even.
def test_f32_to_f16_rounds_half_up(orc):
    # 1 + 2^-11 is exactly halfway between two f16 values: RNE gives 0x3C00,
    # the reference's encoder gives 0x3C01.
    assert orc.f32_to_f16(1.0 + 2.0 ** -11) == 0x3C01


# model.rs:348-381
def test_dequant_known_blocks_via_qtensor(orc):
    raw = bytearray(34)
    raw[0:2] = f16le(0x3800)
    raw[2] = 0
    raw[3] = 1
    raw[4] = (-2) & 0xFF
    for i in range(5, 34):
        raw[i] = 3
    d = orc.to_dense(8, np.frombuffer(bytes(raw), np.uint8), 1, 32)[0]
    assert list(d[:3]) == [0.0, 0.5, -1.0]
    assert d[31] == 1.5

    raw = bytearray(18)
    raw[0:2] = f16le(0x3C00)
    raw[2] = 0xF8
    d = orc.to_dense(2, np.frombuffer(bytes(raw), np.uint8), 1, 32)[0]
    assert d[0] == 0.0 and d[16] == 7.0 and d[1] == -8.0

    raw = bytearray(22)
    raw[0:2] = f16le(0x3C00)
    raw[2:6] = (1).to_bytes(4, "little")
    d = orc.to_dense(6, np.frombuffer(bytes(raw), np.uint8), 1, 32)[0]
    assert d[0] == 0.0 and d[16] == -16.0


# quant.rs:1162-1174
def test_unpack_matches_f32_dequant_reference(orc):
    block = bytearray(24)
    block[0:2] = f16le(0x3800)
    block[2:4] = f16le(0x4000)
    block[4:8] = (1).to_bytes(4, "little")
    block[8] = 0x03
    q, d, m = orc.unpack_block(7, bytes(block))
    assert np.float32(d) * np.float32(q[0]) + np.float32(m) == 11.5
    assert np.float32(d) * np.float32(q[1]) + np.float32(m) == 2.0


# quant.rs:1125-1160
@pytest.mark.skipif("not __import__('oracle').lib().orc_has_avx2()")
def test_avx2_dequant_bit_identical_to_scalar(orc):
    for dtype in FORMATS:
        bb = orc.block_bytes(dtype)
        nb = 7
        raw = orc.rand_bytes(0x12345678, nb * bb).copy()
        for bl in range(nb):
            raw[bl * bb: bl * bb + 2] = [0x55, 0x35]
            if dtype in (3, 7):
                raw[bl * bb + 2: bl * bb + 4] = [0x55, 0xB5]
        a = orc.dequant_row_scalar(dtype, raw)
        b = orc.dequant_row_avx2(dtype, raw)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), dtype


# quant.rs:1176-1185
def test_qtensor_row_roundtrip(orc):
    x = orc.test_matrix(3, 64, 7)
    raw = orc.quantize_q8_0(x)
    dense = orc.to_dense(8, raw, 3, 64)
    assert np.all(np.abs(dense[1] - x[64:128]) < 0.02)


def _dense_check(orc, m, k, n, dtype, sa, sb, tier=0):
    a = orc.test_matrix(1, m * k, sa).reshape(m, k)
    bx = orc.test_matrix(n, k, sb)
    raw = orc.quantize_q8_0(bx) if dtype == 8 else orc.quantize_q5_1(bx)
    fast = orc.matmul_t_q(a, dtype, raw, n, tier=tier)
    ref = orc.matmul_t(a, orc.to_dense(dtype, raw, n, k))
    rms = float(np.sqrt(np.mean(ref.astype(np.float32) ** 2)))
    assert np.all(np.abs(fast - ref) < 0.05 * max(rms, 1.0))


# quant.rs:1187-1206, 1213-1232, 1236-1255, 1259-1278, 1282-1301
@pytest.mark.parametrize("m,k,n,dtype,sa,sb", [
    (7, 96, 33, 8, 11, 13),
    (1500, 384, 1536, 7, 41, 43),
    (37, 96, 41, 8, 17, 19),
    (37, 96, 41, 7, 23, 29),
    (600, 128, 600, 7, 31, 37),
])
def test_matmul_t_q_matches_dense_within_quant_error(orc, m, k, n, dtype, sa, sb):
    _dense_check(orc, m, k, n, dtype, sa, sb)


# quant.rs:1311-1331: repeated calls on one weight (cold path, then cache)
def test_matmul_t_q_repeated_calls_same_tensor_stay_correct(orc):
    k, n = 96, 41
    raw = orc.quantize_q5_1(orc.test_matrix(n, k, 29))
    qt = orc.QTensor(7, raw, n, k)
    dense = orc.to_dense(7, raw, n, k)
    for call in range(5):
        m = 1 + call
        a = orc.test_matrix(1, m * k, 100 + call).reshape(m, k)
        fast = qt.matmul(a)
        ref = orc.matmul_t(a, dense)
        rms = float(np.sqrt(np.mean(ref ** 2)))
        assert np.all(np.abs(fast - ref) < 0.05 * max(rms, 1.0))
        # cold path and cached path give the same bits
        assert np.array_equal(fast, orc.matmul_t_q(a, 7, raw, n))


# quant.rs:1336-1370: the tight scalar int8 oracle, on every tier present.
@pytest.mark.parametrize("tier", [1, 2])
def test_int8_gemm_matches_scalar_reference(orc, tier):
    if tier == 1 and not orc.lib().orc_has_vnni():
        pytest.skip("no VNNI on this host")
    m, k, n = 5, 128, 20
    a = orc.test_matrix(1, m * k, 41).reshape(m, k)
    raw = orc.quantize_q8_0(orc.test_matrix(n, k, 43))
    fast = orc.matmul_t_q(a, 8, raw, n, tier=tier)
    acc = orc.int8_scalar_matmul(a, 8, raw, n)
    assert np.all(np.abs(fast - acc) < 1e-3 * np.maximum(np.abs(acc), 1.0))


# quant.rs:1372-1384: batch invariance, row 0 at M=8 bit-equals M=1.
def test_matmul_t_q_parallel_matches_serial(orc):
    m, k, n = 8, 128, 1200
    a = orc.test_matrix(1, m * k, 21).reshape(m, k)
    raw = orc.quantize_q8_0(orc.test_matrix(n, k, 23))
    par = orc.matmul_t_q(a, 8, raw, n)
    one = orc.matmul_t_q(a[:1].copy(), 8, raw, n)
    assert np.array_equal(par[0], one[0])


# Extension beyond the reference's tests (it has none for Q4_x/Q5_0 int8
# dots): the integer block dots reproduce the scalar int8 matmul exactly,
# and each tier sits within the reference's 1e-3 rule of it, all formats.
@pytest.mark.parametrize("dtype", FORMATS)
def test_all_formats_tiers_match_scalar_int8(orc, dtype):
    from rusty_whisper_b200 import synth
    m, k, n = 9, 256, 37
    a = synth.normal(3, m * k).reshape(m, k)
    raw = synth.random_blocks(dtype, n, k, 11)
    ref = orc.int8_scalar_matmul(a, dtype, raw, n)
    qa, da, sa = orc.quantize_acts_i8(a)
    S = orc.block_dots(qa, dtype, raw, n)
    # recombine S with the scales in float64: the int8 semantics exactly
    nb = k // QK
    dense = np.zeros((n, nb), np.float64)
    mins = np.zeros((n, nb), np.float64)
    bb = orc.block_bytes(dtype)
    for j in range(n):
        for bl in range(nb):
            _, d, mm = orc.unpack_block(dtype, bytes(raw[(j * nb + bl) * bb:(j * nb + bl + 1) * bb]))
            dense[j, bl], mins[j, bl] = d, mm
    exact = np.einsum("ijb,ib,jb->ij", S.astype(np.float64), da.astype(np.float64), dense) + \
        np.einsum("ib,ib,jb->ij", da.astype(np.float64), sa.astype(np.float64), mins)
    assert np.all(np.abs(ref - exact) < 1e-4 * np.maximum(np.abs(exact), 1.0))
    for tier in (1, 2):
        if tier == 1 and not orc.lib().orc_has_vnni():
            continue
        got = orc.matmul_t_q(a, dtype, raw, n, tier=tier)
        assert np.all(np.abs(got - ref) < 1e-3 * np.maximum(np.abs(ref), 1.0)), tier
    # f32 fallback == matmul_t(a, to_dense) bit for bit (same dot kernels)
    f32 = orc.matmul_t_q(a, dtype, raw, n, tier=3)
    assert np.array_equal(f32, orc.matmul_t(a, orc.to_dense(dtype, raw, n, k)))


# quant.rs:690-716 edge cases: zero block, NaN-free clamp, rounding.
def test_quantize_acts_edges(orc):
    a = np.zeros((2, 64), np.float32)
    a[1, :32] = np.linspace(-1, 1, 32, dtype=np.float32)
    a[1, 32] = 127.0
    a[1, 33] = 0.5   # 0.5 * 127/127 = 0.5 -> rounds away from zero to 1
    q, d, s = orc.quantize_acts_i8(a)
    assert np.all(q[0] == 0) and np.all(d[0] == 0) and np.all(s[0] == 0)
    assert q[1, 31] == 127 and q[1, 0] == -127
    assert q[1, 32] == 127 and q[1, 33] == 1
    assert s[1, 0] == int(q[1, :32].astype(np.int32).sum())
