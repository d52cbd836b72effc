"""Seeded synthetic inputs for the quantized-matmul configurations.

One documented generator feeds every test and benchmark so that the GPU
path, the CPU oracle and the timed CPU baseline see identical bytes:

* SplitMix64 (Steele, Lea & Flood 2014) produces 64-bit words;
* ``uniform``: top 24 bits -> float in [0, 1);
* ``normal``: Box-Muller on two uniforms (float64 math, cast to f32);
* f16 scales are encoded with rusty_whisper's own ``f32_to_f16``
  (model.rs:90-115), which rounds half-up on the first dropped bit, not
  to nearest-even.

Block construction follows BASELINE configs 1 and 2: uniform random
nibbles / high bits / int8 codes, d ~ U(0.001, 0.02), m ~ U(-0.05, 0.05),
and activations ~ N(0, 1).  No dataset is involved.
"""
from __future__ import annotations

import numpy as np

from .formats import QK, block_bytes, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, count: int) -> np.ndarray:
    """``count`` SplitMix64 outputs for state ``seed`` (vectorised)."""
    with np.errstate(over="ignore"):
        idx = np.arange(1, count + 1, dtype=np.uint64)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + idx * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    return z


def uniform(seed: int, count: int, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    u = (splitmix64(seed, count) >> np.uint64(40)).astype(np.float64) * (1.0 / (1 << 24))
    return (lo + (hi - lo) * u).astype(np.float32)


def normal(seed: int, count: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    half = (count + 1) // 2
    w = splitmix64(seed, 2 * half)
    u1 = ((w[0::2] >> np.uint64(40)).astype(np.float64) + 1.0) * (1.0 / (1 << 24))  # (0, 1]
    u2 = (w[1::2] >> np.uint64(40)).astype(np.float64) * (1.0 / (1 << 24))
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * half, np.float64)
    z[0::2] = r * np.cos(2.0 * np.pi * u2)
    z[1::2] = r * np.sin(2.0 * np.pi * u2)
    return (mean + std * z[:count]).astype(np.float32)


def randint(seed: int, count: int, lo: int, hi_inclusive: int) -> np.ndarray:
    span = np.uint64(hi_inclusive - lo + 1)
    return ((splitmix64(seed, count) >> np.uint64(11)) % span).astype(np.int64) + lo


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    """rusty_whisper's f32 -> f16 (model.rs:90-115), vectorised: half-up."""
    x = np.ascontiguousarray(x, np.float32)
    bits = x.view(np.uint32).astype(np.int64)
    sign = (bits >> 16) & 0x8000
    exp = (bits >> 23) & 0xFF
    frac = bits & 0x7FFFFF
    e = exp - 127 + 15
    out = np.zeros(x.shape, np.int64)
    # normal range
    norm = (half := ((e << 10) | (frac >> 13))) + ((frac >> 12) & 1)
    out = np.where((e > 0) & (e < 0x1F), sign | norm, out)
    # overflow -> inf
    out = np.where((e >= 0x1F) & (exp != 0xFF), sign | 0x7C00, out)
    # nan / inf
    out = np.where(exp == 0xFF, sign | 0x7C00 | np.where(frac != 0, 0x200, 0), out)
    # subnormal
    sub = (e <= 0) & (e >= -10)
    f = frac | 0x800000
    shift = np.clip(14 - e, 1, 63)
    subv = (f >> shift) + ((f >> (shift - 1)) & 1)
    out = np.where(sub, sign | subv, out)
    out = np.where(e < -10, sign, out)
    del half
    return out.astype(np.uint16)


def random_blocks(dtype: int, n: int, k: int, seed: int) -> np.ndarray:
    """Raw ggml bytes for an ``[n, k]`` weight: codes uniform over their
    range, d ~ U(0.001, 0.02), m ~ U(-0.05, 0.05)."""
    assert k % QK == 0
    nblk = n * (k // QK)
    bb = block_bytes(dtype)
    raw = np.zeros((nblk, bb), np.uint8)
    d = f32_to_f16_bits(uniform(seed * 4 + 1, nblk, 0.001, 0.02))
    raw[:, 0] = d & 0xFF
    raw[:, 1] = d >> 8
    if dtype in (Q4_1, Q5_1):
        mm = f32_to_f16_bits(uniform(seed * 4 + 2, nblk, -0.05, 0.05))
        raw[:, 2] = mm & 0xFF
        raw[:, 3] = mm >> 8
    if dtype == Q8_0:
        codes = randint(seed * 4 + 3, nblk * QK, -127, 127).astype(np.int8)
        raw[:, 2:] = codes.view(np.uint8).reshape(nblk, QK)
    else:
        body = randint(seed * 4 + 3, nblk * (bb - (2 if dtype in (Q4_0, Q5_0) else 4)), 0, 255)
        off = 2 if dtype in (Q4_0, Q5_0) else 4
        raw[:, off:] = body.astype(np.uint8).reshape(nblk, bb - off)
    return raw.reshape(-1)


def config1_inputs(seed: int = 0):
    """Q8_0 W[1536x384], X[1500x384] ~ N(0,1), seed 0."""
    w = random_blocks(Q8_0, 1536, 384, seed)
    x = normal(seed * 4 + 7, 1500 * 384).reshape(1500, 384)
    return x, w


# whisper-small encoder shapes and decoder GEMVs.
SWEEP_FORMATS = (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0)
SWEEP_SHAPES = ((768, 768), (768, 3072), (3072, 768))   # (K, N)
SWEEP_GEMV_M = (1, 5)
ENCODER_M = 1500


def sweep_weight(dtype: int, k: int, n: int, seed: int = 0) -> np.ndarray:
    return random_blocks(dtype, n, k, 1000 + 97 * seed + 13 * dtype + k // 32 + 7 * (n // 32))


def sweep_acts(m: int, k: int, seed: int = 0) -> np.ndarray:
    return normal(5000 + 31 * seed + m + 3 * k, m * k).reshape(m, k)


# BASELINE config 5's audio: 30 s windows of 16 kHz band-limited noise at
# about -20 dBFS with random silences of 0.2-2 s (synthetic speech stand-in).
AUDIO_WINDOW = 480_000


def speechlike_window(seed: int, n: int = AUDIO_WINDOW) -> np.ndarray:
    x = normal(seed, n, 0.0, 1.0).astype(np.float64)
    # band-limit with a 9-tap Hann smoother, then scale to ~-20 dBFS RMS
    k = np.hanning(11)[1:-1]
    x = np.convolve(x, k / k.sum(), mode="same")
    x *= 0.1 / max(float(np.sqrt(np.mean(x * x))), 1e-12)
    starts = randint(seed + 1, 8, 0, n - 1)
    lens = randint(seed + 2, 8, 3200, 32000)
    for a, ln in zip(starts, lens):
        x[int(a):int(a) + int(ln)] = 0.0
    return x.astype(np.float32)
