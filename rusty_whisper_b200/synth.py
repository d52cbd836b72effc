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


def random_blocks(dtype: int, n: int, k: int, seed: int, d_range=(0.001, 0.02), m_range=(-0.05, 0.05)) -> np.ndarray:
    """Raw ggml bytes for an ``[n, k]`` weight: codes uniform over their
    range, d ~ U(d_range), m ~ U(m_range) (defaults)."""
    assert k % QK == 0
    nblk = n * (k // QK)
    bb = block_bytes(dtype)
    raw = np.zeros((nblk, bb), np.uint8)
    d = f32_to_f16_bits(uniform(seed * 4 + 1, nblk, *d_range))
    raw[:, 0] = d & 0xFF
    raw[:, 1] = d >> 8
    if dtype in (Q4_1, Q5_1):
        mm = f32_to_f16_bits(uniform(seed * 4 + 2, nblk, *m_range))
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


# ------------------------------------------- the same generator in torch
# Bit-identical to ``splitmix64`` / ``uniform`` / ``randint`` /
# ``f32_to_f16_bits`` / ``random_blocks`` above, on int64 torch tensors
# (two's-complement wrap-around for the multiplies, masked shifts for the
# logical right shifts), so deep models' weights can be drawn on the GPU:
# every layer its own draw in a fraction of the time NumPy takes.
def _s64(x: int) -> int:
    x &= 0xFFFFFFFFFFFFFFFF
    return x - (1 << 64) if x >= (1 << 63) else x


def _t_srl(z, s: int):
    return (z >> s) & ((1 << (64 - s)) - 1)


def splitmix64_torch(seed: int, start: int, count: int, device):
    import torch
    idx = torch.arange(start + 1, start + count + 1, dtype=torch.int64, device=device)
    z = idx * _s64(0x9E3779B97F4A7C15) + _s64(seed)
    z = (z ^ _t_srl(z, 30)) * _s64(0xBF58476D1CE4E5B9)
    z = (z ^ _t_srl(z, 27)) * _s64(0x94D049BB133111EB)
    return z ^ _t_srl(z, 31)


def uniform_torch(seed: int, count: int, lo: float, hi: float, device):
    import torch
    u = _t_srl(splitmix64_torch(seed, 0, count, device), 40).to(torch.float64) * (1.0 / (1 << 24))
    return (lo + (hi - lo) * u).to(torch.float32)


def f32_to_f16_bits_torch(x):
    """``f32_to_f16_bits`` (the reference's half-up f32 -> f16) in torch."""
    import torch
    bits = x.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    sign = (bits >> 16) & 0x8000
    exp = (bits >> 23) & 0xFF
    frac = bits & 0x7FFFFF
    e = exp - 127 + 15
    out = torch.zeros_like(bits)
    norm = ((e << 10) | (frac >> 13)) + ((frac >> 12) & 1)
    out = torch.where((e > 0) & (e < 0x1F), sign | norm, out)
    out = torch.where((e >= 0x1F) & (exp != 0xFF), sign | 0x7C00, out)
    out = torch.where(exp == 0xFF, sign | 0x7C00 | torch.where(frac != 0, 0x200, 0), out)
    sub = (e <= 0) & (e >= -10)
    f = frac | 0x800000
    shift = torch.clamp(14 - e, 1, 63)
    subv = (f >> shift) + ((f >> (shift - 1)) & 1)
    out = torch.where(sub, sign | subv, out)
    out = torch.where(e < -10, sign, out)
    return out


def random_blocks_torch(dtype: int, n: int, k: int, seed: int, d_range=(0.001, 0.02), m_range=(-0.05, 0.05),
                        device="cuda", chunk: int = 1 << 26):
    """``random_blocks`` drawn on ``device``: a uint8 tensor with the same
    bytes as the NumPy version."""
    import torch
    assert k % QK == 0
    nblk = n * (k // QK)
    bb = block_bytes(dtype)
    raw = torch.zeros((nblk, bb), dtype=torch.uint8, device=device)
    d = f32_to_f16_bits_torch(uniform_torch(seed * 4 + 1, nblk, *d_range, device))
    raw[:, 0] = (d & 0xFF).to(torch.uint8)
    raw[:, 1] = (d >> 8).to(torch.uint8)
    if dtype in (Q4_1, Q5_1):
        mm = f32_to_f16_bits_torch(uniform_torch(seed * 4 + 2, nblk, *m_range, device))
        raw[:, 2] = (mm & 0xFF).to(torch.uint8)
        raw[:, 3] = (mm >> 8).to(torch.uint8)
    if dtype == Q8_0:
        off, lo, hi = 2, -127, 127
    else:
        off, lo, hi = (2 if dtype in (Q4_0, Q5_0) else 4), 0, 255
    body = raw[:, off:].reshape(-1)
    span = hi - lo + 1
    for c0 in range(0, body.numel(), chunk):
        c = min(chunk, body.numel() - c0)
        v = _t_srl(splitmix64_torch(seed * 4 + 3, c0, c, device), 11) % span + lo
        body[c0:c0 + c] = (v & 0xFF).to(torch.uint8)
    raw[:, off:] = body.view(nblk, bb - off)
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


# ---------------------------------------------------------------- models
def quantize_q5_1(x: np.ndarray) -> np.ndarray:
    """rusty_whisper's Q5_1 test quantizer (quant.rs:1088-1113), vectorised:
    per block d = (max-min)/31, q = round((x-min)/d) clamped to [0, 31]
    (half away from zero), d and min as f16 (half-up, model.rs:90-115)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, QK)
    mn = x.min(axis=1)
    mx = x.max(axis=1)
    d = ((mx - mn) / np.float32(31.0)).astype(np.float32)
    inv = np.where(d > 0, np.float32(1.0) / np.where(d > 0, d, np.float32(1.0)), np.float32(0.0)).astype(np.float32)
    t = ((x - mn[:, None]).astype(np.float32) * inv[:, None]).astype(np.float32)
    q = np.clip(np.floor(t.astype(np.float64) + 0.5), 0, 31).astype(np.uint32)
    nblk = x.shape[0]
    raw = np.zeros((nblk, 24), np.uint8)
    db = f32_to_f16_bits(d)
    mb = f32_to_f16_bits(mn.astype(np.float32))
    raw[:, 0], raw[:, 1] = db & 0xFF, db >> 8
    raw[:, 2], raw[:, 3] = mb & 0xFF, mb >> 8
    qh = np.zeros(nblk, np.uint32)
    for e in range(QK):
        qh |= ((q[:, e] >> 4) & 1) << np.uint32(e)
    raw[:, 4:8] = qh.view(np.uint8).reshape(nblk, 4)
    raw[:, 8:24] = ((q[:, :16] & 0xF) | ((q[:, 16:] & 0xF) << 4)).astype(np.uint8)
    return raw.reshape(-1)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """rusty_whisper's Q8_0 test quantizer (quant.rs:1071-1083), vectorised:
    per block d = amax/127, q = round(x/d) half away from zero, clamped to
    [-127, 127], d as f16 (half-up)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, QK)
    amax = np.abs(x).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    inv = np.where(d > 0, np.float32(1.0) / np.where(d > 0, d, np.float32(1.0)), np.float32(0.0)).astype(np.float32)
    t = (x * inv[:, None]).astype(np.float32).astype(np.float64)
    q = np.clip(np.sign(t) * np.floor(np.abs(t) + 0.5), -127, 127).astype(np.int8)
    nblk = x.shape[0]
    raw = np.zeros((nblk, 34), np.uint8)
    db = f32_to_f16_bits(d)
    raw[:, 0], raw[:, 1] = db & 0xFF, db >> 8
    raw[:, 2:] = q.view(np.uint8)
    return raw.reshape(-1)


# Random-code model weights (formats without a reference quantizer): block
# scales chosen so that the weights' standard deviation is about 0.02, like
# the N(0, 0.02) init the other formats are quantized from.
MODEL_CODE_SCALES = {
    Q4_0: ((0.002, 0.007), (0.0, 0.0)),        # q in -8..7: std ~ 4.6 d
    Q4_1: ((0.002, 0.007), (-0.04, -0.02)),    # q in 0..15, m ~ -7.5 d
    Q5_0: ((0.001, 0.0035), (0.0, 0.0)),       # q in -16..15: std ~ 9.2 d
}


def encoder_tensors(n_mels: int, n_ctx: int, n_state: int, n_layer: int, dtype: int, seed: int,
                    reuse_layers: bool = False, gen_device=None) -> dict:
    """Random-init whisper encoder tensors by their whisper.cpp names
    (encoder.rs:130-234): dense entries are f32 arrays, the six linears of
    each block ``(dtype, raw, n, k)``.  Weights ~ N(0, 0.02); Q5_1 and Q8_0
    linears are quantized from them with the reference's own test
    quantizers (BASELINE config 3 is Q5_1), the other formats get random
    codes with block scales giving a similar spread (MODEL_CODE_SCALES);
    LayerNorm weights 1 + N(0, 0.02);
    positions are whisper's sinusoids.  With ``reuse_layers`` every block
    gets block 0's values (each still becomes its own device copy).
    ``gen_device`` (e.g. "cuda"): the random-code linears are drawn there
    by ``random_blocks_torch`` (the same bytes, much faster for deep
    models) and returned as host arrays."""
    t = {}
    ctr = [seed * 1000]

    def nrm(*shape, std=0.02, mean=0.0):
        ctr[0] += 1
        return normal(ctr[0], int(np.prod(shape)), mean, std).reshape(shape)

    def lin(n, k):
        ctr[0] += 1
        if dtype == Q5_1:
            return (dtype, quantize_q5_1(normal(ctr[0], n * k, 0.0, 0.02)), n, k)
        if dtype == Q8_0:
            return (dtype, quantize_q8_0(normal(ctr[0], n * k, 0.0, 0.02)), n, k)
        if gen_device is not None:
            raw = random_blocks_torch(dtype, n, k, ctr[0], *MODEL_CODE_SCALES[dtype], device=gen_device)
            return (dtype, raw.cpu().numpy(), n, k)
        return (dtype, random_blocks(dtype, n, k, ctr[0], *MODEL_CODE_SCALES[dtype]), n, k)

    t["encoder.conv1.weight"] = nrm(n_state, n_mels, 3)
    t["encoder.conv1.bias"] = nrm(n_state)
    t["encoder.conv2.weight"] = nrm(n_state, n_state, 3)
    t["encoder.conv2.bias"] = nrm(n_state)
    half = n_state // 2
    inc = np.log(10000.0) / (half - 1)
    inv = np.exp(-inc * np.arange(half))
    ang = np.arange(n_ctx)[:, None] * inv[None, :]
    t["encoder.positional_embedding"] = np.concatenate([np.sin(ang), np.cos(ang)], axis=1).astype(np.float32)
    for l in range(n_layer):
        p = f"encoder.blocks.{l}"
        if reuse_layers and l > 0:
            for key in [x for x in t if x.startswith("encoder.blocks.0.")]:
                t[key.replace("encoder.blocks.0.", f"{p}.", 1)] = t[key]
            continue
        t[f"{p}.attn_ln.weight"] = nrm(n_state, mean=1.0)
        t[f"{p}.attn_ln.bias"] = nrm(n_state)
        t[f"{p}.attn.query.weight"] = lin(n_state, n_state)
        t[f"{p}.attn.query.bias"] = nrm(n_state)
        t[f"{p}.attn.key.weight"] = lin(n_state, n_state)
        t[f"{p}.attn.value.weight"] = lin(n_state, n_state)
        t[f"{p}.attn.value.bias"] = nrm(n_state)
        t[f"{p}.attn.out.weight"] = lin(n_state, n_state)
        t[f"{p}.attn.out.bias"] = nrm(n_state)
        t[f"{p}.mlp_ln.weight"] = nrm(n_state, mean=1.0)
        t[f"{p}.mlp_ln.bias"] = nrm(n_state)
        t[f"{p}.mlp.0.weight"] = lin(4 * n_state, n_state)
        t[f"{p}.mlp.0.bias"] = nrm(4 * n_state)
        t[f"{p}.mlp.2.weight"] = lin(n_state, 4 * n_state)
        t[f"{p}.mlp.2.bias"] = nrm(n_state)
    t["encoder.ln_post.weight"] = nrm(n_state, mean=1.0)
    t["encoder.ln_post.bias"] = nrm(n_state)
    return t


def encoder_mel(n_windows: int, n_mels: int, n_frames: int, seed: int) -> np.ndarray:
    """Log-mel input of BASELINE config 3: N(-0.5, 0.3) clamped to [-1.5, 1.5]."""
    x = normal(seed, n_windows * n_mels * n_frames, -0.5, 0.3)
    return np.clip(x, -1.5, 1.5).astype(np.float32).reshape(n_windows, n_mels, n_frames)


def decoder_tensors(n_vocab: int, n_ctx: int, n_state: int, n_layer: int, dtype: int, seed: int,
                    reuse_layers: bool = False, gen_device=None) -> dict:
    """Random-init whisper decoder tensors by their whisper.cpp names
    (decoder.rs:36-321), same conventions as :func:`encoder_tensors`; the
    token embedding (also the tied logits matrix) is quantized like the
    block linears; learned positions ~ N(0, 0.02)."""
    t = {}
    ctr = [seed * 1000 + 500]

    def nrm(*shape, std=0.02, mean=0.0):
        ctr[0] += 1
        return normal(ctr[0], int(np.prod(shape)), mean, std).reshape(shape)

    def lin(n, k):
        ctr[0] += 1
        if dtype == Q5_1:
            return (dtype, quantize_q5_1(normal(ctr[0], n * k, 0.0, 0.02)), n, k)
        if dtype == Q8_0:
            return (dtype, quantize_q8_0(normal(ctr[0], n * k, 0.0, 0.02)), n, k)
        if gen_device is not None:
            raw = random_blocks_torch(dtype, n, k, ctr[0], *MODEL_CODE_SCALES[dtype], device=gen_device)
            return (dtype, raw.cpu().numpy(), n, k)
        return (dtype, random_blocks(dtype, n, k, ctr[0], *MODEL_CODE_SCALES[dtype]), n, k)

    t["decoder.token_embedding.weight"] = lin(n_vocab, n_state)
    t["decoder.positional_embedding"] = nrm(n_ctx, n_state)
    for l in range(n_layer):
        p = f"decoder.blocks.{l}"
        if reuse_layers and l > 0:
            for key in [x for x in t if x.startswith("decoder.blocks.0.")]:
                t[key.replace("decoder.blocks.0.", f"{p}.", 1)] = t[key]
            continue
        for ln in ("attn_ln", "cross_attn_ln", "mlp_ln"):
            t[f"{p}.{ln}.weight"] = nrm(n_state, mean=1.0)
            t[f"{p}.{ln}.bias"] = nrm(n_state)
        for a in ("attn", "cross_attn"):
            t[f"{p}.{a}.query.weight"] = lin(n_state, n_state)
            t[f"{p}.{a}.query.bias"] = nrm(n_state)
            t[f"{p}.{a}.key.weight"] = lin(n_state, n_state)
            t[f"{p}.{a}.value.weight"] = lin(n_state, n_state)
            t[f"{p}.{a}.value.bias"] = nrm(n_state)
            t[f"{p}.{a}.out.weight"] = lin(n_state, n_state)
            t[f"{p}.{a}.out.bias"] = nrm(n_state)
        t[f"{p}.mlp.0.weight"] = lin(4 * n_state, n_state)
        t[f"{p}.mlp.0.bias"] = nrm(4 * n_state)
        t[f"{p}.mlp.2.weight"] = lin(n_state, 4 * n_state)
        t[f"{p}.mlp.2.bias"] = nrm(n_state)
    t["decoder.ln.weight"] = nrm(n_state, mean=1.0)
    t["decoder.ln.bias"] = nrm(n_state)
    return t
