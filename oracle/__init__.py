"""CPU oracle for rusty_whisper's quantized-matmul path (TEST INFRASTRUCTURE).

ctypes front-end over ``oracle/_build/librwq_oracle.so`` (built from
``oracle/rwq_oracle.cpp`` by ``oracle/build.sh``).  It restates the
reference's Rust (``src/quant.rs``, ``src/model.rs``, ``src/tensor.rs``)
and is pinned by the reference's own known-answer tests (see
``tests/test_oracle_pins.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may
import this package.  The product path (``rusty_whisper_b200``) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "librwq_oracle.so")
_lib = None

QK = 32
TIER_AUTO, TIER_VNNI, TIER_AVX2, TIER_F32 = 0, 1, 2, 3
TIER_NAMES = {1: "avx512-vnni", 2: "avx2", 3: "f32-fallback"}


def build() -> str:
    """Compile the oracle library (g++, -ffp-contract=off)."""
    subprocess.check_call(["sh", os.path.join(_HERE, "build.sh")])
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        i32, u32, sz, f32 = ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t, ctypes.c_float
        sig = {
            "orc_f16_to_f32": (f32, [ctypes.c_uint16]),
            "orc_f32_to_f16": (ctypes.c_uint16, [f32]),
            "orc_block_bytes": (i32, [i32]),
            "orc_has_avx2": (i32, []),
            "orc_has_vnni": (i32, []),
            "orc_default_threads": (i32, []),
            "orc_dispatch_tier": (i32, []),
            "orc_unpack_block": (i32, [i32, P, P, P, P]),
            "orc_dequant_row_scalar": (i32, [i32, P, sz, P]),
            "orc_dequant_row_avx2": (i32, [i32, P, sz, P]),
            "orc_quantize_acts_i8": (i32, [P, i32, i32, P, P, P]),
            "orc_block_dots": (i32, [P, i32, i32, i32, P, i32, P]),
            "orc_int8_scalar_matmul": (i32, [P, i32, i32, i32, P, i32, P]),
            "orc_matmul_t_q": (i32, [P, i32, i32, i32, P, i32, P, i32, i32, i32]),
            "orc_matmul_t": (i32, [P, i32, i32, P, i32, P, i32]),
            "orc_to_dense": (i32, [i32, P, i32, i32, P]),
            "orc_test_matrix": (None, [i32, i32, u32, P]),
            "orc_rand_bytes": (None, [u32, sz, P]),
            "orc_quantize_q8_0": (None, [P, sz, P]),
            "orc_quantize_q5_1": (None, [P, sz, P]),
            "orc_qtensor_new": (P, [i32, P, i32, i32]),
            "orc_qtensor_free": (None, [P]),
            "orc_qtensor_matmul": (i32, [P, P, i32, P, i32, i32]),
            "orc_hann_window": (None, [i32, P]),
            "orc_fft": (i32, [P, P, i32, P, P, i32]),
            "orc_mel_filterbank": (None, [i32, i32, i32, P]),
            "orc_log_mel": (i32, [P, i32, P, i32, P, P, i32]),
            "orc_encoder_new": (P, [i32, i32, i32, i32, i32]),
            "orc_encoder_free": (None, [P]),
            "orc_encoder_set": (i32, [P, ctypes.c_char_p, P, sz, i32, P, i32, i32]),
            "orc_encode": (i32, [P, P, P, i32]),
            "orc_layernorm": (None, [P, sz, i32, P, P]),
            "orc_set_model_tier": (None, [i32]),
            "orc_set_attn_f16": (None, [i32]),
            "orc_round_f16": (ctypes.c_float, [ctypes.c_float]),
            "orc_gelu": (None, [P, sz]),
            "orc_mha": (i32, [P, i32, P, P, i32, i32, i32, i32, P, i32]),
            "orc_conv1d": (i32, [P, i32, i32, P, i32, i32, P, i32, P, i32]),
            "orc_decoder_new": (P, [i32, i32, i32, i32, i32]),
            "orc_decoder_free": (None, [P]),
            "orc_decoder_set": (i32, [P, ctypes.c_char_p, P, sz, i32, P, i32, i32]),
            "orc_decoder_begin": (i32, [P, P, i32, i32]),
            "orc_decoder_forward": (i32, [P, P, i32, P, i32]),
            "orc_decoder_reset": (None, [P]),
            "orc_decoder_n_past": (i32, [P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def _check(rc: int, what: str):
    if rc != 0:
        raise RuntimeError(f"oracle {what} failed with status {rc}")


# ------------------------------------------------------------------ scalars
def f16_to_f32(h: int) -> float:
    return lib().orc_f16_to_f32(h)


def f32_to_f16(x: float) -> int:
    return lib().orc_f32_to_f16(x)


def block_bytes(dtype: int) -> int:
    return lib().orc_block_bytes(dtype)


def dispatch_tier() -> int:
    return lib().orc_dispatch_tier()


def default_threads() -> int:
    return lib().orc_default_threads()


# ------------------------------------------------------------------ blocks
def unpack_block(dtype: int, block: bytes):
    b = np.frombuffer(bytes(block), dtype=np.uint8).copy()
    q = np.zeros(QK, np.int8)
    d = np.zeros(1, np.float32)
    m = np.zeros(1, np.float32)
    _check(lib().orc_unpack_block(dtype, _p(b), _p(q), _p(d), _p(m)), "unpack_block")
    return q, float(d[0]), float(m[0])


def dequant_row_scalar(dtype: int, raw: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw, np.uint8)
    nbl = raw.size // block_bytes(dtype)
    out = np.zeros(nbl * QK, np.float32)
    _check(lib().orc_dequant_row_scalar(dtype, _p(raw), nbl, _p(out)), "dequant_row_scalar")
    return out


def dequant_row_avx2(dtype: int, raw: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw, np.uint8)
    nbl = raw.size // block_bytes(dtype)
    out = np.zeros(nbl * QK, np.float32)
    _check(lib().orc_dequant_row_avx2(dtype, _p(raw), nbl, _p(out)), "dequant_row_avx2")
    return out


def to_dense(dtype: int, raw: np.ndarray, n: int, k: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, np.uint8)
    out = np.zeros((n, k), np.float32)
    _check(lib().orc_to_dense(dtype, _p(raw), n, k, _p(out)), "to_dense")
    return out


# ------------------------------------------------------------- activations
def quantize_acts_i8(a: np.ndarray):
    a = np.ascontiguousarray(a, np.float32)
    m, k = a.shape
    nb = k // QK
    q = np.zeros((m, k), np.int8)
    d = np.zeros((m, nb), np.float32)
    s = np.zeros((m, nb), np.int32)
    _check(lib().orc_quantize_acts_i8(_p(a), m, k, _p(q), _p(d), _p(s)), "quantize_acts_i8")
    return q, d, s


def block_dots(qa: np.ndarray, dtype: int, raw: np.ndarray, n: int) -> np.ndarray:
    qa = np.ascontiguousarray(qa, np.int8)
    raw = np.ascontiguousarray(raw, np.uint8)
    m, k = qa.shape
    S = np.zeros((m, n, k // QK), np.int32)
    _check(lib().orc_block_dots(_p(qa), m, k, dtype, _p(raw), n, _p(S)), "block_dots")
    return S


# ---------------------------------------------------------------- matmuls
def int8_scalar_matmul(a: np.ndarray, dtype: int, raw: np.ndarray, n: int) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    raw = np.ascontiguousarray(raw, np.uint8)
    m, k = a.shape
    out = np.zeros((m, n), np.float32)
    _check(lib().orc_int8_scalar_matmul(_p(a), m, k, dtype, _p(raw), n, _p(out)), "int8_scalar_matmul")
    return out


def matmul_t_q(a: np.ndarray, dtype: int, raw: np.ndarray, n: int, tier: int = TIER_AUTO,
               threads: int = 0, packed: bool = False) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    raw = np.ascontiguousarray(raw, np.uint8)
    m, k = a.shape
    out = np.zeros((m, n), np.float32)
    _check(lib().orc_matmul_t_q(_p(a), m, k, dtype, _p(raw), n, _p(out), tier, threads, int(packed)),
           "matmul_t_q")
    return out


def matmul_t(a: np.ndarray, b: np.ndarray, threads: int = 0) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    n = b.shape[0]
    out = np.zeros((m, n), np.float32)
    _check(lib().orc_matmul_t(_p(a), m, k, _p(b), n, _p(out), threads), "matmul_t")
    return out


class QTensor:
    """Persistent weight with the reference's call-count gated int8 cache."""

    def __init__(self, dtype: int, raw: np.ndarray, n: int, k: int):
        self._raw = np.ascontiguousarray(raw, np.uint8)
        self.dtype, self.n, self.k = dtype, n, k
        self._h = lib().orc_qtensor_new(dtype, _p(self._raw), n, k)
        if not self._h:
            raise ValueError("bad qtensor")

    def matmul(self, a: np.ndarray, tier: int = TIER_AUTO, threads: int = 0, out=None) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        if out is None:
            out = np.zeros((a.shape[0], self.n), np.float32)
        _check(lib().orc_qtensor_matmul(self._h, _p(a), a.shape[0], _p(out), tier, threads), "qtensor_matmul")
        return out

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_qtensor_free(self._h)
            self._h = None


# ------------------------------------------------------ reference test data
def test_matrix(n: int, k: int, seed: int) -> np.ndarray:
    out = np.zeros(n * k, np.float32)
    lib().orc_test_matrix(n, k, seed, _p(out))
    return out


def rand_bytes(seed: int, count: int) -> np.ndarray:
    out = np.zeros(count, np.uint8)
    lib().orc_rand_bytes(seed, count, _p(out))
    return out


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(x.size // QK * 34, np.uint8)
    lib().orc_quantize_q8_0(_p(x), x.size, _p(out))
    return out


def quantize_q5_1(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(x.size // QK * 24, np.uint8)
    lib().orc_quantize_q5_1(_p(x), x.size, _p(out))
    return out


# ---------------------------------------------------------------- log-mel
N_FFT, HOP_LENGTH, N_FREQS, SAMPLE_RATE = 400, 160, 201, 16000


def hann_window(n: int = N_FFT) -> np.ndarray:
    out = np.zeros(n, np.float32)
    lib().orc_hann_window(n, _p(out))
    return out


def fft(re: np.ndarray, im: np.ndarray, naive: bool = False):
    re = np.ascontiguousarray(re, np.float32)
    im = np.ascontiguousarray(im, np.float32)
    n = re.size
    o_re, o_im = np.zeros(n, np.float32), np.zeros(n, np.float32)
    _check(lib().orc_fft(_p(re), _p(im), n, _p(o_re), _p(o_im), int(naive)), "fft")
    return o_re, o_im


def mel_filterbank(n_mels: int = 80, n_fft: int = N_FFT, sample_rate: int = SAMPLE_RATE) -> np.ndarray:
    out = np.zeros((n_mels, n_fft // 2 + 1), np.float32)
    lib().orc_mel_filterbank(n_mels, n_fft, sample_rate, _p(out))
    return out


def log_mel_spectrogram(samples: np.ndarray, filters: np.ndarray, n_mels: int, threads: int = 0) -> np.ndarray:
    """audio.rs:147-198: [n_mels, n_samples // 160] f32."""
    samples = np.ascontiguousarray(samples, np.float32)
    filters = np.ascontiguousarray(filters, np.float32)
    n_frames = samples.size // HOP_LENGTH
    out = np.zeros((n_mels, n_frames), np.float32)
    nf = ctypes.c_int(0)
    _check(lib().orc_log_mel(_p(samples), samples.size, _p(filters), n_mels, _p(out), ctypes.byref(nf), threads),
           "log_mel")
    return out


# ---------------------------------------------------------------- encoder
def set_model_tier(tier: int) -> None:
    """Tier of every quantized linear in the Encoder/Decoder restatements:
    0 dispatched (default), 1 VNNI, 2 AVX2.  A test switch: the two x86
    tiers are both the reference, and their outputs' drift through
    requantized layers bounds what a faithful port can be held to."""
    lib().orc_set_model_tier(int(tier))


def set_attn_f16(on: bool) -> None:
    """Round the attention operands (q, k, v, unnormalised softmax weights)
    to f16 in the Encoder/Decoder restatements and ``mha``: a test switch
    measuring the effect of the GPU kernels' f16 attention operands."""
    lib().orc_set_attn_f16(1 if on else 0)


def round_f16(x: float) -> float:
    return float(lib().orc_round_f16(float(x)))


def layernorm(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """tensor.rs:274-289 over the last dimension (returns a copy)."""
    x = np.array(x, np.float32, order="C")
    w = np.ascontiguousarray(w, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    lib().orc_layernorm(_p(x), x.size // x.shape[-1], x.shape[-1], _p(w), _p(b))
    return x


def gelu(x: np.ndarray) -> np.ndarray:
    """tensor.rs:291-306 (tanh approximation; returns a copy)."""
    x = np.array(x, np.float32, order="C")
    lib().orc_gelu(_p(x), x.size)
    return x


def mha(q: np.ndarray, k: np.ndarray, v: np.ndarray, n_head: int, causal: bool = False,
        threads: int = 0) -> np.ndarray:
    """encoder.rs:107-121 multi_head_attention over projected [t, n_state]."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    out = np.zeros_like(q)
    _check(lib().orc_mha(_p(q), q.shape[0], _p(k), _p(v), k.shape[0], q.shape[1], n_head, int(causal), _p(out),
                         threads), "mha")
    return out


def conv1d(x: np.ndarray, w: np.ndarray, b: np.ndarray, stride: int, threads: int = 0) -> np.ndarray:
    """tensor.rs:335-370: x [in_ch, t], w [out_ch, in_ch, kernel]."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    in_ch, t = x.shape
    out_ch, _, kernel = w.shape
    t_out = (t + 2 * (kernel // 2) - kernel) // stride + 1
    out = np.zeros((out_ch, t_out), np.float32)
    _check(lib().orc_conv1d(_p(x), in_ch, t, _p(w), out_ch, kernel, _p(b), stride, _p(out), threads), "conv1d")
    return out


class Encoder:
    """encoder.rs:180-234 with every quantized linear on matmul_t_q.

    ``tensors`` maps whisper.cpp names to either an f32 array (dense) or a
    ``(dtype, raw_bytes, n, k)`` tuple (quantized linear)."""

    def __init__(self, n_mels: int, n_ctx: int, n_state: int, n_head: int, n_layer: int, tensors: dict):
        self.shape = (n_mels, n_ctx, n_state, n_head, n_layer)
        self._h = lib().orc_encoder_new(n_mels, n_ctx, n_state, n_head, n_layer)
        if not self._h:
            raise ValueError("bad encoder shape")
        self._keep = []
        for name, t in tensors.items():
            if isinstance(t, tuple):
                dtype, raw, n, k = t
                raw = np.ascontiguousarray(raw, np.uint8)
                self._keep.append(raw)
                rc = lib().orc_encoder_set(self._h, name.encode(), None, 0, dtype, _p(raw), n, k)
            else:
                a = np.ascontiguousarray(t, np.float32).ravel()
                self._keep.append(a)
                rc = lib().orc_encoder_set(self._h, name.encode(), _p(a), a.size, 0, None, 0, 0)
            _check(rc, f"encoder_set({name})")

    def encode(self, mel: np.ndarray, threads: int = 0) -> np.ndarray:
        n_mels, n_ctx, n_state = self.shape[:3]
        mel = np.ascontiguousarray(mel, np.float32)
        assert mel.shape == (n_mels, 2 * n_ctx)
        out = np.zeros((n_ctx, n_state), np.float32)
        _check(lib().orc_encode(self._h, _p(mel), _p(out), threads), "encode")
        return out

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_encoder_free(self._h)
            self._h = None


class Decoder:
    """decoder.rs:36-321: ``begin(enc_out)`` is ``Decoder::new`` (cross K/V
    of one window), ``forward(tokens)`` returns logits [n_tok, n_vocab]."""

    def __init__(self, n_vocab: int, n_ctx: int, n_state: int, n_head: int, n_layer: int, tensors: dict):
        self.shape = (n_vocab, n_ctx, n_state, n_head, n_layer)
        self._h = lib().orc_decoder_new(n_vocab, n_ctx, n_state, n_head, n_layer)
        if not self._h:
            raise ValueError("bad decoder shape")
        self._keep = []
        for name, t in tensors.items():
            if isinstance(t, tuple):
                dtype, raw, n, k = t
                raw = np.ascontiguousarray(raw, np.uint8)
                self._keep.append(raw)
                rc = lib().orc_decoder_set(self._h, name.encode(), None, 0, dtype, _p(raw), n, k)
            else:
                a = np.ascontiguousarray(t, np.float32).ravel()
                self._keep.append(a)
                rc = lib().orc_decoder_set(self._h, name.encode(), _p(a), a.size, 0, None, 0, 0)
            _check(rc, f"decoder_set({name})")

    def begin(self, enc_out: np.ndarray, threads: int = 0) -> None:
        e = np.ascontiguousarray(enc_out, np.float32)
        _check(lib().orc_decoder_begin(self._h, _p(e), e.shape[0], threads), "decoder_begin")

    def forward(self, tokens, threads: int = 0) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32).ravel()
        out = np.zeros((t.size, self.shape[0]), np.float32)
        _check(lib().orc_decoder_forward(self._h, _p(t), t.size, _p(out), threads), "decoder_forward")
        return out

    def reset(self) -> None:
        lib().orc_decoder_reset(self._h)

    @property
    def n_past(self) -> int:
        return lib().orc_decoder_n_past(self._h)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_decoder_free(self._h)
            self._h = None
