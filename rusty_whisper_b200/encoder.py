"""The Whisper encoder forward on the GPU (mirror of the reference's
``encoder::encode``, src/encoder.rs:180-234, over the C ABI ``rwq_encoder_*``).

    enc = Encoder(n_mels, n_ctx, n_state, n_head, n_layer, tensors)
    out = enc.encode(mel)        # mel [W, n_mels, 2*n_ctx] CUDA f32 -> [W, n_ctx, n_state]

``tensors`` maps whisper.cpp names to f32 arrays (dense tensors) or
``(dtype, raw_ggml_bytes, n, k)`` tuples (the six quantized linears of each
block), the layout :func:`rusty_whisper_b200.synth.encoder_tensors` makes.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .quant import _ptr, _stream_ptr, _torch


class Encoder:
    def __init__(self, n_mels: int, n_ctx: int, n_state: int, n_head: int, n_layer: int, tensors: dict | None = None,
                 device: int | None = None):
        torch = _torch()
        self.device = torch.cuda.current_device() if device is None else device
        self.shape = (n_mels, n_ctx, n_state, n_head, n_layer)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().rwq_encoder_new(n_mels, n_ctx, n_state, n_head, n_layer, ctypes.byref(h)))
        self._h = h
        for name, t in (tensors or {}).items():
            self.set(name, t)

    def set(self, name: str, t) -> None:
        torch = _torch()
        with torch.cuda.device(self.device):
            if isinstance(t, tuple):
                dtype, raw, n, k = t
                raw = np.ascontiguousarray(raw, np.uint8)
                _lib.check(_lib.lib().rwq_encoder_set_quant(self._h, name.encode(), dtype,
                                                            raw.ctypes.data_as(ctypes.c_void_p), raw.nbytes, n, k))
            else:
                a = np.ascontiguousarray(t, np.float32).ravel()
                _lib.check(_lib.lib().rwq_encoder_set_dense(self._h, name.encode(), a.ctypes.data_as(ctypes.c_void_p),
                                                            a.size))

    def encode(self, mel, out=None):
        """mel: CUDA f32 [W, n_mels, 2*n_ctx] -> [W, n_ctx, n_state] (async on
        the current stream)."""
        torch = _torch()
        n_mels, n_ctx, n_state = self.shape[:3]
        if mel.dim() == 2:
            mel = mel.unsqueeze(0)
        assert mel.is_cuda and mel.dtype == torch.float32 and tuple(mel.shape[1:]) == (n_mels, 2 * n_ctx)
        mel = mel.contiguous()
        if out is None:
            out = torch.empty((mel.shape[0], n_ctx, n_state), device=mel.device, dtype=torch.float32)
        _lib.check(_lib.lib().rwq_encoder_encode_dev(self._h, _ptr(mel), mel.shape[0], _ptr(out),
                                                     ctypes.c_void_p(_stream_ptr(mel.device))))
        return out

    def encode_host(self, mel: np.ndarray) -> np.ndarray:
        """Host buffers through rwq_encoder_encode (copies inside the call)."""
        n_mels, n_ctx, n_state = self.shape[:3]
        mel = np.ascontiguousarray(mel, np.float32).reshape(-1, n_mels, 2 * n_ctx)
        out = np.zeros((mel.shape[0], n_ctx, n_state), np.float32)
        _lib.check(_lib.lib().rwq_encoder_encode(self._h, mel.ctypes.data_as(ctypes.c_void_p), mel.shape[0],
                                                 out.ctypes.data_as(ctypes.c_void_p)))
        return out

    def free(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().rwq_encoder_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def multi_head_attention(q, k, v, n_head: int):
    """Non-causal attention over projected q, k, v (CUDA f32 [W, t, n_state]
    or [t, n_state]); encoder.rs:107-121."""
    torch = _torch()
    squeeze = q.dim() == 2
    q, k, v = (x.unsqueeze(0) if squeeze else x for x in (q, k, v))
    q, k, v = (x.contiguous() for x in (q, k, v))
    out = torch.empty_like(q)
    _lib.check(_lib.lib().rwq_attention_dev(_ptr(q), _ptr(k), _ptr(v), q.shape[0], q.shape[1], q.shape[2], n_head,
                                            _ptr(out), ctypes.c_void_p(_stream_ptr(q.device))))
    return out[0] if squeeze else out


def layer_norm(x, w, b, add=None, quantize: bool = False, want_y: bool = True):
    """tensor.rs:274-289 LayerNorm (eps 1e-5) over the rows of CUDA f32
    x [m, k] (k % 128 == 0), as the encoder and decoder run it: with
    ``add``, x is first replaced in place by x + add (the residual stream);
    with ``quantize`` the rows are also quantized by quant.rs:690-716.
    Returns ``y`` ([m, k] f32, None when not ``want_y``) and, with
    ``quantize``, ``(y, (q, d, sum))``."""
    torch = _torch()
    if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.float32 and x.dim() == 2
            and x.is_contiguous()):
        raise TypeError("layer_norm takes a contiguous 2-D CUDA float32 tensor")
    m, k = x.shape
    w, b = (t.contiguous() for t in (w, b))
    if add is not None:
        add = add.contiguous()
        if add.shape != x.shape:
            raise ValueError("add must have x's shape")
    out = torch.empty_like(x) if want_y else None
    q = d = s = None
    if quantize:
        q = torch.empty((m, k), dtype=torch.int8, device=x.device)
        d = torch.empty((m, k // 32), dtype=torch.float32, device=x.device)
        s = torch.empty((m, k // 32), dtype=torch.int32, device=x.device)
    def p(t):
        return _ptr(t) if t is not None else None

    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().rwq_layer_norm_dev(_ptr(x), p(add), _ptr(x) if add is not None else None, _ptr(w),
                                                 _ptr(b), m, k, p(out), p(q), p(d), p(s),
                                                 ctypes.c_void_p(_stream_ptr(x.device))))
    return (out, (q, d, s)) if quantize else out


def conv1d(x, w, b, stride: int):
    """tensor.rs:335-370 conv1d (kernel 3, padding 1) on the tensor cores:
    x CUDA f32 [n_win, in_ch, t] (or [in_ch, t]), w [out_ch, in_ch, 3], b
    [out_ch] or None -> [n_win, t_out, out_ch] (time-major: the
    reference's [out_ch, t_out] transposed)."""
    torch = _torch()
    squeeze = x.dim() == 2
    if squeeze:
        x = x.unsqueeze(0)
    x, w = x.contiguous(), w.contiguous()
    n_win, in_ch, t = x.shape
    out_ch = w.shape[0]
    if w.shape != (out_ch, in_ch, 3):
        raise ValueError("w must be [out_ch, in_ch, 3]")
    t_out = (t - 1) // stride + 1
    out = torch.empty((n_win, t_out, out_ch), device=x.device, dtype=torch.float32)
    bp = None
    if b is not None:
        b = b.contiguous()
        bp = _ptr(b)
    _lib.check(_lib.lib().rwq_conv1d_dev(_ptr(x), n_win, in_ch, t, _ptr(w), out_ch, bp, stride, _ptr(out),
                                         ctypes.c_void_p(_stream_ptr(x.device))))
    return out[0] if squeeze else out
