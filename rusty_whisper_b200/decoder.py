"""The KV-cached Whisper decoder on the GPU (mirror of the reference's
``decoder::Decoder``, src/decoder.rs:36-321, over the C ABI ``rwq_decoder_*``).

    dec = Decoder(n_vocab, n_text_ctx, n_state, n_head, n_layer, tensors)
    dec.begin(enc_out, stream_window)     # Decoder::new for every stream
    logits = dec.step(tokens)             # forward(&[token]) for every stream
    best = dec.step(tokens, want="best", limit=eot)   # greedy choice on the device

Streams step in lockstep; streams that decode the same window (beams)
share its cross-attention K/V.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .quant import _ptr, _stream_ptr, _torch


class Decoder:
    def __init__(self, n_vocab: int, n_ctx: int, n_state: int, n_head: int, n_layer: int, tensors: dict | None = None,
                 device: int | None = None):
        torch = _torch()
        self.device = torch.cuda.current_device() if device is None else device
        self.shape = (n_vocab, n_ctx, n_state, n_head, n_layer)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().rwq_decoder_new(n_vocab, n_ctx, n_state, n_head, n_layer, ctypes.byref(h)))
        self._h = h
        self.n_streams = 0
        for name, t in (tensors or {}).items():
            self.set(name, t)

    def set(self, name: str, t) -> None:
        torch = _torch()
        with torch.cuda.device(self.device):
            if isinstance(t, tuple):
                dtype, raw, n, k = t
                raw = np.ascontiguousarray(raw, np.uint8)
                _lib.check(_lib.lib().rwq_decoder_set_quant(self._h, name.encode(), dtype,
                                                            raw.ctypes.data_as(ctypes.c_void_p), raw.nbytes, n, k))
            else:
                a = np.ascontiguousarray(t, np.float32).ravel()
                _lib.check(_lib.lib().rwq_decoder_set_dense(self._h, name.encode(), a.ctypes.data_as(ctypes.c_void_p),
                                                            a.size))

    def begin(self, enc_out, stream_window=None) -> None:
        """enc_out: CUDA f32 [W, n_audio, n_state]; stream_window: host
        sequence of window ids, one per stream (default: stream i -> window i)."""
        torch = _torch()
        if enc_out.dim() == 2:
            enc_out = enc_out.unsqueeze(0)
        enc_out = enc_out.contiguous()
        self._enc = enc_out
        W, T = enc_out.shape[0], enc_out.shape[1]
        if stream_window is None:
            sw = None
            S = W
        else:
            self._sw = np.ascontiguousarray(stream_window, np.int32)
            sw = self._sw.ctypes.data_as(ctypes.c_void_p)
            S = self._sw.size
        _lib.check(_lib.lib().rwq_decoder_begin(self._h, _ptr(enc_out), W, T, sw, S,
                                                ctypes.c_void_p(_stream_ptr(enc_out.device))))
        self.n_streams = S
        self._tok = torch.empty(S, dtype=torch.int32, device=enc_out.device)

    def step(self, tokens, want: str = "logits", limit: int = -1, out=None):
        """tokens: one id per stream (CUDA int32 tensor, or a host sequence).
        want: "logits" -> [S, n_vocab] f32, "best" -> [S] int32 greedy ids,
        "none" -> a prompt position, nothing projected."""
        torch = _torch()
        if not torch.is_tensor(tokens) or not tokens.is_cuda:
            self._tok.copy_(torch.as_tensor(np.asarray(tokens, np.int32)))
            tokens = self._tok
        S = self.n_streams
        dev = tokens.device
        lg = best = None
        if want == "logits":
            lg = out if out is not None else torch.empty((S, self.shape[0]), device=dev, dtype=torch.float32)
        elif want == "best":
            best = out if out is not None else torch.empty(S, device=dev, dtype=torch.int32)
        _lib.check(_lib.lib().rwq_decoder_step(self._h, _ptr(tokens), _ptr(lg) if lg is not None else None,
                                               _ptr(best) if best is not None else None, limit,
                                               ctypes.c_void_p(_stream_ptr(dev))))
        return lg if want == "logits" else best

    def reset(self) -> None:
        _lib.check(_lib.lib().rwq_decoder_reset(self._h))

    @property
    def n_past(self) -> int:
        n = ctypes.c_int64()
        _lib.check(_lib.lib().rwq_decoder_n_past(self._h, ctypes.byref(n)))
        return n.value

    def free(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().rwq_decoder_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
