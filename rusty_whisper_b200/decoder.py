"""The KV-cached Whisper decoder on the GPU (mirror of the reference's
``decoder::Decoder``, src/decoder.rs:36-321, over the C ABI ``rwq_decoder_*``).

    dec = Decoder(n_vocab, n_text_ctx, n_state, n_head, n_layer, tensors)
    dec.begin(enc_out, stream_window)     # Decoder::new for every stream
    logits = dec.step(tokens)             # forward(&[token]) for every stream
    best = dec.step(tokens, want="best", limit=eot)   # greedy choice on the device
    hidden = dec.step(tokens, want="hidden")          # forward_hidden
    logits = dec.project(hidden)                      # project_logits, stacked
    dec.fork(src)                          # Decoder::fork for a beam step

Streams step in lockstep; streams that decode the same window (beams)
share its cross-attention K/V.  ``BeamSearch`` runs the reference's beam
step (transcribe.rs:886-990) on the device.
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
        "hidden" -> [S, n_state] f32 final-layernormed states (no
        projection), "none" -> a prompt position, nothing projected."""
        torch = _torch()
        if not torch.is_tensor(tokens) or not tokens.is_cuda:
            self._tok.copy_(torch.as_tensor(np.asarray(tokens, np.int32)))
            tokens = self._tok
        S = self.n_streams
        dev = tokens.device
        lg = best = None
        if want == "hidden":
            hid = out if out is not None else torch.empty((S, self.shape[2]), device=dev, dtype=torch.float32)
            _lib.check(_lib.lib().rwq_decoder_step_hidden(self._h, _ptr(tokens), _ptr(hid),
                                                          ctypes.c_void_p(_stream_ptr(dev))))
            return hid
        if want == "logits":
            lg = out if out is not None else torch.empty((S, self.shape[0]), device=dev, dtype=torch.float32)
        elif want == "best":
            best = out if out is not None else torch.empty(S, device=dev, dtype=torch.int32)
        _lib.check(_lib.lib().rwq_decoder_step(self._h, _ptr(tokens), _ptr(lg) if lg is not None else None,
                                               _ptr(best) if best is not None else None, limit,
                                               ctypes.c_void_p(_stream_ptr(dev))))
        return lg if want == "logits" else best

    def project(self, hidden, out=None):
        """project_logits (decoder.rs:315-321) of stacked hidden rows
        [rows <= S, n_state] (CUDA f32) -> [rows, n_vocab]."""
        torch = _torch()
        hidden = hidden.contiguous()
        rows = hidden.shape[0]
        lg = out if out is not None else torch.empty((rows, self.shape[0]), device=hidden.device, dtype=torch.float32)
        _lib.check(_lib.lib().rwq_decoder_project(self._h, _ptr(hidden), rows, _ptr(lg),
                                                  ctypes.c_void_p(_stream_ptr(hidden.device))))
        return lg

    def fork(self, src) -> None:
        """Decoder::fork for a beam step: stream i continues stream src[i]'s
        history (CUDA int32 [S], same window; see rwq_decoder_fork)."""
        torch = _torch()
        if not torch.is_tensor(src) or not src.is_cuda:
            src = torch.as_tensor(np.asarray(src, np.int32)).cuda(self.device)
        src = src.contiguous()
        _lib.check(_lib.lib().rwq_decoder_fork(self._h, _ptr(src), ctypes.c_void_p(_stream_ptr(src.device))))

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


def beam_topk(logits, k: int, limit: int = -1):
    """log_softmax + top_k of each row (transcribe.rs:482-486, 672-685) on
    the device: (lp [rows, k] f32, id [rows, k] int32)."""
    torch = _torch()
    logits = logits.contiguous()
    rows, V = logits.shape
    lp = torch.empty((rows, k), device=logits.device, dtype=torch.float32)
    ids = torch.empty((rows, k), device=logits.device, dtype=torch.int32)
    _lib.check(_lib.lib().rwq_beam_topk(_ptr(logits), rows, V, limit, k, _ptr(lp), _ptr(ids),
                                        ctypes.c_void_p(_stream_ptr(logits.device))))
    return lp, ids


class BeamSearch:
    """The reference's beam step (transcribe.rs:886-990) for W windows of B
    beams on one Decoder, all on the device: per step the stacked logits of
    every beam, top-k per beam, the per-window ranking of the candidates
    (rwq_beam_select) and the cache fork, with no host round trip.  Ids
    >= ``limit`` are never chosen (``limit`` = end-of-text keeps every beam
    decoding; the finished-hypothesis bookkeeping is the caller's)."""

    def __init__(self, dec: Decoder, n_windows: int, beams: int, limit: int = -1):
        torch = _torch()
        self.dec, self.W, self.B, self.limit = dec, n_windows, beams, limit
        S = n_windows * beams
        dev = torch.device("cuda", dec.device)
        z = lambda dt: torch.zeros(S, device=dev, dtype=dt)   # noqa: E731
        self.sum, self.rank = z(torch.float32), z(torch.int32)
        self.src, self.tok, self.step_lp = z(torch.int32), z(torch.int32), z(torch.float32)
        self.sum_next, self.rank_next = z(torch.float32), z(torch.int32)
        self.lp = torch.empty((S, beams), device=dev, dtype=torch.float32)
        self.ids = torch.empty((S, beams), device=dev, dtype=torch.int32)
        self.logits = torch.empty((S, dec.shape[0]), device=dev, dtype=torch.float32)
        self.live = 1

    def step(self, tokens):
        """Feed `tokens` (one per stream), rank, fork; returns the next
        tokens (CUDA int32 [S]), also in ``self.tok``."""
        L = _lib.lib()
        st = ctypes.c_void_p(_stream_ptr(self.logits.device))
        self.dec.step(tokens, want="logits", out=self.logits)
        _lib.check(L.rwq_beam_topk(_ptr(self.logits), self.logits.shape[0], self.logits.shape[1], self.limit, self.B,
                                   _ptr(self.lp), _ptr(self.ids), st))
        first = self.live == 1
        _lib.check(L.rwq_beam_select(_ptr(self.lp), _ptr(self.ids), self.B, None if first else _ptr(self.sum),
                                     None if first else _ptr(self.rank), self.W, self.B, self.live, _ptr(self.src),
                                     _ptr(self.tok), _ptr(self.sum_next), _ptr(self.step_lp), _ptr(self.rank_next), st))
        self.dec.fork(self.src)
        self.sum, self.sum_next = self.sum_next, self.sum
        self.rank, self.rank_next = self.rank_next, self.rank
        self.live = self.B
        return self.tok
