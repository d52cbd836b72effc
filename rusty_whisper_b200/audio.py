"""Host-side mirror of rusty_whisper's audio front end (src/audio.rs) over
the GPU kernels of ``librwq.so``.

* constants ``SAMPLE_RATE``, ``N_FFT``, ``HOP_LENGTH``, ``N_MEL``,
  ``N_FREQS``, ``N_SAMPLES_30S``                    audio.rs:10-15, :132
* ``mel_filterbank(n_mels, n_fft, sample_rate)``    audio.rs:107-130
* ``pad_or_trim(samples, n)``                       audio.rs:136-140
* ``log_mel_spectrogram(samples, filters, n_mels)`` audio.rs:147-198,
  returning ``(mel [n_mels, n_frames], n_frames)`` like the reference
* ``LogMel(filters, n_mels)``: a reusable GPU plan; ``LogMel.batch`` runs
  many windows at once on torch's current stream.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

SAMPLE_RATE = 16_000
N_FFT = 400
HOP_LENGTH = 160
N_MEL = 80
N_FREQS = N_FFT // 2 + 1
N_SAMPLES_30S = 30 * SAMPLE_RATE


def mel_filterbank(n_mels: int = N_MEL, n_fft: int = N_FFT, sample_rate: int = SAMPLE_RATE) -> np.ndarray:
    out = np.zeros((n_mels, n_fft // 2 + 1), np.float32)
    _lib.check(_lib.lib().rwq_mel_filterbank(n_mels, n_fft, sample_rate, out.ctypes.data_as(ctypes.c_void_p)))
    return out


def pad_or_trim(samples, n: int = N_SAMPLES_30S) -> np.ndarray:
    s = np.asarray(samples, np.float32)[:n]
    return np.pad(s, (0, n - s.size)) if s.size < n else s.copy()


class LogMel:
    """A filterbank ([n_mels, 201] f32) prepared for the GPU."""

    def __init__(self, filters, n_mels: int):
        f = np.ascontiguousarray(filters, np.float32).reshape(-1)
        if f.size != n_mels * N_FREQS:
            raise ValueError("filterbank shape mismatch")
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().rwq_mel_new(f.ctypes.data_as(ctypes.c_void_p), n_mels, ctypes.byref(h)))
        self._h = h
        self.n_mels = n_mels

    def __call__(self, samples) -> np.ndarray:
        """One window (host array) -> [n_mels, n // 160] host array."""
        s = np.ascontiguousarray(samples, np.float32)
        out = np.empty((self.n_mels, s.size // HOP_LENGTH), np.float32)
        _lib.check(_lib.lib().rwq_log_mel(self._h, s.ctypes.data_as(ctypes.c_void_p), s.size,
                                          out.ctypes.data_as(ctypes.c_void_p)))
        return out

    def batch(self, windows, out=None):
        """CUDA float32 [n_windows, n_samples] -> [n_windows, n_mels, n_samples // 160]."""
        import torch
        if not (isinstance(windows, torch.Tensor) and windows.is_cuda and windows.dtype == torch.float32):
            raise ValueError("windows must be a CUDA float32 tensor")
        windows = windows.contiguous()
        nw, ns = windows.shape
        if out is None:
            out = torch.empty((nw, self.n_mels, ns // HOP_LENGTH), dtype=torch.float32, device=windows.device)
        with torch.cuda.device(windows.device):
            _lib.check(_lib.lib().rwq_log_mel_dev(self._h, ctypes.c_void_p(windows.data_ptr()), nw, ns,
                                                  ctypes.c_void_p(out.data_ptr()),
                                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
        return out

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                _lib.lib().rwq_mel_free(h)
            finally:
                self._h = None


def log_mel_spectrogram(samples, filters, n_mels: int):
    """audio.rs:147: ``(mel, n_frames)``, mel [n_mels, n_frames] row-major."""
    mel = LogMel(filters, n_mels)(samples)
    return mel, mel.shape[1]
