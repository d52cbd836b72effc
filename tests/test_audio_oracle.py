"""The log-mel restatement in oracle/ against the reference's own audio
tests (src/audio.rs:203-285), and the library's filterbank generator
against the oracle's (no GPU)."""
import ctypes

import numpy as np
import pytest

import oracle as o


def test_fft_matches_dft():
    """audio.rs:203-226: the 400-point FFT equals the naive DFT."""
    re = np.asarray([((i * 7 + 3) % 13) / 13.0 - 0.5 for i in range(400)], np.float32)
    im = np.zeros(400, np.float32)
    fr, fi = o.fft(re, im)
    dr, di = o.fft(re, im, naive=True)
    assert np.max(np.abs(fr - dr)) < 1e-2 and np.max(np.abs(fi - di)) < 1e-2


def test_hann_endpoints_and_symmetry():
    """audio.rs:228-236."""
    w = o.hann_window(400)
    assert abs(w[0]) < 1e-7 and abs(w[200] - 1.0) < 1e-6
    assert np.max(np.abs(w[1:] - w[1:][::-1])) < 1e-5


def test_filterbank_shape_and_coverage():
    """audio.rs:238-248."""
    fb = o.mel_filterbank(80)
    assert fb.shape == (80, 201)
    assert (fb >= 0).all() and (fb.max(axis=1) > 0).all()


def test_pure_tone_lands_in_matching_mel_band():
    """audio.rs:250-274."""
    fb = o.mel_filterbank(80)
    sr = 16000
    x = np.sin(2.0 * np.float32(np.pi) * 1000.0 * np.arange(sr, dtype=np.float32) / sr).astype(np.float32)
    mel = o.log_mel_spectrogram(x, fb, 80)
    assert mel.shape == (80, sr // 160)
    hot = int(np.argmax(mel[:, mel.shape[1] // 2]))
    peak_hz = int(np.argmax(fb[hot])) * sr / 400
    assert abs(peak_hz - 1000.0) < 100.0


def test_output_is_normalized():
    """audio.rs:276-284."""
    mel = o.log_mel_spectrogram(np.full(16000, 0.01, np.float32), o.mel_filterbank(80), 80)
    assert mel.max() - mel.min() <= 2.0 + 1e-5


@pytest.mark.parametrize("n_mels", (80, 128))
def test_library_filterbank_matches_oracle(n_mels):
    from rusty_whisper_b200 import _lib
    out = np.zeros((n_mels, 201), np.float32)
    _lib.check(_lib.lib().rwq_mel_filterbank(n_mels, 400, 16000, out.ctypes.data_as(ctypes.c_void_p)))
    want = o.mel_filterbank(n_mels)
    assert np.array_equal(out, want)
