"""GPU log-mel (rwq_log_mel*, reference src/audio.rs:147-198) against the
C restatement of the reference in oracle/.  The FFT's rounding differs
from the reference's f32 recursion, so outputs agree to a tolerance, not
bitwise: the normalised values ((log10 + 4) / 4, O(1)) to TOL absolute."""
import numpy as np
import pytest

import oracle as o

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def au():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rusty_whisper_b200 import audio, quant
    quant.init(0)
    return audio


def _noise(seed, n, scale=0.1):
    return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)


def _speechlike(seed, n):
    """Band-limited noise bursts with silences (the shape of config 5's input)."""
    rng = np.random.default_rng(seed)
    x = np.convolve(rng.standard_normal(n), np.hanning(9) / 4.0, mode="same") * 0.1
    for _ in range(6):
        a = int(rng.integers(0, n - 8000))
        x[a:a + int(rng.integers(3200, 8000))] = 0.0
    return x.astype(np.float32)


@pytest.mark.parametrize("n_mels", (80, 128))
def test_single_window_matches_oracle(au, n_mels):
    fb = o.mel_filterbank(n_mels)
    for x in (_noise(1, 16000), _speechlike(2, 480000)):
        want = o.log_mel_spectrogram(x, fb, n_mels)
        got, nf = au.log_mel_spectrogram(x, fb, n_mels)
        assert nf == x.size // 160 and got.shape == want.shape
        assert np.max(np.abs(got - want)) < TOL


def test_batch_windows_normalised_independently(au):
    import torch
    fb = o.mel_filterbank(80)
    xs = np.stack([_speechlike(10, 480000), _noise(11, 480000, 0.5), _noise(12, 480000, 1e-3)])
    plan = au.LogMel(fb, 80)
    got = plan.batch(torch.from_numpy(xs).cuda()).cpu().numpy()
    for i in range(3):
        want = o.log_mel_spectrogram(xs[i], fb, 80)
        assert np.max(np.abs(got[i] - want)) < TOL
        assert got[i].max() - got[i].min() <= 2.0 + 1e-5


def test_pure_tone_and_edges(au):
    """audio.rs:250-274 on the GPU path, plus lengths that are not a
    multiple of the hop and the shortest accepted input."""
    fb = o.mel_filterbank(80)
    sr = 16000
    tone = np.sin(2.0 * np.float32(np.pi) * 1000.0 * np.arange(sr, dtype=np.float32) / sr).astype(np.float32)
    mel, nf = au.log_mel_spectrogram(tone, fb, 80)
    hot = int(np.argmax(mel[:, nf // 2]))
    assert abs(int(np.argmax(fb[hot])) * sr / 400 - 1000.0) < 100.0
    assert np.max(np.abs(mel - o.log_mel_spectrogram(tone, fb, 80))) < TOL
    for n in (201, 1000, 16001, 33333):
        x = _noise(n, n)
        got, nf = au.log_mel_spectrogram(x, fb, 80)
        assert nf == n // 160
        if nf:
            assert np.max(np.abs(got - o.log_mel_spectrogram(x, fb, 80))) < TOL
    with pytest.raises(ValueError):
        au.log_mel_spectrogram(np.zeros(200, np.float32), fb, 80)


def test_model_filters_through_plan(au):
    """Filters as a model file embeds them (rows with leading and trailing
    zeros, an all-zero row) give the oracle's result."""
    fb = o.mel_filterbank(80)
    fb[5] = 0.0
    x = _speechlike(20, 160000)
    got, _ = au.log_mel_spectrogram(x, fb, 80)
    assert np.max(np.abs(got - o.log_mel_spectrogram(x, fb, 80))) < TOL
