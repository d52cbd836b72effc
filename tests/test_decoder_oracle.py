"""The oracle's restatement of the reference decoder (decoder.rs:36-321),
pinned by the reference's own decoder tests (decoder.rs:432-530).  CPU."""
import numpy as np
import pytest

import oracle
from rusty_whisper_b200 import synth

V, CTX, D, H, L = 64, 8, 64, 1, 1


def _dec(dtype=8):
    t = synth.decoder_tensors(V, CTX, D, L, dtype, 3)
    dec = oracle.Decoder(V, CTX, D, H, L, t)
    dec.begin(synth.normal(9, 6 * D).reshape(6, D))
    return dec, t


def test_forward_logits_shape():
    """decoder.rs:432-440."""
    dec, _ = _dec()
    logits = dec.forward([0, 3])
    assert logits.shape == (2, V) and np.all(np.isfinite(logits))
    assert dec.n_past == 2


def test_kv_cached_incremental_matches_full_forward():
    """decoder.rs:442-463."""
    tokens = [1, 5, 2, 7]
    full, _ = _dec()
    last_full = full.forward(tokens)[3]
    inc, _ = _dec()
    for tk in tokens:
        last = inc.forward([tk])[0]
    assert np.max(np.abs(last - last_full)) < 1e-4


def test_reset_clears_self_cache_but_keeps_cross():
    """decoder.rs:465-479."""
    dec, _ = _dec()
    first = dec.forward([2])
    assert np.all(np.isfinite(dec.forward([4])))
    dec.reset()
    assert dec.n_past == 0
    assert np.max(np.abs(dec.forward([2]) - first)) < 1e-6


def test_context_overflow_is_an_error():
    """decoder.rs:523-530 (a status code here instead of a panic)."""
    dec, _ = _dec()
    dec.forward(list(range(CTX)))
    with pytest.raises(RuntimeError):
        dec.forward([4])
