"""Writers of whisper model files for the loader tests (test helpers only).

* ``ggml_bin``  the legacy ggml container as rusty_whisper reads it
  (src/model.rs:145-275) and as its tests build it (src/model.rs:294-412):
  magic, 11 i32 hyper-parameters, the mel filterbank, the vocabulary, then
  tensors (n_dims, name length, dtype, ggml dims fastest first, name,
  payload) until the end of the file.
* ``gguf``      GGUF v3 as ``gguf::write`` lays it out (src/gguf.rs:288-420):
  general.architecture, general.alignment (32), the 11 ``whisper.*``
  hyper-parameters as i32, ``tokenizer.ggml.tokens``; tensor descriptors
  with the mel filters first as ``whisper.mel_filters`` then the tensors in
  sorted name order, offsets aligned to 32, data section aligned to 32.
"""
from __future__ import annotations

import struct

import numpy as np

GGML_MAGIC = 0x67676D6C
GGUF_MAGIC = 0x46554747
ALIGN = 32
N_FREQS = 201   # n_fft 400 / 2 + 1 (audio.rs)
HPARAM_KEYS = ("whisper.n_vocab", "whisper.n_audio_ctx", "whisper.n_audio_state", "whisper.n_audio_head",
               "whisper.n_audio_layer", "whisper.n_text_ctx", "whisper.n_text_state", "whisper.n_text_head",
               "whisper.n_text_layer", "whisper.n_mels", "whisper.ftype")


def _i32(v):
    return struct.pack("<i", int(v))


def ggml_bin(hparams, mel=(0, 0, ()), tokens=(), tensors=()):
    """``tensors``: (name: bytes, dtype, ggml dims fastest first, payload)."""
    b = bytearray(_i32(GGML_MAGIC - (1 << 32) if GGML_MAGIC >= 1 << 31 else GGML_MAGIC))
    for v in hparams:
        b += _i32(v)
    n_mel, n_bins, vals = mel
    b += _i32(n_mel) + _i32(n_bins)
    b += np.asarray(vals, np.float32).tobytes()
    b += _i32(len(tokens))
    for t in tokens:
        b += _i32(len(t)) + bytes(t)
    for name, dtype, ne, payload in tensors:
        b += _i32(len(ne)) + _i32(len(name)) + _i32(dtype)
        for d in ne:
            b += _i32(d)
        b += bytes(name) + bytes(payload)
    return bytes(b)


def _str(s: bytes) -> bytes:
    return struct.pack("<Q", len(s)) + bytes(s)


def gguf(hparams, mel_filters, vocab, tensors, arch=b"whisper", version=3):
    """``tensors``: {name: (dtype, row-major shape, payload bytes)};
    ``mel_filters``: f32 [n_mels, N_FREQS] (may be empty)."""
    mel = np.asarray(mel_filters, np.float32)
    has_filters = mel.size > 0
    names = sorted(tensors)
    out = bytearray(struct.pack("<IIQQ", GGUF_MAGIC, version, len(names) + has_filters, 3 + len(HPARAM_KEYS)))
    out += _str(b"general.architecture") + struct.pack("<I", 8) + _str(arch)
    out += _str(b"general.alignment") + struct.pack("<II", 4, ALIGN)
    for key, v in zip(HPARAM_KEYS, hparams):
        out += _str(key.encode()) + struct.pack("<Ii", 5, int(v))
    out += _str(b"tokenizer.ggml.tokens") + struct.pack("<IIQ", 9, 8, len(vocab))
    for t in vocab:
        out += _str(bytes(t))
    described = []
    if has_filters:
        described.append((b"whisper.mel_filters", list(mel.shape), 0, mel.tobytes()))
    for name in names:
        dt, shape, payload = tensors[name]
        described.append((name.encode(), list(shape), dt, bytes(payload)))
    offset = 0
    placed = []
    for name, shape, dt, payload in described:
        out += _str(name) + struct.pack("<I", len(shape))
        for d in reversed(shape):
            out += struct.pack("<Q", d)
        out += struct.pack("<IQ", dt, offset)
        placed.append((offset, payload))
        offset = (offset + len(payload) + ALIGN - 1) // ALIGN * ALIGN
    out += b"\0" * ((-len(out)) % ALIGN)
    data_start = len(out)
    for off, payload in placed:
        out += b"\0" * (data_start + off - len(out))
        out += payload
    return bytes(out)


def sample_gguf_model():
    """gguf.rs:57-99's sample model: a dense bias, a Q8_0 [2, 32] matrix
    with d = 1 and codes row+1, 2 x N_FREQS filters, 4 byte-level tokens."""
    hp = (4, 10, 8, 2, 1, 6, 8, 2, 1, 2, 1)
    raw = b"".join(struct.pack("<H", 0x3C00) + bytes([row + 1] * 32) for row in range(2))
    tensors = {
        "encoder.conv1.bias": (0, [3], np.asarray([1.0, -2.0, 0.5], np.float32).tobytes()),
        "decoder.token_embedding.weight": (8, [2, 32], raw),
    }
    mel = (np.arange(2 * N_FREQS, dtype=np.float32) * 0.5).reshape(2, N_FREQS)
    vocab = [b"a", b"bc", b"", b"\xff\xfe"]
    return hp, mel, vocab, tensors
