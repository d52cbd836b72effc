"""Model-file loader (rwq_model_*; reference src/model.rs:145-275 and
src/gguf.rs:156-300), parsing only: no GPU is touched.

The cases restate the reference's own loader tests:
``loads_synthetic_model`` and ``loads_quantized_tensor_from_synthetic_file``
(src/model.rs:294-412), ``rejects_bad_magic`` (model.rs:414-418),
``f16_conversion_reference_values`` (model.rs:282-291),
``round_trip_via_load_model`` and ``rejects_wrong_architecture``
(src/gguf.rs:101-138), plus the loader's error paths.
"""
import struct

import numpy as np
import pytest

from model_files import GGUF_MAGIC, ggml_bin, gguf, sample_gguf_model

pytest.importorskip("ctypes")


@pytest.fixture(scope="module")
def mdl():
    from rusty_whisper_b200 import model
    return model


def test_ggml_synthetic_model(mdl):
    """model.rs:294-345."""
    buf = ggml_bin(
        (3, 1500, 8, 2, 4, 448, 8, 2, 4, 2, 1),
        mel=(2, 3, (0.1, 0.2, 0.3, 0.4, 0.5, 0.6)),
        tokens=(b"hi", b"yo"),
        tensors=((b"w", 0, (2, 3), np.arange(1, 7, dtype=np.float32).tobytes()),
                 (b"b", 1, (2,), struct.pack("<HH", 0x3C00, 0xC000))))
    m = mdl.load_model(buf)
    assert m.hparams.n_vocab == 3
    assert m.hparams.model_type() == "tiny"
    assert not m.hparams.is_multilingual()
    assert np.array_equal(m.mel_filters, np.asarray([0.1, 0.2, 0.3, 0.4, 0.5, 0.6], np.float32))
    assert m.mel_shape == (2, 3)
    assert len(m.vocab) == 3 and m.vocab[1] == b"yo" and m.vocab[2] == b"[_extra_token_2]"
    w = m.tensors["w"]
    assert w.shape == (3, 2)   # dims flipped to row-major
    assert w.ravel().tolist() == [1., 2., 3., 4., 5., 6.]
    assert m.tensors["b"].tolist() == [1.0, -2.0]
    assert sorted(m.tensors) == ["b", "w"]


def test_ggml_quantized_tensor_kept_verbatim(mdl):
    """model.rs:380-412: a 2-D Q8_0 tensor stays quantized, blocks verbatim."""
    raw = struct.pack("<H", 0x3C00) + bytes([2] * 32)
    buf = ggml_bin((3, 1500, 8, 2, 4, 448, 8, 2, 4, 2, 8), tensors=((b"q", 8, (32, 1), raw),))
    m = mdl.load_model(buf)
    assert m.tensors.info("q") == (8, [1, 32])
    assert m.raw("q") == raw
    assert m.vocab == [b"[_extra_token_0]", b"[_extra_token_1]", b"[_extra_token_2]"]
    assert m.mel_filters.size == 0


def test_bad_magic(mdl):
    """model.rs:414-418."""
    with pytest.raises(ValueError, match="bad magic"):
        mdl.load_model(struct.pack("<I", 0xDEADBEEF))


def test_f16_widening_is_exact(mdl):
    """Every f16 bit pattern widens exactly (model.rs:68-86, :282-291)."""
    bits = np.arange(1 << 16, dtype=np.uint16)
    buf = ggml_bin((3, 1500, 8, 2, 4, 448, 8, 2, 4, 2, 1), tensors=((b"h", 1, (1 << 16,), bits.tobytes()),))
    got = mdl.load_model(buf).tensors["h"]
    want = bits.view(np.float16).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    m = mdl.load_model(ggml_bin((3,) * 11, tensors=((b"r", 1, (5,), struct.pack("<5H", 0, 0x3C00, 0xC000,
                                                                                   0x3555, 0x0001)),)))
    r = m.tensors["r"]
    assert r[:4].tolist() == [0.0, 1.0, -2.0, 0.333251953125]
    assert abs(r[4] - 5.9604645e-8) < 1e-12


def test_gguf_round_trip(mdl):
    """gguf.rs:101-127 through the magic-sniffing front door."""
    hp, mel, vocab, tensors = sample_gguf_model()
    buf = gguf(hp, mel, vocab, tensors)
    assert buf[:4] == b"GGUF"
    m = mdl.load_model(buf)
    assert tuple(getattr(m.hparams, f) for f in mdl._FIELDS) == hp
    assert m.vocab == vocab
    assert np.array_equal(m.mel_filters, mel.ravel())
    assert m.mel_shape == mel.shape
    assert len(m.tensors) == 2
    assert m.tensors["encoder.conv1.bias"].tolist() == [1.0, -2.0, 0.5]
    assert m.tensors.info("decoder.token_embedding.weight") == (8, [2, 32])
    assert m.raw("decoder.token_embedding.weight") == tensors["decoder.token_embedding.weight"][2]


def test_gguf_file_path(mdl, tmp_path):
    hp, mel, vocab, tensors = sample_gguf_model()
    p = tmp_path / "m.gguf"
    p.write_bytes(gguf(hp, mel, vocab, tensors))
    m = mdl.load_model(p)
    assert m.hparams.n_vocab == 4 and len(m.tensors) == 2


def test_gguf_rejects_wrong_architecture(mdl):
    """gguf.rs:129-138."""
    hp, mel, vocab, tensors = sample_gguf_model()
    buf = bytearray(gguf(hp, mel, vocab, tensors))
    pos = bytes(buf).index(b"whisper")
    buf[pos:pos + 7] = b"whooper"
    with pytest.raises(ValueError, match="architecture"):
        mdl.load_model(bytes(buf))


def test_gguf_errors(mdl):
    hp, mel, vocab, tensors = sample_gguf_model()
    good = gguf(hp, mel, vocab, tensors)
    with pytest.raises(ValueError, match="unsupported version"):
        mdl.load_model(gguf(hp, mel, vocab, tensors, version=4))
    for cut in (8, 30, 200, len(good) - 64):
        with pytest.raises(ValueError, match="truncated|out of bounds"):
            mdl.load_model(good[:cut])
    # a missing hyper-parameter key
    bad = good.replace(b"whisper.ftype", b"whisper.xtype")
    with pytest.raises(ValueError, match="missing metadata key whisper.ftype"):
        mdl.load_model(bad)
    # an unknown metadata value type (the alignment's type id 4 -> 99)
    i = good.index(b"general.alignment") + len(b"general.alignment")
    bad = good[:i] + struct.pack("<I", 99) + good[i + 4:]
    with pytest.raises(ValueError, match="unknown metadata type 99"):
        mdl.load_model(bad)
    # an unsupported tensor type
    bad = gguf(hp, mel, vocab, {"x": (13, [32], bytes(64))})
    with pytest.raises(ValueError, match="unsupported dtype 13"):
        mdl.load_model(bad)


def test_ggml_errors(mdl):
    hp = (3, 1500, 8, 2, 4, 448, 8, 2, 4, 2, 1)
    with pytest.raises(ValueError, match="not divisible by block size"):
        mdl.load_model(ggml_bin(hp, tensors=((b"q", 8, (31, 1), bytes(34)),)))
    with pytest.raises(ValueError, match="unsupported dtype 5"):
        mdl.load_model(ggml_bin(hp, tensors=((b"q", 5, (32, 1), bytes(34)),)))
    good = ggml_bin(hp, mel=(2, 3, range(6)), tokens=(b"a",),
                    tensors=((b"w", 0, (4,), np.ones(4, np.float32).tobytes()),))
    with pytest.raises(ValueError, match="truncated"):
        mdl.load_model(good[:-3])
    with pytest.raises(ValueError, match="truncated"):
        mdl.load_model(good[:50])
    # fewer than 4 bytes after the last tensor end the list, like an EOF
    m = mdl.load_model(good + b"\0\0")
    assert list(m.tensors) == ["w"]
    with pytest.raises(KeyError):
        m.tensors["nope"]


def test_gguf_magic_value():
    assert GGUF_MAGIC.to_bytes(4, "little") == b"GGUF"
