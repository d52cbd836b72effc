"""The oracle's restatement of the reference encoder (encoder.rs), pinned by
the reference's own encoder tests (encoder.rs:236-373), and the synthetic
model generator's Q5_1 quantizer pinned bit-for-bit against the oracle's
restatement of quant.rs:1088-1113.  CPU only."""
import numpy as np

import oracle
from rusty_whisper_b200 import synth


def _fill(shape, seed):
    """encoder.rs:243-253: LCG values in [-0.1, 0.1]."""
    n = int(np.prod(shape))
    state = (seed * 2654435761 + 1) & 0xFFFFFFFF
    out = np.empty(n, np.float32)
    for i in range(n):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(np.float32(state >> 8) / np.float32(1 << 24) * np.float32(0.2) - np.float32(0.1))
    return out.reshape(shape)


def _toy_tensors(dtype=8):
    """encoder.rs:257-307's toy model, with its 2-D linears stored as
    quantized blocks (the reference's toy keeps them dense; the quantized
    matmul is the path under test here).  n_state 4 is not a multiple of
    32, so the toy uses n_state = 32 with the same structure."""
    t = {}
    d, f = 32, 128
    seed = [0]

    def add(name, shape):
        seed[0] += 1
        t[name] = _fill(shape, seed[0])

    def addq(name, n, k):
        seed[0] += 1
        t[name] = (dtype, oracle.quantize_q8_0(_fill((n, k), seed[0])), n, k)

    add("encoder.conv1.weight", (d, 2, 3))
    add("encoder.conv1.bias", (d,))
    add("encoder.conv2.weight", (d, d, 3))
    add("encoder.conv2.bias", (d,))
    add("encoder.positional_embedding", (3, d))
    p = "encoder.blocks.0"
    add(f"{p}.attn_ln.weight", (d,))
    add(f"{p}.attn_ln.bias", (d,))
    addq(f"{p}.attn.query.weight", d, d)
    add(f"{p}.attn.query.bias", (d,))
    addq(f"{p}.attn.key.weight", d, d)
    addq(f"{p}.attn.value.weight", d, d)
    add(f"{p}.attn.value.bias", (d,))
    addq(f"{p}.attn.out.weight", d, d)
    add(f"{p}.attn.out.bias", (d,))
    add(f"{p}.mlp_ln.weight", (d,))
    add(f"{p}.mlp_ln.bias", (d,))
    addq(f"{p}.mlp.0.weight", f, d)
    add(f"{p}.mlp.0.bias", (f,))
    addq(f"{p}.mlp.2.weight", d, f)
    add(f"{p}.mlp.2.bias", (d,))
    add("encoder.ln_post.weight", (d,))
    add("encoder.ln_post.bias", (d,))
    return t


def test_encoder_output_shape_and_finiteness():
    """encoder.rs:309-319."""
    enc = oracle.Encoder(2, 3, 32, 2, 1, _toy_tensors())
    out = enc.encode(_fill((2, 6), 99))
    assert out.shape == (3, 32)
    assert np.all(np.isfinite(out))
    assert np.any(np.abs(out) > 1e-6)


def test_encoder_is_deterministic():
    """encoder.rs:321-326."""
    enc = oracle.Encoder(2, 3, 32, 2, 1, _toy_tensors())
    mel = _fill((2, 6), 99)
    assert np.array_equal(enc.encode(mel), enc.encode(mel))


def test_mha_single_head_hand_computed():
    """encoder.rs:328-345."""
    k = np.array([[1.0], [-1.0]], np.float32)
    v = np.array([[10.0], [20.0]], np.float32)
    out = oracle.mha(np.array([[0.0]], np.float32), k, v, 1)
    assert abs(out[0, 0] - 15.0) < 1e-4
    out = oracle.mha(np.array([[50.0]], np.float32), k, v, 1)
    assert abs(out[0, 0] - 10.0) < 1e-3


def test_mha_causal_mask_blocks_future():
    """encoder.rs:347-358."""
    k = np.array([[0.0], [100.0], [100.0]], np.float32)
    v = np.array([[7.0], [8.0], [9.0]], np.float32)
    q = np.ones((3, 1), np.float32)
    out = oracle.mha(q, k, v, 1, causal=True)
    assert abs(out[0, 0] - 7.0) < 1e-5
    assert out[2, 0] > 7.5


def test_mha_incremental_query_aligns_to_end():
    """encoder.rs:360-373."""
    k, v, qf = _fill((3, 4), 31), _fill((3, 4), 32), _fill((3, 4), 33)
    full = oracle.mha(qf, k, v, 2, causal=True)
    inc = oracle.mha(qf[2:3], k, v, 2, causal=True)
    assert np.max(np.abs(inc[0] - full[2])) < 1e-5


def test_layernorm_gelu_conv_basics():
    x = np.arange(8, dtype=np.float32).reshape(2, 4)
    y = oracle.layernorm(x, np.ones(4, np.float32), np.zeros(4, np.float32))
    assert np.allclose(y.mean(axis=1), 0, atol=1e-6) and np.allclose(y.std(axis=1), 1, atol=1e-3)
    g = oracle.gelu(np.array([0.0, 1.0, -1.0, 3.0], np.float32))
    assert g[0] == 0 and abs(g[1] - 0.8411920) < 1e-5 and abs(g[2] + 0.1588080) < 1e-5
    # conv1d with an identity centre tap reproduces its input (pad 1).
    w = np.zeros((2, 2, 3), np.float32)
    w[0, 0, 1] = w[1, 1, 1] = 1.0
    x = _fill((2, 7), 5)
    assert np.array_equal(oracle.conv1d(x, w, np.zeros(2, np.float32), 1), x)
    assert np.array_equal(oracle.conv1d(x, w, np.zeros(2, np.float32), 2), x[:, ::2])


def test_synth_q5_1_matches_reference_quantizer():
    """The generator's vectorised Q5_1 quantizer is byte-identical to the
    oracle's restatement of quant.rs:1088-1113."""
    for seed in (1, 2, 3):
        x = synth.normal(seed, 32 * 257, 0.0, 0.02)
        x[::97] = 0.0
        x[5 * 32:6 * 32] = 0.25          # a constant block: d = 0
        assert np.array_equal(synth.quantize_q5_1(x), oracle.quantize_q5_1(x))


def test_synth_q8_0_matches_reference_quantizer():
    """quant.rs:1071-1083, byte-identical to the oracle's restatement."""
    for seed in (4, 5):
        x = synth.normal(seed, 32 * 301, 0.0, 0.02)
        x[::89] = 0.0
        x[7 * 32:8 * 32] = 0.0           # an all-zero block: d = 0
        assert np.array_equal(synth.quantize_q8_0(x), oracle.quantize_q8_0(x))


def test_encoder_tensors_are_complete():
    t = synth.encoder_tensors(80, 16, 64, 2, 7, 1)
    enc = oracle.Encoder(80, 16, 64, 1, 2, t)
    out = enc.encode(synth.encoder_mel(1, 80, 32, 3)[0])
    assert out.shape == (16, 64) and np.all(np.isfinite(out))
