"""GPU encoder forward against the oracle's restatement of the reference
encoder (encoder.rs:48-234), marked gpu.

Bars:
  * attention (f16 tensor-core MMAs, f32 accumulation) against the f32
    reference multi_head_attention: |err| <= 5e-3 * max|ref| per window;
  * the whole encoder (int8 activations between layers, so a rounding
    difference upstream can move an activation code by one): relative RMS
    error <= 2e-2 per window and max |err| <= 0.25 on LayerNorm-scaled
    outputs, against the oracle encoder run on the same tensors;
  * batch composition: a window encodes the same alone or in a batch
    (within 1e-4 relative RMS: the tensor-core GEMMs' K splits may differ
    with the batch's row count);
  * the conv stem's conv1d on the tensor cores against the reference's f32
    conv1d.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rusty_whisper_b200 import quant
    quant.init(0)
    return torch


def _rel_rms(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.sqrt(np.mean((got - ref) ** 2)) / max(np.sqrt(np.mean(ref ** 2)), 1e-30))


@pytest.mark.parametrize("w,t,n_head", [(1, 37, 1), (2, 100, 4), (1, 1500, 2), (3, 64, 8)])
def test_attention_matches_reference_mha(torch_mod, w, t, n_head):
    import oracle
    from rusty_whisper_b200 import encoder, synth
    d = 64 * n_head
    q = synth.normal(1 + t, w * t * d).reshape(w, t, d)
    k = synth.normal(2 + t, w * t * d).reshape(w, t, d)
    v = synth.normal(3 + t, w * t * d).reshape(w, t, d)
    out = encoder.multi_head_attention(*(torch_mod.from_numpy(x).cuda() for x in (q, k, v)), n_head)
    got = out.cpu().numpy()
    for i in range(w):
        ref = oracle.mha(q[i], k[i], v[i], n_head)
        err = np.max(np.abs(got[i] - ref))
        assert err <= 5e-3 * np.max(np.abs(ref)), (i, err)


@pytest.mark.parametrize("w,in_ch,t,out_ch,stride", [(1, 80, 3000, 512, 1), (2, 512, 3000, 512, 2),
                                                     (1, 128, 200, 1280, 1), (3, 7, 33, 20, 2), (1, 3, 1, 5, 1)])
def test_conv1d_matches_reference(torch_mod, w, in_ch, t, out_ch, stride):
    """The encoder stem's conv1d (tensor.rs:335-370) on the hi|lo tensor-core
    GEMM against the reference's f32 conv: within 1e-5 of each output
    window's scale (f32-level: the two sums round differently by ~2e-6),
    and the 1e-3 rule (quant.rs:1365)."""
    import oracle
    from rusty_whisper_b200 import encoder, synth
    x = synth.normal(1 + t, w * in_ch * t, -0.5, 0.3).reshape(w, in_ch, t)
    wt = synth.normal(2 + in_ch, out_ch * in_ch * 3, 0.0, 0.02).reshape(out_ch, in_ch, 3)
    b = synth.normal(3 + out_ch, out_ch, 0.0, 0.02)
    got = encoder.conv1d(*(torch_mod.from_numpy(a).cuda() for a in (x, wt, b)), stride).cpu().numpy()
    for i in range(w):
        ref = oracle.conv1d(x[i], wt, b, stride).T
        assert got[i].shape == ref.shape
        err = np.abs(got[i].astype(np.float64) - ref)
        assert err.max() <= 1e-5 * np.abs(ref).max(), (i, err.max(), np.abs(ref).max())
        assert (err / np.maximum(np.abs(ref), 1.0)).max() < 1e-3


def _ln_inputs(m, k, seed):
    from rusty_whisper_b200 import synth
    x = synth.normal(seed, m * k, 0.3, 1.5).reshape(m, k)
    add = synth.normal(seed + 1, m * k, -0.1, 0.7).reshape(m, k)
    w = synth.normal(seed + 2, k, 1.0, 0.02)
    b = synth.normal(seed + 3, k, 0.0, 0.02)
    return x, add, w, b


@pytest.mark.parametrize("m,k", [(1, 512), (37, 384), (2500, 512), (2048, 1280), (3000, 2048), (4099, 128)])
def test_layer_norm_matches_reference(torch_mod, m, k):
    """The encoder's row transform (residual add + LayerNorm, tensor.rs:
    274-289, + the int8 quantizer, quant.rs:690-716) against the oracle:
    x + add bit-exact (one f32 add), the LayerNorm within 1e-5 of each
    row's scale (the row sums are added in another order), and the codes,
    scales and sums bit-exact against the oracle quantizer run on the
    kernel's own LayerNorm rows.  m >= 2048 runs the one-warp-per-row
    kernel, smaller m the four-warp one."""
    import oracle
    from rusty_whisper_b200 import encoder
    x, add, w, b = _ln_inputs(m, k, 40 + m + k)
    dx, da, dw, db = (torch_mod.from_numpy(a).cuda() for a in (x, add, w, b))
    y, (q, d, s) = encoder.layer_norm(dx, dw, db, add=da, quantize=True)
    xs = x + add
    assert np.array_equal(dx.cpu().numpy(), xs)
    got = y.cpu().numpy()
    ref = oracle.layernorm(xs, w, b)
    err = np.abs(got.astype(np.float64) - ref).max(axis=1)
    assert np.all(err <= 1e-5 * np.abs(ref).max(axis=1)), err.max()
    rq, rd, rs = oracle.quantize_acts_i8(got)
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(d.cpu().numpy(), rd)
    assert np.array_equal(s.cpu().numpy(), rs)
    y2 = encoder.layer_norm(torch_mod.from_numpy(xs).cuda(), dw, db)   # no add, no codes
    assert np.array_equal(y2.cpu().numpy(), got)


@pytest.mark.parametrize("k", [384, 512, 1280, 2048])
def test_layer_norm_rows_independent_of_batch(torch_mod, k):
    """A row's LayerNorm and codes are the same bits alone in a small batch
    (four warps per row) and inside an encoder-sized one (one warp per row):
    the decoder's stream-count invariance and the encoder's batch
    composition rest on it."""
    from rusty_whisper_b200 import encoder
    x, _, w, b = _ln_inputs(3000, k, 7 + k)
    dw, db = torch_mod.from_numpy(w).cuda(), torch_mod.from_numpy(b).cuda()
    big_y, big_q = encoder.layer_norm(torch_mod.from_numpy(x).cuda(), dw, db, quantize=True)
    for r0, r1 in [(0, 1), (5, 300), (2990, 3000)]:
        y, q = encoder.layer_norm(torch_mod.from_numpy(np.ascontiguousarray(x[r0:r1])).cuda(), dw, db,
                                  quantize=True)
        assert np.array_equal(y.cpu().numpy(), big_y[r0:r1].cpu().numpy()), (k, r0)
        for a, c in zip(q, big_q):
            assert np.array_equal(a.cpu().numpy(), c[r0:r1].cpu().numpy()), (k, r0)


def test_layer_norm_errors(torch_mod):
    from rusty_whisper_b200 import encoder
    x = torch_mod.zeros((4, 100), device="cuda")
    w = torch_mod.ones(100, device="cuda")
    with pytest.raises(ValueError):
        encoder.layer_norm(x, w, w)                          # k % 128 != 0
    x = torch_mod.zeros((4, 128), device="cuda")
    w = torch_mod.ones(128, device="cuda")
    with pytest.raises(ValueError):
        encoder.layer_norm(x, w, w, want_y=False)            # no output
    with pytest.raises(ValueError):
        encoder.layer_norm(x, w, w, add=torch_mod.zeros((3, 128), device="cuda"))
    with pytest.raises(TypeError):
        encoder.layer_norm(x.double(), w, w)
    y = encoder.layer_norm(torch_mod.zeros((0, 128), device="cuda"), w, w)
    assert y.shape == (0, 128)


def _encoder_pair(dtype, n_ctx=100, n_state=256, n_head=4, n_layer=2, n_mels=80, seed=5):
    import oracle
    from rusty_whisper_b200 import encoder, synth
    t = synth.encoder_tensors(n_mels, n_ctx, n_state, n_layer, dtype, seed)
    gpu = encoder.Encoder(n_mels, n_ctx, n_state, n_head, n_layer, t)
    cpu = oracle.Encoder(n_mels, n_ctx, n_state, n_head, n_layer, t)
    return gpu, cpu


@pytest.mark.parametrize("dtype", [7, 2, 8])
def test_encoder_matches_oracle(torch_mod, dtype):
    from rusty_whisper_b200 import synth
    gpu, cpu = _encoder_pair(dtype)
    mel = synth.encoder_mel(3, 80, 200, 11)
    got = gpu.encode(torch_mod.from_numpy(mel).cuda()).cpu().numpy()
    assert np.all(np.isfinite(got))
    for i in range(3):
        ref = cpu.encode(mel[i])
        assert _rel_rms(got[i], ref) <= 2e-2, (dtype, i, _rel_rms(got[i], ref))
        assert np.max(np.abs(got[i] - ref)) <= 0.25, (dtype, i, np.max(np.abs(got[i] - ref)))


def test_encoder_batch_composition_and_host_path(torch_mod):
    from rusty_whisper_b200 import synth
    gpu, _ = _encoder_pair(7, n_ctx=128, n_layer=1)
    mel = synth.encoder_mel(4, 80, 256, 12)
    batch = gpu.encode(torch_mod.from_numpy(mel).cuda()).cpu().numpy()
    one = gpu.encode(torch_mod.from_numpy(mel[2:3]).cuda()).cpu().numpy()
    assert _rel_rms(one[0], batch[2]) <= 1e-4
    host = gpu.encode_host(mel)
    assert _rel_rms(host, batch) <= 1e-4


def test_encoder_errors(torch_mod):
    from rusty_whisper_b200 import encoder, synth
    with pytest.raises(ValueError):
        encoder.Encoder(80, 16, 200, 4, 1)          # head dim 50
    e = encoder.Encoder(80, 16, 256, 4, 1)
    with pytest.raises(ValueError):
        e.set("encoder.conv1.bias", np.zeros(3, np.float32))        # wrong size
    with pytest.raises(ValueError):
        e.set("encoder.blocks.5.attn.key.weight", (7, b"", 256, 256))   # no such block
    with pytest.raises(ValueError):
        e.encode(torch_mod.zeros((1, 80, 32), device="cuda"))        # tensors missing
    t = synth.encoder_tensors(80, 16, 256, 1, 7, 3)
    for name, v in t.items():
        e.set(name, v)
    out = e.encode(torch_mod.zeros((2, 80, 32), device="cuda"))
    assert out.shape == (2, 16, 256) and bool(torch_mod.isfinite(out).all())
