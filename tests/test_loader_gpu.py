"""Model files into device weights (rwq_model_qtensor / rwq_model_dense):
weights read from a file compute exactly what weights made from the same
raw blocks compute, and quantized tensors of other ranks dequantize
bit-exactly (quant.rs `to_dense`, as model.rs:245-248 does at load)."""
import numpy as np
import pytest

from model_files import ggml_bin, gguf, sample_gguf_model

pytestmark = pytest.mark.gpu
TOL = 1e-3  # quant.rs:1365


@pytest.fixture(scope="module")
def rq():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rusty_whisper_b200 import quant
    quant.init(0)
    return quant


def test_gguf_sample_model_weights(rq):
    """gguf.rs:113-126: the Q8_0 matrix dequantizes to rows of 1 and 2."""
    from rusty_whisper_b200 import model
    hp, mel, vocab, tensors = sample_gguf_model()
    m = model.load_model(gguf(hp, mel, vocab, tensors))
    q = m.tensors["decoder.token_embedding.weight"]
    assert q.shape == [2, 32] and q.dtype == 8
    d = q.to_dense().cpu().numpy()
    assert (d[0] == 1.0).all() and (d[1] == 2.0).all()


@pytest.mark.parametrize("dtype", (2, 3, 6, 7, 8))
def test_file_weights_match_direct_weights(rq, orc, dtype):
    import torch
    from rusty_whisper_b200 import model, synth
    n, k, m_rows = 96, 256, 37
    raw = synth.random_blocks(dtype, n, k, 101 + dtype)
    hp = (51865, 1500, 512, 8, 6, 448, 512, 8, 6, 80, dtype)
    buf = gguf(hp, np.zeros((0,)), [b"x"], {"encoder.blocks.0.mlp.0.weight": (dtype, [n, k], raw.tobytes())})
    mf = model.load_model(buf)
    w_file = mf.tensors["encoder.blocks.0.mlp.0.weight"]
    w_direct = rq.QTensor([n, k], dtype, raw)
    a = torch.from_numpy(synth.normal(7, m_rows * k).reshape(m_rows, k)).cuda()
    for mm in (1, 5, m_rows):
        y_file = rq.matmul_t_q(a[:mm], w_file)
        y_direct = rq.matmul_t_q(a[:mm], w_direct)
        assert torch.equal(y_file, y_direct)
    ref = orc.matmul_t_q(a.cpu().numpy(), dtype, raw, n)
    got = rq.matmul_t_q(a, w_file).cpu().numpy()
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)) < TOL


@pytest.mark.parametrize("dtype", (2, 7, 8))
def test_rank1_quantized_tensor_dequantized_exactly(rq, orc, dtype):
    from rusty_whisper_b200 import model, synth
    k = 96
    raw = synth.random_blocks(dtype, 1, k, 55)
    buf = ggml_bin((3, 1500, 8, 2, 4, 448, 8, 2, 4, 2, dtype), tensors=((b"v", dtype, (k,), raw.tobytes()),))
    v = model.load_model(buf).tensors["v"]
    want = orc.to_dense(dtype, raw, 1, k).ravel()
    assert v.shape == (k,)
    assert np.array_equal(v.view(np.uint32), want.astype(np.float32).view(np.uint32))
