"""GPU decoder step against the oracle's restatement of the reference
decoder (decoder.rs:36-321), marked gpu.

Teacher-forced: every stream is fed the same token sequence on both sides
and the logits of every position are compared.  Bars: relative RMS error
<= 2e-2 per stream and position (int8 activations between layers, f16
attention inputs), and the device argmax equals numpy's choice on the
device logits under the reference's greedy rule."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

V, CTX, D, H, L, T_AUDIO = 512, 12, 256, 4, 2, 64


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


def _setup(dtype, n_win, stream_window, seed=4):
    import oracle
    from rusty_whisper_b200 import decoder, synth
    t = synth.decoder_tensors(V, CTX, D, L, dtype, seed)
    enc = synth.normal(seed + 50, n_win * T_AUDIO * D).reshape(n_win, T_AUDIO, D)
    gpu = decoder.Decoder(V, CTX, D, H, L, t)
    refs = []
    for w in stream_window:
        r = oracle.Decoder(V, CTX, D, H, L, t)
        r.begin(enc[w])
        refs.append(r)
    return gpu, refs, enc


@pytest.mark.parametrize("dtype,n_win,stream_window", [
    (7, 3, [0, 1, 2]),                       # greedy: one stream per window
    (6, 2, [0, 0, 0, 1, 1]),                 # beams sharing windows
    (2, 2, [0, 1, 0, 1, 0, 1, 0, 1, 0, 1]),  # 10 streams: the tensor-core GEMM path
])
def test_decoder_matches_oracle(torch_mod, dtype, n_win, stream_window):
    from rusty_whisper_b200 import synth
    gpu, refs, enc = _setup(dtype, n_win, stream_window)
    gpu.begin(torch_mod.from_numpy(enc).cuda(), stream_window)
    S = len(stream_window)
    toks = synth.randint(77 + dtype, S * 6, 0, V - 1).reshape(6, S)
    for p in range(6):
        got = gpu.step(torch_mod.from_numpy(toks[p].astype(np.int32)).cuda()).cpu().numpy()
        for i in range(S):
            ref = refs[i].forward([int(toks[p, i])])[0]
            assert _rel_rms(got[i], ref) <= 2e-2, (dtype, p, i, _rel_rms(got[i], ref))
    assert gpu.n_past == 6


def test_decoder_beam_groups_split_keys(torch_mod):
    """Streams sharing a window attend to its K/V as one group on the
    tensor-core kernel, a window with more than 8 streams as several
    groups, and enough encoder frames split the keys over several CTAs per
    (head, group).  Against the oracle, and bit-identical on a rerun (the
    splits are added in a fixed order whichever CTA finishes last)."""
    import oracle
    from rusty_whisper_b200 import decoder, synth
    T = 640
    sw = [0] * 5 + [1] * 9
    t = synth.decoder_tensors(V, CTX, D, L, 6, 11)
    enc = synth.normal(61, 2 * T * D).reshape(2, T, D)
    toks = synth.randint(19, len(sw) * 3, 0, V - 1).reshape(3, len(sw))
    outs = []
    for _ in range(2):
        gpu = decoder.Decoder(V, CTX, D, H, L, t)
        gpu.begin(torch_mod.from_numpy(enc).cuda(), sw)
        outs.append([gpu.step(torch_mod.from_numpy(toks[p].astype(np.int32)).cuda()).cpu() for p in range(3)])
    for a, b in zip(*outs):
        assert torch_mod.equal(a, b)
    for i in (0, 4, 5, 12, 13):
        r = oracle.Decoder(V, CTX, D, H, L, t)
        r.begin(enc[sw[i]])
        for p in range(3):
            ref = r.forward([int(toks[p, i])])[0]
            err = _rel_rms(outs[0][p].numpy()[i], ref)
            assert err <= 2e-2, (i, p, err)


def test_decoder_greedy_choice_and_prompt_positions(torch_mod):
    from rusty_whisper_b200 import synth
    gpu, refs, enc = _setup(7, 2, [0, 1])
    gpu.begin(torch_mod.from_numpy(enc).cuda())
    gpu.step([3, 4], want="none")                    # prompt positions: no projection
    gpu.step([5, 6], want="none")
    assert gpu.n_past == 2
    for limit in (-1, 300):
        g2, _, _ = _setup(7, 2, [0, 1])
        g2.begin(torch_mod.from_numpy(enc).cuda())
        g2.step([3, 4], want="none")
        lg = g2.step([5, 6]).cpu().numpy()
        g3, _, _ = _setup(7, 2, [0, 1])
        g3.begin(torch_mod.from_numpy(enc).cuda())
        g3.step([3, 4], want="none")
        best = g3.step([5, 6], want="best", limit=limit).cpu().numpy()
        for i in range(2):
            row = lg[i]
            if limit < 0:
                want = int(np.argmax(row))
            else:
                j = int(np.argmax(row[:limit]))
                want = j if row[j] > row[limit] else limit
            assert best[i] == want


def test_decoder_reset_and_errors(torch_mod):
    from rusty_whisper_b200 import decoder, synth
    gpu, _, enc = _setup(8, 1, [0])
    encd = torch_mod.from_numpy(enc).cuda()
    gpu.begin(encd)
    first = gpu.step([2]).cpu().numpy()
    gpu.step([4])
    gpu.reset()
    assert gpu.n_past == 0
    again = gpu.step([2]).cpu().numpy()
    assert np.array_equal(first, again)             # reset reproduces the first step exactly
    for _ in range(CTX - 1):
        gpu.step([1], want="none")
    with pytest.raises(ValueError):
        gpu.step([1])                               # context overflow (decoder.rs:115-120)
    d2 = decoder.Decoder(V, CTX, D, H, L)
    with pytest.raises(ValueError):
        d2.begin(encd)                              # tensors missing
    with pytest.raises(ValueError):
        gpu.begin(encd, [0, 3])                     # window 3 does not exist
