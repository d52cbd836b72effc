"""Beam search on the device (marked gpu): the split step, fork, top-k and
candidate ranking against the reference's semantics.

* split_forward_equals_combined (decoder.rs:481-495): forward_hidden +
  project_logits gives the logits of forward, and stacking rows projects
  them as one at a time would.  Here: the same bits.
* forked_decoder_branches_independently (decoder.rs:497-521): after a
  shared prefix, a fork's continuation equals a fresh decoder fed the
  whole sequence.  Here: the same bits, and the oracle within the decoder
  tests' bound.
* The device beam step (BeamSearch: rwq_beam_topk, rwq_beam_select,
  rwq_decoder_fork) against the reference's algorithm (transcribe.rs:
  886-990: log_softmax, top_k, scores sum + max(lp, -30), stable sort, the
  best B kept) run on the host over the device's own logits, and every
  beam's next logits against a fresh decoder fed that beam's tokens.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

V, CTX, D, H, L, T_AUDIO = 2000, 48, 256, 4, 2, 96


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


def _model(seed=23):
    from rusty_whisper_b200 import synth
    t = synth.decoder_tensors(V, CTX, D, L, 7, seed=seed)
    # scaled positions: a random model then picks different ids per step
    t["decoder.positional_embedding"] = (t["decoder.positional_embedding"] * np.float32(25.0)).astype(np.float32)
    return t


def _enc(n_win, seed=24):
    from rusty_whisper_b200 import synth
    return synth.normal(seed, n_win * T_AUDIO * D).reshape(n_win, T_AUDIO, D)


def test_split_forward_equals_combined(torch_mod):
    from rusty_whisper_b200 import decoder
    t, enc = _model(), torch_mod.from_numpy(_enc(2)).cuda()
    sw = [0, 1, 1]
    toks = [[1, 7, 9], [5, 5, 2]]
    a = decoder.Decoder(V, CTX, D, H, L, t)
    a.begin(enc, sw)
    b = decoder.Decoder(V, CTX, D, H, L, t)
    b.begin(enc, sw)
    for tk in toks:
        combined = a.step(tk)
        hidden = b.step(tk, want="hidden")
        split = b.project(hidden)
        assert torch_mod.equal(combined, split)
        for r in range(3):   # one row at a time: the same as stacked
            assert torch_mod.equal(b.project(hidden[r:r + 1]), split[r:r + 1])


def test_forked_decoder_branches_independently(torch_mod, orc):
    from rusty_whisper_b200 import decoder
    t, enc_np = _model(), _enc(1)
    enc = torch_mod.from_numpy(enc_np).cuda()
    a = decoder.Decoder(V, CTX, D, H, L, t)
    a.begin(enc, [0, 0])
    a.step([1, 3])
    a.step([5, 4])                  # stream 1 has its own prefix [3, 4] ...
    a.fork([0, 0])                  # ... until it forks from stream 0's [1, 5]
    got = a.step([2, 7]).cpu().numpy()
    fresh = decoder.Decoder(V, CTX, D, H, L, t)
    fresh.begin(enc, [0, 0])
    for tk in ([1, 1], [5, 5]):
        fresh.step(tk)
    want = fresh.step([2, 7]).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    for i, last in enumerate((2, 7)):
        ref = orc.Decoder(V, CTX, D, H, L, t)
        ref.begin(enc_np[0])
        ref.forward([1])
        ref.forward([5])
        assert _rel_rms(got[i], ref.forward([last])[0]) <= 2e-2
    # a source that is itself copied this step, or in another window, is ignored
    b = decoder.Decoder(V, CTX, D, H, L, t)
    b.begin(torch_mod.from_numpy(_enc(2)).cuda(), [0, 0, 1])
    b.step([1, 3, 6])
    b.fork([1, 0, 0])               # 0 <- 1 and 1 <- 0 (sources not kept), 2 <- 0 (other window)
    after = b.step([2, 2, 2]).cpu().numpy()
    c = decoder.Decoder(V, CTX, D, H, L, t)
    c.begin(torch_mod.from_numpy(_enc(2)).cuda(), [0, 0, 1])
    c.step([1, 3, 6])
    assert np.array_equal(after.view(np.uint32), c.step([2, 2, 2]).cpu().numpy().view(np.uint32))


def _log_softmax(row):
    """transcribe.rs:482-486 in f32."""
    row = row.astype(np.float32)
    mx = np.float32(np.max(row))
    lse = np.float32(mx + np.float32(np.log(np.sum(np.exp(row - mx, dtype=np.float32), dtype=np.float32))))
    return (row - lse).astype(np.float32)


def _top_k(lps, k):
    order = sorted(range(lps.size), key=lambda i: (-float(lps[i]), i))
    return [(float(lps[i]), i) for i in order[:k] if lps[i] > -np.inf]


def test_topk_matches_reference(torch_mod):
    from rusty_whisper_b200 import decoder, synth
    lg = synth.normal(5, 7 * 3001).reshape(7, 3001) * np.float32(4.0)
    lg[2, 100:] = -np.inf                          # fewer choosable ids than k beyond 100 masked
    lg[2, :97] = -np.inf
    for k, limit in ((5, -1), (8, 2990), (1, 50)):
        lp, ids = decoder.beam_topk(torch_mod.from_numpy(lg).cuda(), k, limit)
        lp, ids = lp.cpu().numpy(), ids.cpu().numpy()
        for r in range(7):
            row = lg[r, :limit] if limit >= 0 else lg[r]
            want = _top_k(_log_softmax(row), k)
            assert [int(i) for i in ids[r, :len(want)]] == [i for _, i in want], (k, r)
            assert np.allclose(lp[r, :len(want)], [v for v, _ in want], rtol=0, atol=2e-5)
            assert all(ids[r, len(want):] == -1) and all(np.isneginf(lp[r, len(want):]))


def test_topk_vocab_rows_chunk_ties(torch_mod):
    """Rows of a whisper vocabulary (split over the kernel's chunks), with
    the maximum repeated across chunk boundaries: equal values rank by the
    smaller id, as the reference's stable sort does."""
    from rusty_whisper_b200 import decoder, synth
    n_v = 51865
    lg = synth.normal(6, 5 * n_v).reshape(5, n_v) * np.float32(3.0)
    lg[1, ::997] = np.float32(40.0)          # 53 equal maxima spread over every chunk
    lg[3, 6400:6560] = np.float32(30.0)      # a run of ties straddling a chunk boundary
    lg[4, :] = np.float32(1.0)               # all equal
    for k, limit in ((5, 50257), (8, -1), (3, 6500)):
        lp, ids = decoder.beam_topk(torch_mod.from_numpy(lg).cuda(), k, limit)
        lp, ids = lp.cpu().numpy(), ids.cpu().numpy()
        for r in range(5):
            row = lg[r, :limit] if limit >= 0 else lg[r]
            want = _top_k(_log_softmax(row), k)
            assert [int(i) for i in ids[r, :len(want)]] == [i for _, i in want], (k, r)
            assert np.allclose(lp[r, :len(want)], [v for v, _ in want], rtol=0, atol=2e-5)


def _select_ref(lp, ids, k, sum_in, rank_in, W, B, n_live):
    """transcribe.rs:890-925 for each window (candidates of the live beams
    in rank order, each beam's in top-k order, scored sum + max(lp, -30),
    stable sort, best B kept), with the slot rule of rwq_beam_select: the
    best survivor of each parent keeps the parent's slot, the others take
    the slots no survivor descends from in slot order, and slots left over
    repeat the best survivor ranked last."""
    S = W * B
    src, tok = np.zeros(S, np.int64), np.zeros(S, np.int64)
    sm, stp, rk = np.zeros(S, np.float32), np.zeros(S, np.float32), np.zeros(S, np.int64)
    for w in range(W):
        s0 = w * B
        order = []
        for r in range(n_live):
            for b in range(B):
                if (rank_in[s0 + b] if rank_in is not None else b) == r:
                    order.append(b)
                    break
        cands = []
        for b in order:
            for j in range(k):
                i = int(ids[s0 + b, j])
                if i < 0:
                    continue
                st = np.float32(max(np.float32(lp[s0 + b, j]), np.float32(-30.0)))
                sc = np.float32(np.float32(sum_in[s0 + b] if sum_in is not None else 0.0) + st)
                cands.append((sc, st, b, i))
        cands.sort(key=lambda c: -float(c[0]))
        sel = cands[:B]
        parents = {c[2] for c in sel}
        used, slots = set(), []
        for c in sel:
            if c[2] not in used:
                slots.append(c[2])
                used.add(c[2])
            else:
                slots.append(None)
        free = [b for b in range(B) if b not in parents]
        for n, c in enumerate(sel):
            if slots[n] is None:
                slots[n] = free.pop(0)
                used.add(slots[n])
        for n, (c, b) in enumerate(zip(sel, slots)):
            src[s0 + b], tok[s0 + b], sm[s0 + b], stp[s0 + b], rk[s0 + b] = s0 + c[2], c[3], c[0], c[1], n
        extra = len(sel)
        for b in range(B):
            if b in used:
                continue
            if sel:
                c = sel[0]
                src[s0 + b], tok[s0 + b], sm[s0 + b], stp[s0 + b] = s0 + c[2], c[3], c[0], c[1]
            else:
                src[s0 + b], tok[s0 + b], sm[s0 + b], stp[s0 + b] = s0 + b, 0, -np.inf, -np.inf
            rk[s0 + b] = extra
            extra += 1
    return src, tok, sm, stp, rk


@pytest.mark.parametrize("W,B,k,n_live", [(16, 5, 5, 5), (3, 8, 8, 8), (4, 3, 1, 2), (5, 5, 5, 1), (2, 6, 4, 6)])
def test_beam_select_matches_reference(torch_mod, W, B, k, n_live):
    """rwq_beam_select against the reference's ranking on crafted
    candidates: tied scores (stable order), invalid ids (-1: fewer
    candidates than beams), permuted beam ranks, -30 clamping."""
    import ctypes
    from rusty_whisper_b200 import _lib
    torch = torch_mod
    rng = np.random.default_rng(W * 100 + B * 10 + k)
    S = W * B
    lp = np.round(rng.normal(-3, 2, (S, k)) * 4) / np.float32(4)          # many exact ties
    lp[rng.random((S, k)) < 0.1] = np.float32(-45.0)                       # clamped to -30
    ids = rng.integers(0, 50000, (S, k)).astype(np.int32)
    ids[rng.random((S, k)) < 0.15] = -1
    if W > 2:
        ids[2 * B:3 * B] = -1                                              # a window with no candidate
    sum_in = (np.round(rng.normal(-10, 3, S) * 2) / 2).astype(np.float32)
    rank_in = np.concatenate([rng.permutation(B) for _ in range(W)]).astype(np.int32)
    lp = np.ascontiguousarray(lp.astype(np.float32))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()     # noqa: E731
    g_lp, g_id, g_sum, g_rank = dev(lp), dev(ids), dev(sum_in), dev(rank_in)
    outs = [torch.zeros(S, dtype=dt, device="cuda") for dt in (torch.int32, torch.int32, torch.float32,
                                                              torch.float32, torch.int32)]
    p = lambda t: ctypes.c_void_p(t.data_ptr())                            # noqa: E731
    _lib.check(_lib.lib().rwq_beam_select(p(g_lp), p(g_id), k, p(g_sum), p(g_rank), W, B, n_live,
                                          *[p(o) for o in outs], ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    got = [o.cpu().numpy() for o in outs]
    want = _select_ref(lp, ids, k, sum_in, rank_in, W, B, n_live)
    for g, wv, name in zip(got, want, ("src", "tok", "sum", "step_lp", "rank")):
        assert np.array_equal(g.astype(np.float64), np.asarray(wv, np.float64)), name


def test_beam_search_device_matches_reference_algorithm(torch_mod):
    from rusty_whisper_b200 import decoder
    W, B, steps, limit = 2, 3, 12, 1990
    t = _model()
    enc = torch_mod.from_numpy(_enc(W)).cuda()
    dec = decoder.Decoder(V, CTX, D, H, L, t)
    sw = [w for w in range(W) for _ in range(B)]
    dec.begin(enc, sw)
    prompt = [1990, 1991, 1992, 1993]
    for tk in prompt[:-1]:
        dec.step([tk] * (W * B), want="none")
    bs = decoder.BeamSearch(dec, W, B, limit=limit)
    tok = torch_mod.tensor([prompt[-1]] * (W * B), dtype=torch_mod.int32, device="cuda")
    # host mirror of the reference's beams: per window a list of
    # (slot, tokens, sum) in the reference's order
    beams = [[(0, [], 0.0)] for _ in range(W)]
    for step in range(steps):
        tok = bs.step(tok)
        logits = bs.logits.cpu().numpy()
        src, new_tok = bs.src.cpu().numpy(), tok.cpu().numpy()
        sums, rank = bs.sum.cpu().numpy(), bs.rank.cpu().numpy()
        for w in range(W):
            cands = []
            for slot, toks, s in beams[w]:
                lps = _log_softmax(logits[w * B + slot, :limit])
                for lp, i in _top_k(lps, B):
                    st = max(lp, -30.0)
                    cands.append((np.float32(s) + np.float32(st), slot, i, toks))
            cands.sort(key=lambda c: -float(c[0]))          # stable, as Rust's sort_by
            cands = cands[:B]
            got = sorted(range(B), key=lambda b: rank[w * B + b])
            nxt = []
            for r, (sc, parent, i, toks) in enumerate(cands):
                b = got[r]
                s = w * B + b
                assert int(new_tok[s]) == i, (step, w, r)
                assert int(src[s]) == w * B + parent, (step, w, r)
                assert abs(float(sums[s]) - float(sc)) <= 1e-4 * max(1.0, abs(float(sc))), (step, w, r)
                nxt.append((b, toks + [i], float(sums[s])))
            beams[w] = nxt
    # every beam's state is that of a fresh decoder fed its whole sequence
    fresh = decoder.Decoder(V, CTX, D, H, L, t)
    fresh.begin(enc, sw)
    hist = [None] * (W * B)
    for w in range(W):
        for b, toks, _ in beams[w]:
            hist[w * B + b] = prompt + toks[:-1]
    for p in range(len(hist[0])):
        fresh.step([h[p] for h in hist], want="none")
    last = [beams[w][[x[0] for x in beams[w]].index(b)][1][-1] for w in range(W) for b in range(B)]
    want = fresh.step(last).cpu().numpy()
    got = dec.step(torch_mod.tensor(last, dtype=torch_mod.int32, device="cuda")).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
