"""Benchmark of the B200 quantized-matmul path (BASELINE config 2 sweep).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one pass of the config-2 encoder sweep: for each of the three
whisper-small shapes (K, N) in {(768,768), (768,3072), (3072,768)} the
M=1500 activations are quantized once and multiplied by the five weight
formats (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0): 3 quantizer + 15 GEMM launches.
`value` is whole-job throughput in TOPS (2*M*N*K per GEMM, inputs resident
in HBM, L2 flushed before every timed step).  The decoder GEMVs of the same
config (M in {1, 5}) are timed in the `gemv` object against HBM bandwidth,
over rotating weight copies larger than L2.  `e2e` is the same sweep
through the reference-shaped host-buffer entry point (rwq_matmul_t_q:
host activations in, host outputs back, copies inside the timed region).

Multi-GPU (torchrun): every rank runs its own sweep on its own windows'
activations (weak scaling, no collective on the data path); the timed
region is bracketed by barriers and the max over ranks is reported.

`--impl reference` times the reference's CPU path (the C++ restatement in
oracle/, rusty_whisper being Rust with no toolchain here) on the host
cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from rusty_whisper_b200 import synth  # noqa: E402
from rusty_whisper_b200.formats import NAMES, QK, block_bytes  # noqa: E402

METRIC = "config-2 encoder quant-GEMM throughput (5 formats x whisper-small shapes, M=1500)"
UNIT = "TOPS"
# A spin kernel this long (~2 ms) runs before each timed step so that the
# host enqueues the whole step before the GPU reaches it: the CUDA events
# then bracket device work only, with no host gaps inside.
GATE_CYCLES = 4_000_000
WORKLOAD = ("BASELINE config 2: Q4_0/Q4_1/Q5_0/Q5_1/Q8_0 x (K,N) in {(768,768),(768,3072),(3072,768)}, "
            "M=1500 GEMMs (int8 activation semantics); decoder GEMVs M in {1,5} reported under gemv")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def profile_traffic(name: str):
    """dram bytes per launch recorded from an ncu capture (profiles/)."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def sweep_inputs(rank: int):
    """Seeded config-2 inputs; each rank processes its own activations."""
    acts = {}
    weights = {}
    for (k, n) in synth.SWEEP_SHAPES:
        acts[(k, n)] = synth.sweep_acts(synth.ENCODER_M, k, seed=rank)
        for dt in synth.SWEEP_FORMATS:
            weights[(dt, k, n)] = synth.sweep_weight(dt, k, n)
    return acts, weights


def gemm_ops():
    return sum(2.0 * synth.ENCODER_M * n * k for (k, n) in synth.SWEEP_SHAPES) * len(synth.SWEEP_FORMATS)


class Clocks:
    """nvidia-smi sampling during the timed region."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "50", "-i", str(self.index)], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *exc):
        self.rows = []
        if self.p is None:
            return False
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.p.kill()
            out, _ = self.p.communicate()
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 8:
                self.rows.append(f)
        return False

    def summary(self):
        rows = getattr(self, "rows", [])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for nm, v in zip(names, r[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# --------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from rusty_whisper_b200 import quant

    torch.cuda.set_device(local_rank)
    quant.init(local_rank)
    quant.set_gemm_path(args.gemm_path)
    dev = torch.device("cuda", local_rank)
    hbm_peak, tc_peak, peak_kind = peaks()

    acts_np, w_np = sweep_inputs(rank)
    acts = {s: torch.from_numpy(a).to(dev) for s, a in acts_np.items()}
    W = {key: quant.QTensor([key[2], key[1]], key[0], raw) for key, raw in w_np.items()}
    for w in W.values():
        w.prepare_gemm()
    Y = {key: torch.empty((synth.ENCODER_M, key[2]), dtype=torch.float32, device=dev) for key in W}
    qa = {s: quant.QActs(synth.ENCODER_M, s[0]) for s in synth.SWEEP_SHAPES}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def step(per_gemm=None):
        for s in synth.SWEEP_SHAPES:
            qa[s].quantize(acts[s])
            for dt in synth.SWEEP_FORMATS:
                key = (dt, s[0], s[1])
                if per_gemm is not None:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    qa[s].matmul(W[key], out=Y[key])
                    e1.record(stream)
                    per_gemm.append((key, e0, e1))
                else:
                    qa[s].matmul(W[key], out=Y[key])

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    quant.stream_check()

    # ---- timed region: K steps, L2 flushed before each, one event pair per
    # step (no events between the step's kernels)
    steps = []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local_rank).__enter__()
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda._sleep(GATE_CYCLES)   # hold the GPU until the whole step is enqueued
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step()
        e1.record(stream)
        steps.append((e0, e1))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    quant.stream_check()
    # ---- per-kernel pass (roofline): for each GEMM, R back-to-back launches
    # of that kernel between one event pair (its steady-state launch time)
    per_gemm = []
    R = 8
    for s_ in synth.SWEEP_SHAPES:
        qa[s_].quantize(acts[s_])
        for dt in synth.SWEEP_FORMATS:
            key = (dt, s_[0], s_[1])
            torch.cuda.synchronize()
            torch.cuda._sleep(GATE_CYCLES)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(R):
                qa[s_].matmul(W[key], out=Y[key])
            e1.record(stream)
            per_gemm.append((key, e0, e1, R))
    torch.cuda.synchronize()
    t_steps = sum(a.elapsed_time(b) for a, b in steps) / 1e3      # seconds
    t_gemm = sum(a.elapsed_time(b) / r for _, a, b, r in per_gemm) / 1e3
    tmax = t_steps
    if world > 1:
        t = torch.tensor([t_steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tmax = float(t.item())
    ops_step = gemm_ops()
    value = world * ops_step * args.steps / tmax / 1e12
    gemm_tops = ops_step / t_gemm / 1e12   # kernel-level, this rank

    # per-format kernel numbers (this rank)
    by_fmt = {}
    for key, a, b, r in per_gemm:
        dt, k, n = key
        by_fmt.setdefault(NAMES[dt], [0.0, 0.0])
        by_fmt[NAMES[dt]][0] += 2.0 * synth.ENCODER_M * n * k
        by_fmt[NAMES[dt]][1] += a.elapsed_time(b) / r / 1e3
    by_fmt = {f: round(o / t / 1e12, 2) for f, (o, t) in by_fmt.items()}

    config1 = run_config1(args, dev, quant, stream, rank, world) if args.only == "all" else None
    gemv = run_gemv(args, dev, quant, w_np, hbm_peak, stream) if args.only == "all" else None
    e2e = run_e2e(args, dev, quant, W, acts_np, world) if args.only == "all" else None
    frontend = run_frontend(args, dev, hbm_peak, stream, rank, world) if args.only == "all" else None
    enc = run_encoder(args, dev, tc_peak, stream, rank, world) if args.only == "all" else None
    dec = run_decoder_beams(args, dev, hbm_peak, stream, rank, world) if args.only == "all" else None
    large = run_large_v3(args, dev, stream, rank, world) if args.only == "all" else None
    clk.__exit__(None, None, None)

    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(tmax / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 codes (exact on f16 tensor cores), f32 scales/accumulation",
        "data": "synthetic (seeded SplitMix64; BASELINE config 2 distributions)",
        "config": {"workload": WORKLOAD, "M": synth.ENCODER_M, "shapes_KN": list(synth.SWEEP_SHAPES),
                   "formats": [NAMES[d] for d in synth.SWEEP_FORMATS], "parallelism": f"replicas x{world}",
                   "l2": "256 MiB buffer written before every timed step (L2 126 MB)"},
        "gpu_launches": 18 * args.steps,
        "roofline": {
            "bound": "tensor",
            "kernel": "k_gemm_fold_w (N=3072: 128x256 tiles) + k_gemm_fold<64> (N=768) (tcgen05 kind::f16, "
                      "weight scales folded into an f16 hi|lo operand)",
            "achieved": round(gemm_tops, 2), "peak": tc_peak, "unit": "TFLOP/s",
            "frac": round(gemm_tops / tc_peak, 4), "peak_kind": f"{peak_kind} dense bf16 (burst)",
            "traffic": profile_traffic("k_gemm_fold_w_config2_768x3072.md"),
            "traffic_launch": "ncu, k_gemm_fold_w Q4_0 M=1500 K=768 N=3072 launch (profiles/)",
            "per_format_tops": by_fmt,
            # The int8 tier's block scaling costs two f16 MMAs per unit of
            # work (the weight operand as hi + lo): what the tensor pipe
            # actually issues, against the same peak.
            "issued_mma_tflops": round(2 * gemm_tops, 2),
            "issued_mma_frac": round(2 * gemm_tops / tc_peak, 4),
        },
        "config1": config1,
        "gemv": gemv,
        "frontend": frontend,
        "encoder": enc,
        "decoder_beams": dec,
        "large_v3_e2e": large,
        "e2e": e2e,
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(acts_np, w_np)
    print(json.dumps(line), flush=True)


def run_frontend(args, dev, hbm_peak, stream, rank, world):
    """BASELINE config 5's front end: log-mel of 256 windows of 30 s
    (audio.rs:147-198) on the GPU in one batch, against the C restatement
    of the reference on this host's cores (a bounded sample)."""
    import torch
    from rusty_whisper_b200 import audio
    n_win, n_mels = 256, 80
    distinct = [synth.speechlike_window(500 + 7 * i) for i in range(8)]
    host = np.stack([distinct[i % 8] for i in range(n_win)])
    x = torch.from_numpy(host).to(dev)
    fb = audio.mel_filterbank(n_mels)
    plan = audio.LogMel(fb, n_mels)
    out = torch.empty((n_win, n_mels, synth.AUDIO_WINDOW // audio.HOP_LENGTH), device=dev)
    for _ in range(3):
        plan.batch(x, out)
    torch.cuda.synchronize()
    reps = max(3, min(args.steps, 10))
    torch.cuda._sleep(GATE_CYCLES)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        plan.batch(x, out)
    e1.record(stream)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / reps
    frames = synth.AUDIO_WINDOW // audio.HOP_LENGTH
    # samples read once; mel written, then read and written by the normaliser
    nbytes = n_win * (4.0 * synth.AUDIO_WINDOW + 3 * 4.0 * n_mels * frames)
    res = {"workload": f"{n_win} windows x 30 s, {n_mels} mels (BASELINE config 5 front end)",
           "windows_per_s": round(world * n_win / t, 1), "audio_s_per_s": round(world * n_win * 30.0 / t, 1),
           "us_per_window": round(t / n_win * 1e6, 3), "GB/s": round(nbytes / t / 1e9, 1),
           "frac_of_measured_hbm": round(nbytes / t / 1e9 / hbm_peak, 4), "bound": "hbm",
           "kernels": "k_log_mel + k_mel_norm (csrc/rwq_mel.cu)", "gpu_launches": 3 * reps}
    if rank == 0 and world == 1 and not args.no_cpu:
        import time
        import oracle
        threads = oracle.default_threads()
        t0 = time.perf_counter()
        for i in range(2):
            oracle.log_mel_spectrogram(distinct[i], fb, n_mels, threads=threads)
        tc = (time.perf_counter() - t0) / 2
        res["cpu_baseline"] = {"audio_s_per_s": round(30.0 / tc, 1), "s_per_window": round(tc, 4),
                               "cores": threads, "kind": "port",
                               "sample": "2 windows of 30 s through the C restatement of audio.rs:147-198"}
    return res


ENC_BASE = dict(n_mels=80, n_ctx=1500, n_state=512, n_head=8, n_layer=6)   # whisper-base


def encoder_flops(n_ctx, n_state, n_layer, n_mels):
    """Per window: quantized linears 2*T*(4*D*D + 2*D*4D) per block,
    attention 2 * 2*T*T*D per block, conv stem 2*(2T*D*3*n_mels + T*D*3*D)."""
    T, D = n_ctx, n_state
    lin = n_layer * 2.0 * T * (4 * D * D + 8 * D * D)
    att = n_layer * 4.0 * T * T * D
    conv = 2.0 * (2 * T * D * 3 * n_mels + T * D * 3 * D)
    return lin, att, conv


def run_encoder(args, dev, tc_peak, stream, rank, world):
    """whisper-base encoder forward, Q5_1 linears from
    N(0, 0.02) weights, batch of 8 windows (log-mel N(-0.5, 0.3) clamped
    to +-1.5), audio-seconds per second; the oracle's restatement of
    encoder.rs timed beside it on the host cores (one window)."""
    import torch
    from rusty_whisper_b200 import encoder
    cfg = ENC_BASE
    n_win = 8
    t = synth.encoder_tensors(cfg["n_mels"], cfg["n_ctx"], cfg["n_state"], cfg["n_layer"], 7, seed=3)
    enc = encoder.Encoder(cfg["n_mels"], cfg["n_ctx"], cfg["n_state"], cfg["n_head"], cfg["n_layer"], t)
    mel_np = synth.encoder_mel(n_win, cfg["n_mels"], 2 * cfg["n_ctx"], seed=100 + rank)
    mel = torch.from_numpy(mel_np).to(dev)
    out = torch.empty((n_win, cfg["n_ctx"], cfg["n_state"]), device=dev)
    for _ in range(2):
        enc.encode(mel, out)
    torch.cuda.synchronize()
    reps = max(3, min(args.steps, 10))
    times = []
    for _ in range(reps):
        torch.cuda._sleep(GATE_CYCLES)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        enc.encode(mel, out)
        e1.record(stream)
        times.append((e0, e1))
    torch.cuda.synchronize()
    from rusty_whisper_b200 import quant
    quant.stream_check()
    tb = statistics.median(a.elapsed_time(b) for a, b in times) / 1e3
    lin, att, conv = encoder_flops(cfg["n_ctx"], cfg["n_state"], cfg["n_layer"], cfg["n_mels"])
    fl = n_win * (lin + att + conv)
    res = {"workload": f"BASELINE config 3: whisper-base encoder (6 x d512/8 heads/FFN 2048), Q5_1 linears, "
                       f"batch {n_win} windows of 30 s",
           "audio_s_per_s": round(world * n_win * 30.0 / tb, 1), "ms_per_batch": round(tb * 1e3, 3),
           "windows_per_s": round(world * n_win / tb, 2),
           "gflop_per_window": {"quant_linear": round(lin / 1e9, 2), "attention": round(att / 1e9, 2),
                                "conv": round(conv / 1e9, 2)},
           "achieved_TFLOPs": round(fl / tb / 1e12, 1), "frac_of_measured_bf16": round(fl / tb / 1e12 / tc_peak, 4),
           "kernels": "k_rows_quant, k_gemm_fold_w (Q/K/V writing f16 heads, fc1 with GELU + quantize in its "
                      "epilogue), k_gemm_fold, k_attn (its output rows quantized in the kernel); "
                      "conv stem: k_im2col_split + k_gemm_hl (f16 hi|lo "
                      "tensor cores, bias + GELU (+ positions) in its epilogue)",
           # stem 2 x (im2col, GEMM); per block 6 GEMMs (Q/K/V write heads, fc1
           # quantizes its output), attention, 2 LayerNorms; ln_post
           "gpu_launches_per_batch": 4 + 6 * 9 + 1,
           "data": "synthetic (seeded): random-init weights N(0, 0.02) quantized to Q5_1, mel N(-0.5, 0.3)"}
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        threads = oracle.default_threads()
        ref = oracle.Encoder(cfg["n_mels"], cfg["n_ctx"], cfg["n_state"], cfg["n_head"], cfg["n_layer"], t)
        ref.encode(mel_np[0], threads=threads)       # first call: the reference's cold weight path
        t0 = time.perf_counter()
        ref.encode(mel_np[1], threads=threads)
        tc = time.perf_counter() - t0
        res["cpu_baseline"] = {"audio_s_per_s": round(30.0 / tc, 2), "s_per_window": round(tc, 3), "cores": threads,
                               "kind": "port", "tier": oracle.TIER_NAMES[oracle.dispatch_tier()],
                               "sample": "1 window (second call, packed weights) through the C++ restatement "
                                         "of encoder.rs:180-234"}
    return res


DEC_MEDIUM = dict(n_vocab=51865, n_ctx=448, n_state=1024, n_head=16, n_layer=24)   # whisper-medium decoder (config 4)
LARGE_V3 = dict(n_mels=128, n_audio=1500, n_state=1280, n_head=20, enc_layers=32, dec_layers=32, n_vocab=51866,
                n_ctx=448)


def run_decoder_beams(args, dev, hbm_peak, stream, rank, world):
    """whisper-medium decoder, Q5_0, 16 windows, beam 5
    (80 streams; the five beams of a window share its cross K/V), 224
    fixed steps after a seeded random 4-token prompt per window,
    cross-attention over a 1500 x 1024 N(0, 1) encoder output per window.
    Every step is the reference's beam step (transcribe.rs:886-990) on the
    device: the step with its stacked logits projection, log_softmax +
    top-5 per beam, the per-window ranking of the 25 candidates and the
    fork of the survivors' self-attention caches.  End-of-text and the
    other special ids are never chosen, so every beam decodes all 224 steps
    (the finished-hypothesis bookkeeping is host policy).  Tokens per
    second of all beams."""
    import torch
    from rusty_whisper_b200 import decoder
    c = DEC_MEDIUM
    n_win, beams, steps, prefix = 16, 5, 224, 4
    S = n_win * beams
    eot = 50257
    t = synth.decoder_tensors(c["n_vocab"], c["n_ctx"], c["n_state"], c["n_layer"], 6, seed=7, gen_device=dev)
    dec = decoder.Decoder(c["n_vocab"], c["n_ctx"], c["n_state"], c["n_head"], c["n_layer"], t)
    enc = torch.from_numpy(synth.normal(300 + rank, n_win * 1500 * c["n_state"]).reshape(n_win, 1500, c["n_state"]))
    enc = enc.to(dev)
    sw = [w for w in range(n_win) for _ in range(beams)]
    pre_w = synth.randint(400 + rank, prefix * n_win, 0, 50256).astype(np.int32).reshape(prefix, n_win)
    pre = torch.from_numpy(np.repeat(pre_w, beams, axis=1).copy()).to(dev)   # a window's beams share its prompt
    search = decoder.BeamSearch(dec, n_win, beams, limit=eot)

    def run(n_steps):
        dec.begin(enc, sw)
        search.live = 1
        for i in range(prefix - 1):
            dec.step(pre[i], want="none")
        tok = pre[prefix - 1]
        for _ in range(n_steps):
            tok = search.step(tok)
        return tok

    run(8)
    torch.cuda.synchronize()
    torch.cuda._sleep(GATE_CYCLES)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run(steps)
    e1.record(stream)
    torch.cuda.synchronize()
    from rusty_whisper_b200 import quant
    quant.stream_check()
    tt = e0.elapsed_time(e1) / 1e3
    D, Lr = c["n_state"], c["n_layer"]
    cross_bytes = n_win * Lr * 2 * 1500 * D * 2.0
    res = {"workload": "BASELINE config 4: whisper-medium decoder (24 x d1024/16 heads/FFN 4096, vocab 51865), Q5_0, "
                       f"{n_win} windows x beam {beams}, {steps} beam steps after a {prefix}-token prompt",
           "tokens_per_s": round(world * S * steps / tt, 1), "ms_per_step": round(tt / (steps + prefix) * 1e3, 3),
           "streams": S,
           "bytes_per_step": {"quantized_weights": round(sum(v[1].nbytes for v in t.values() if isinstance(v, tuple)) / 1e6, 1),
                              "cross_kv_f16_MB": round(cross_bytes / 1e6, 1)},
           "beam": beams,
           "note": "linears on the tiled integer-MMA GEMV (k_gemv_tile: 80 streams as 32-row tiles, bit-identical "
                   "to the per-stream GEMV); the decoder step replays from a CUDA graph, then k_beam_topk, "
                   "k_beam_select and k_self_fork (copies only the survivors not kept in their parent's slot)",
           "data": "synthetic (seeded): random-code Q5_0 weights (every block its own draw), encoder output N(0, 1)"}
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        threads = oracle.default_threads()
        ref = oracle.Decoder(c["n_vocab"], c["n_ctx"], c["n_state"], c["n_head"], c["n_layer"], t)
        ref.begin(enc[0].cpu().numpy(), threads=threads)
        ref.forward([1], threads=threads)               # first call: the reference's cold weight path
        t0 = time.perf_counter()
        for tk in (2, 3, 4):
            ref.forward([tk], threads=threads)
        tc = (time.perf_counter() - t0) / 3
        res["cpu_baseline"] = {"tokens_per_s": round(1.0 / tc, 2), "s_per_token": round(tc, 4), "cores": threads,
                               "kind": "port", "tier": oracle.TIER_NAMES[oracle.dispatch_tier()],
                               "sample": "3 decode steps of one stream (forward(&[token]), packed weights) through the "
                                         "C++ restatement of decoder.rs:102-206, 315-321"}
    return res


def run_large_v3(args, dev, stream, rank, world):
    """large-v3-shaped end to end, Q4_0: 256 windows of 30 s
    synthetic audio sharded evenly over the ranks through shard.run_sharded
    (the reference's transcribe_parallel + merge_parallel_results,
    transcribe.rs:1528-1586); per rank, host audio -> log-mel (128 mels) ->
    encoder (32 blocks, d1280) -> decoder (32 blocks, vocab 51866) greedy for
    224 tokens after the 4-token start sequence -> token ids back on the
    host, then every window's tokens gathered on rank 0 in window order.
    Audio-seconds per second of all ranks (device time, max over ranks)."""
    import torch
    import torch.distributed as dist
    from rusty_whisper_b200 import audio, decoder, encoder, shard
    c = LARGE_V3
    total_win, steps = 256, 224
    share = list(shard.window_range(total_win, world, rank))
    n_win = len(share)
    te = synth.encoder_tensors(c["n_mels"], c["n_audio"], c["n_state"], c["enc_layers"], 2, seed=11, gen_device=dev)
    td = synth.decoder_tensors(c["n_vocab"], c["n_ctx"], c["n_state"], c["dec_layers"], 2, seed=12, gen_device=dev)
    enc = encoder.Encoder(c["n_mels"], c["n_audio"], c["n_state"], c["n_head"], c["enc_layers"], te)
    dec = decoder.Decoder(c["n_vocab"], c["n_ctx"], c["n_state"], c["n_head"], c["dec_layers"], td)
    del te, td
    mel_plan = audio.LogMel(audio.mel_filterbank(c["n_mels"]), c["n_mels"])
    distinct = [synth.speechlike_window(900 + 13 * i) for i in range(8)]
    host = torch.from_numpy(np.stack([distinct[i % 8] for i in share])).pin_memory()
    toks_host = torch.empty((steps, n_win), dtype=torch.int32).pin_memory()
    sot = torch.tensor([50258, 50259, 50360, 50364], dtype=torch.int32)     # sot, lang, transcribe, notimestamps
    prompt = sot.repeat(n_win, 1).t().contiguous().to(dev)
    eot = 50257

    marks = {}

    def pipeline(n_steps, copy_out=True):
        x = host.to(dev, non_blocking=True)
        mel = mel_plan.batch(x)
        eo = enc.encode(mel)
        marks["enc"] = torch.cuda.Event(enable_timing=True)
        marks["enc"].record(stream)
        dec.begin(eo)
        marks["begin"] = torch.cuda.Event(enable_timing=True)
        marks["begin"].record(stream)
        for i in range(3):
            dec.step(prompt[i], want="none")
        out = torch.empty((n_steps, n_win), dtype=torch.int32, device=dev)
        tok = dec.step(prompt[3], want="best", limit=eot, out=out[0])
        for i in range(1, n_steps):
            tok = dec.step(tok, want="best", limit=eot, out=out[i])
        if copy_out:
            toks_host[:n_steps].copy_(out, non_blocking=True)
        return out

    pipeline(4)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)

    def run_share(batch):
        assert list(batch) == share
        e0.record(stream)
        pipeline(steps)
        e1.record(stream)
        torch.cuda.synchronize()
        return [toks_host[:, j].clone() for j in range(n_win)]

    w0 = time.perf_counter()
    gathered = shard.run_sharded(list(range(total_win)), run_share, timeout_s=300.0)
    wall = time.perf_counter() - w0
    from rusty_whisper_b200 import quant
    quant.stream_check()
    if rank == 0:
        assert len(gathered) == total_win and all(g.shape == (steps,) for g in gathered)
    tt = e0.elapsed_time(e1) / 1e3
    tmax = tt
    if world > 1:
        tm = torch.tensor([tt, wall], dtype=torch.float64, device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        tmax, wall = float(tm[0].item()), float(tm[1].item())
    stages = {"audio_mel_encoder_s": round(e0.elapsed_time(marks["enc"]) / 1e3, 3),
              "cross_kv_s": round(marks["enc"].elapsed_time(marks["begin"]) / 1e3, 3),
              "decode_s": round(marks["begin"].elapsed_time(e1) / 1e3, 3)}
    res = {"workload": "BASELINE config 5: large-v3 shape (128 mels; encoder 32 x d1280/20 heads/FFN 5120; decoder 32 "
                       "blocks, vocab 51866), Q4_0, 256 windows x 30 s sharded over the ranks, greedy 224 tokens",
           "audio_s_per_s": round(total_win * 30.0 / tmax, 1), "s_per_job": round(tmax, 3),
           "rank0_stages": stages, "ms_per_decode_step": round(stages["decode_s"] / (steps + 4) * 1e3, 3),
           "windows_per_rank": n_win, "scaling": "strong (256 windows in total)",
           "h2d_bytes_per_rank": int(host.numel() * 4), "d2h_bytes_per_rank": int(steps * n_win * 4),
           "timing": "CUDA events around host audio -> tokens on the host, max over ranks; the host gather of "
                     "every window's tokens on rank 0 (shard.run_sharded) follows it",
           "gather": {"windows_on_rank0": total_win if rank == 0 else None,
                      "wall_s_incl_gather": round(wall, 3)},
           "data": "synthetic (seeded): band-limited noise at -20 dBFS with 0.2-2 s silences; random-code Q4_0 "
                   "weights (every block its own draw)"}
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        threads = oracle.default_threads()
        tc0 = time.perf_counter()
        # blocks 0 and 1 of the same model (the generator draws blocks in order)
        te = synth.encoder_tensors(c["n_mels"], c["n_audio"], c["n_state"], 2, 2, seed=11, gen_device=dev)
        ref_e = oracle.Encoder(c["n_mels"], c["n_audio"], c["n_state"], c["n_head"], 2, te)   # 2 of the 32 blocks
        mel1 = mel_plan(distinct[0])
        t0 = time.perf_counter()
        eo1 = ref_e.encode(mel1, threads=threads)
        t_enc2 = time.perf_counter() - t0
        del ref_e, te
        td = synth.decoder_tensors(c["n_vocab"], c["n_ctx"], c["n_state"], c["dec_layers"], 2, seed=12,
                                   gen_device=dev)
        ref_d = oracle.Decoder(c["n_vocab"], c["n_ctx"], c["n_state"], c["n_head"], c["dec_layers"], td)
        ref_d.begin(eo1, threads=threads)
        ref_d.forward([50258], threads=threads)
        t0 = time.perf_counter()
        for tk in (50259, 50360):
            ref_d.forward([tk], threads=threads)
        t_tok = (time.perf_counter() - t0) / 2
        # extrapolation: the encoder's 32 blocks from 2 (the conv stem is in
        # both), the decoder's 228 positions from 2
        t_win = t_enc2 * 16 + t_tok * (steps + 4)
        res["cpu_baseline"] = {"audio_s_per_s": round(30.0 / t_win, 4), "s_per_window": round(t_win, 2),
                               "cores": threads, "kind": "port", "tier": oracle.TIER_NAMES[oracle.dispatch_tier()],
                               "sample": f"one window: encoder with 2 of 32 blocks ({t_enc2:.1f} s) and 2 decoder "
                                         f"positions ({t_tok:.2f} s each) through the C++ restatement, extrapolated "
                                         f"linearly to 32 blocks and 228 positions (extrapolated; "
                                         f"{time.perf_counter() - tc0:.0f} s of CPU work)"}
    return res


def run_profile_driver(args):
    """Small fixed workloads for ncu captures (no timing line of record):
    `logits` -- config 4's tied-logits GEMV (Q5_0 51865 x 1024, four weight
    copies) at --m rows, --steps back-to-back launches; `gemv` -- the same
    for config 5's decoder projection (Q4_0 1280 x 1280, eight copies);
    `decode` -- the config-4 decoder (80 streams; config 5's with --m 32..256 windows),
    begin then --steps greedy steps; `attention` -- --steps calls of the
    encoder's attention (rwq_attention_dev) at config 3's shape, 8 windows
    x 1500 frames x 8 heads of 64."""
    import torch
    from rusty_whisper_b200 import quant
    quant.init(0)
    dev = torch.device("cuda", 0)
    if args.only in ("logits", "gemv"):
        n, k, dt, copies = (51865, 1024, 6, 4) if args.only == "logits" else (1280, 1280, 2, 8)
        raw = synth.random_blocks(dt, n, k, 5)
        W = [quant.QTensor([n, k], dt, raw) for _ in range(copies)]
        x = torch.from_numpy(synth.normal(9, args.m * k).reshape(args.m, k)).to(dev)
        qa = quant.QActs(args.m, k).quantize(x)
        y = torch.empty((args.m, n), device=dev)
        for r in range(args.steps):
            qa.matmul(W[r % copies], out=y)
        # The same launches replayed from a CUDA graph, timed with events
        # (no host gaps between them).
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            qa.matmul(W[0], out=y)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=st):
            for r in range(args.steps):
                qa.matmul(W[r % copies], out=y)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            gr.replay()
            e0.record(st)
            gr.replay()
            e1.record(st)
        torch.cuda.synchronize()
        us_per_launch = e0.elapsed_time(e1) * 1e3 / max(args.steps, 1)
        del gr
    elif args.only == "attention":
        from rusty_whisper_b200 import encoder
        nw, t_ctx, d, heads = 8, 1500, 512, 8
        q, k, v = (torch.from_numpy(synth.normal(40 + i, nw * t_ctx * d).reshape(nw, t_ctx, d)).to(dev)
                   for i in range(3))
        encoder.multi_head_attention(q, k, v, heads)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            encoder.multi_head_attention(q, k, v, heads)
        e1.record()
        torch.cuda.synchronize()
        us_per_call = e0.elapsed_time(e1) * 1e3 / max(args.steps, 1)
        attn_flop = 4.0 * nw * heads * t_ctx * t_ctx * 64
    else:
        from rusty_whisper_b200 import decoder
        if args.m in (32, 64, 128, 256):   # config 5's decoder: large-v3 shape, Q4_0, m windows (256 / ranks)
            c = dict(n_vocab=LARGE_V3["n_vocab"], n_ctx=448, n_state=1280, n_head=20, n_layer=32)
            n_win, per, dt = args.m, 1, 2
        else:               # config 4: whisper-medium, Q5_0, 16 windows x 5 streams
            c, n_win, per, dt = DEC_MEDIUM, 16, 5, 6
        t = synth.decoder_tensors(c["n_vocab"], c["n_ctx"], c["n_state"], c["n_layer"], dt, seed=7, gen_device=dev)
        dec = decoder.Decoder(c["n_vocab"], c["n_ctx"], c["n_state"], c["n_head"], c["n_layer"], t)
        enc = torch.empty((n_win, 1500, c["n_state"]), device=dev)
        for w in range(n_win):   # seeded rows, drawn per window to bound host memory
            enc[w] = torch.from_numpy(synth.normal(300 + w % 8, 1500 * c["n_state"]).reshape(1500, c["n_state"]))
        dec.begin(enc, [w for w in range(n_win) for _ in range(per)])
        tok = torch.zeros(n_win * per, dtype=torch.int32, device=dev)
        if args.only == "beam":   # config 4's benchmarked step: beam 5 (top-k, ranking, fork)
            bs = decoder.BeamSearch(dec, n_win, per, limit=50257)   # end-of-text, as the benchmarked step
            for _ in range(args.steps):
                tok = bs.step(tok)
        else:
            for _ in range(args.steps):
                tok = dec.step(tok, want="best")
    torch.cuda.synchronize()
    quant.stream_check()
    line = {"profile_driver": args.only, "m": args.m, "steps": args.steps}
    if args.only in ("logits", "gemv"):
        line.update(us_per_launch=round(us_per_launch, 2), tops=round(2 * args.m * n * k / us_per_launch / 1e6, 1))
    if args.only == "attention":   # a call: three f16 head conversions + k_attn
        line.update(us_per_call=round(us_per_call, 1), tflops=round(attn_flop / us_per_call / 1e6, 1))
    print(json.dumps(line), flush=True)


def run_gemv(args, dev, quant, w_np, hbm_peak, stream):
    """Decoder GEMVs of config 2: for each weight, R back-to-back launches
    over copies rotated past L2, one event pair per batch."""
    import torch
    total_w = sum(r.nbytes for r in w_np.values())
    copies = max(2, int(np.ceil(300e6 / total_w)))
    Wc = [{key: quant.QTensor([key[2], key[1]], key[0], raw) for key, raw in w_np.items()} for _ in range(copies)]
    res = {}
    for mm in synth.SWEEP_GEMV_M:
        xs = {s: torch.from_numpy(synth.sweep_acts(mm, s[0], seed=9)).to(dev) for s in synth.SWEEP_SHAPES}
        qa = {s: quant.QActs(mm, s[0]) for s in synth.SWEEP_SHAPES}
        for s in synth.SWEEP_SHAPES:
            qa[s].quantize(xs[s])
        ys = {key: torch.empty((mm, key[2]), device=dev) for key in w_np}
        for c in range(copies):
            for key in w_np:
                qa[(key[1], key[2])].matmul(Wc[c][key], out=ys[key])
        torch.cuda.synchronize()
        nbytes = 0.0
        t = 0.0
        per_fmt = {}
        launches = 0
        for key in w_np:
            dt, k, n = key
            s = (k, n)
            torch.cuda._sleep(GATE_CYCLES)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for c in range(copies):
                qa[s].matmul(Wc[c][key], out=ys[key])
            e1.record(stream)
            torch.cuda.synchronize()
            dtm = e0.elapsed_time(e1) / 1e3
            b = copies * (n * (k // QK) * block_bytes(dt) + 4.0 * mm * k + 4.0 * mm * n)
            nbytes += b
            t += dtm
            launches += copies
            pf = per_fmt.setdefault(NAMES[dt], [0.0, 0.0])
            pf[0] += b
            pf[1] += dtm
        gbs = nbytes / t / 1e9
        # The same launches replayed from one CUDA graph (no host launch
        # gaps): what the decoder's graph-captured step sees.
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):   # the stream's workspace exists before capture
            for key in w_np:
                qa[(key[1], key[2])].matmul(Wc[0][key], out=ys[key])
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=st):
            for key in w_np:
                for c in range(copies):
                    qa[(key[1], key[2])].matmul(Wc[c][key], out=ys[key])
        with torch.cuda.stream(st):
            gr.replay()
            torch.cuda._sleep(GATE_CYCLES)
            g0 = torch.cuda.Event(enable_timing=True)
            g1 = torch.cuda.Event(enable_timing=True)
            g0.record(st)
            gr.replay()
            g1.record(st)
        torch.cuda.synchronize()
        tg = g0.elapsed_time(g1) / 1e3
        del gr
        res[f"M={mm}"] = {"GB/s": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm_peak, 4),
                          "us_per_gemv": round(t / launches * 1e6, 3),
                          "graph_GB/s": round(nbytes / tg / 1e9, 1),
                          "graph_us_per_gemv": round(tg / launches * 1e6, 3),
                          "per_format_GBs": {f: round(b / x / 1e9, 1) for f, (b, x) in per_fmt.items()}}
    res["logits_Q5_0_51865x1024"] = gemv_logits(args, dev, quant, hbm_peak, stream)
    res["bound"] = "hbm"
    res["peak_GBs"] = hbm_peak
    res["bytes"] = "N*(K/32)*block_bytes + 4*M*K + 4*M*N per GEMV (algorithmic)"
    res["timing"] = ("back-to-back launches of one GEMV over weight copies, one event pair per batch; graph_*: "
                     "the same launches of all weights replayed from one CUDA graph")
    res["l2"] = f"{copies} rotating weight copies ({copies * total_w / 1e6:.0f} MB > 126 MB L2)"
    return res


GEMV_KERNELS = {1: "k_gemv_i8", 2: "k_gemv_mma", 3: "k_gemv_tile", 4: "k_gemv_rows"}


def gemv_logits(args, dev, quant, hbm_peak, stream):
    """BASELINE config 4's largest GEMV: tied logits, vocab 51865, d=1024,
    Q5_0, M = 1 and 5 (beam), over 4 weight copies (146 MB > L2)."""
    import torch
    n, k, dt = 51865, 1024, 6
    raw = synth.random_blocks(dt, n, k, 77)
    Wl = [quant.QTensor([n, k], dt, raw) for _ in range(4)]
    out = {}
    for mm in (1, 5):
        x = torch.from_numpy(synth.normal(78 + mm, mm * k).reshape(mm, k)).to(dev)
        qa = quant.QActs(mm, k).quantize(x)
        y = torch.empty((mm, n), device=dev)
        for w in Wl:
            qa.matmul(w, out=y)
        torch.cuda.synchronize()
        reps = max(args.steps, 8)
        torch.cuda._sleep(GATE_CYCLES)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for r in range(reps):
            qa.matmul(Wl[r % 4], out=y)
        e1.record(stream)
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / reps
        b = n * (k // QK) * block_bytes(dt) + 4.0 * mm * k + 4.0 * mm * n
        out[f"M={mm}"] = {"GB/s": round(b / t / 1e9, 1), "frac_of_measured_hbm": round(b / t / 1e9 / hbm_peak, 4),
                          "us": round(t * 1e6, 2), "kernel": GEMV_KERNELS[quant.gemv_kernel_for(Wl[0], mm)]}
    return out


def run_config1(args, dev, quant, stream, rank, world):
    """BASELINE config 1 on its own seed-0 inputs: Q8_0 W[1536x384],
    X[1500x384] ~ N(0,1), one matmul_t_q (quantizer + tensor-core GEMM).
    Device-resident: R back-to-back calls between one event pair, L2
    flushed before each batch; end to end: the host-buffer entry point
    (pinned X in, Y out)."""
    import torch
    import torch.distributed as dist
    x_np, raw = synth.config1_inputs(0)
    m, k, n = 1500, 384, 1536
    w = quant.QTensor([n, k], 8, raw)
    w.prepare_gemm()
    x = torch.from_numpy(x_np).to(dev)
    y = torch.empty((m, n), dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    R = 20
    for _ in range(5):
        quant.matmul_t_q(x, w, out=y)
    torch.cuda.synchronize()
    times = []
    for _ in range(max(args.steps // 4, 3)):
        flush.zero_()
        torch.cuda._sleep(GATE_CYCLES)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(R):
            quant.matmul_t_q(x, w, out=y)
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3 / R)
    quant.stream_check()
    t = statistics.median(times)
    ops = 2.0 * m * n * k
    # end to end through the host-buffer call
    xp = torch.from_numpy(x_np).pin_memory()
    yp = torch.empty((m, n), dtype=torch.float32).pin_memory()
    for _ in range(3):
        quant.matmul_t_q(xp.numpy(), w, out=yp.numpy())
    reps = 20
    t0 = time.perf_counter()
    for _ in range(reps):
        quant.matmul_t_q(xp.numpy(), w, out=yp.numpy())
    te = (time.perf_counter() - t0) / reps
    if world > 1:
        tt = torch.tensor([t, te], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t, te = (float(v) for v in tt.tolist())
    out = {"workload": "BASELINE config 1: Q8_0 W[1536x384] (d~U(0.001,0.02), q~U[-127,127]), X[1500x384] ~ N(0,1), "
                       "seed 0; one matmul_t_q (int8 activation quantizer + GEMM)",
           "TOPS": round(world * ops / t / 1e12, 2), "us_per_matmul": round(t * 1e6, 2),
           "e2e": {"TOPS": round(world * ops / te / 1e12, 3), "us_per_call": round(te * 1e6, 1),
                   "h2d_bytes": m * k * 4, "d2h_bytes": m * n * 4,
                   "api": "rwq_matmul_t_q (pinned host buffers, synchronous)"},
           "kernels": "k_quantize + k_gemm_fold", "gpu_launches_per_matmul": 2,
           "l2": "256 MiB written before every batch of 20 calls"}
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        oracle.lib()
        threads = oracle.default_threads()
        oracle.matmul_t_q(x_np, 8, raw, n, tier=oracle.TIER_AUTO, threads=threads, packed=False)
        reps, t0 = 0, time.perf_counter()
        while reps < 3 or time.perf_counter() - t0 < 3.0:
            oracle.matmul_t_q(x_np, 8, raw, n, tier=oracle.TIER_AUTO, threads=threads, packed=False)
            reps += 1
            if reps >= 50:
                break
        tc = (time.perf_counter() - t0) / reps
        out["cpu_baseline"] = {"TOPS": round(ops / tc / 1e12, 4), "ms_per_matmul": round(tc * 1e3, 2),
                               "cores": threads, "kind": "port",
                               "tier": oracle.TIER_NAMES[oracle.dispatch_tier()],
                               "sample": f"{reps} calls of the same matmul (reference's first-call path)"}
    return out


def run_e2e(args, dev, quant, W, acts_np, world):
    """The sweep through the reference-shaped host-buffer entry point."""
    import torch
    import torch.distributed as dist
    pinned_a = {s: torch.from_numpy(a).pin_memory() for s, a in acts_np.items()}
    pinned_y = {key: torch.empty((synth.ENCODER_M, key[2]), dtype=torch.float32).pin_memory() for key in W}
    h2d = d2h = 0

    def step():
        nonlocal h2d, d2h
        h2d = d2h = 0
        for key, w in W.items():
            s = (key[1], key[2])
            quant.matmul_t_q(pinned_a[s].numpy(), w, out=pinned_y[key].numpy())
            h2d += pinned_a[s].numel() * 4
            d2h += pinned_y[key].numel() * 4

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    t = time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([t], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    return {"value": round(world * gemm_ops() * args.steps / t / 1e12, 3), "unit": UNIT,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "api": "rwq_matmul_t_q (host buffers, pinned), one call per GEMM, synchronous"}


# --------------------------------------------------------- CPU baselines
def cpu_sweep(acts_np, w_np, threads, budget_s, max_sweeps):
    import oracle
    oracle.lib()
    t0 = time.perf_counter()
    ops = 0.0
    sweeps = 0
    while sweeps < max_sweeps:
        for (dt, k, n), raw in w_np.items():
            a = acts_np[(k, n)]
            oracle.matmul_t_q(a, dt, raw, n, tier=oracle.TIER_AUTO, threads=threads, packed=False)
            ops += 2.0 * a.shape[0] * n * k
        sweeps += 1
        if time.perf_counter() - t0 > budget_s:
            break
    return ops / (time.perf_counter() - t0) / 1e12, sweeps


def cpu_baseline(acts_np, w_np):
    import oracle
    oracle.lib()
    threads = oracle.default_threads()
    v, sweeps = cpu_sweep(acts_np, w_np, threads, budget_s=10.0, max_sweeps=3)
    # one-thread figure on a one-GEMM sample
    (dt, k, n), raw = next(iter(w_np.items()))
    a = acts_np[(k, n)]
    t0 = time.perf_counter()
    oracle.matmul_t_q(a, dt, raw, n, tier=oracle.TIER_AUTO, threads=1, packed=False)
    t1 = time.perf_counter() - t0
    return {"value": round(v, 4), "unit": UNIT, "cores": threads, "kind": "port",
            "tier": oracle.TIER_NAMES[oracle.dispatch_tier()],
            "sample": f"{sweeps} full config-2 GEMM sweep(s) (15 GEMMs, M=1500), reference's first-call path, "
                      f"{threads} threads over N-chunks",
            "one_thread_value": round(2.0 * a.shape[0] * n * k / t1 / 1e12, 4),
            "one_thread_sample": f"{NAMES[dt]} {a.shape[0]}x{k}x{n}",
            "what": "C++ restatement of rusty_whisper's matmul_t_q (oracle/), the Rust original cannot be built here"}


def run_reference(args, rank):
    if rank != 0:
        return
    import oracle
    acts_np, w_np = sweep_inputs(0)
    oracle.lib()
    threads = oracle.default_threads()
    for _ in range(args.warmup):
        cpu_sweep(acts_np, w_np, threads, budget_s=0.0, max_sweeps=1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_sweep(acts_np, w_np, threads, budget_s=0.0, max_sweeps=1)
    t = time.perf_counter() - t0
    v = gemm_ops() * args.steps / t / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": UNIT, "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 codes, f32 scales (AVX-512 VNNI / AVX2 tier)",
        "data": "synthetic (seeded SplitMix64; BASELINE config 2 distributions)",
        "config": {"workload": WORKLOAD, "M": synth.ENCODER_M, "shapes_KN": list(synth.SWEEP_SHAPES),
                   "formats": [NAMES[d] for d in synth.SWEEP_FORMATS], "parallelism": "host threads"},
        "cpu_baseline": {"value": round(v, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "tier": oracle.TIER_NAMES[oracle.dispatch_tier()],
                         "sample": "one full config-2 GEMM sweep per step (15 GEMMs, M=1500)"},
        "e2e": {"value": round(v, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--gemm-path", type=int, default=0,
                    help="GEMM kernel path of the sweep (rwq_set_gemm_path): 0 automatic (folded-scale), 2 folded-scale, "
                         "3 exact integer, 4 hi|lo")
    ap.add_argument("--m", type=int, default=1,
                    help="--only logits: activation rows; --only decode: 32, 64, 128 or 256 select config 5's "
                         "decoder with that many windows (one rank's share at 8, 4, 2, 1 GPUs)")
    ap.add_argument("--only", default="all", choices=["all", "gemm", "encoder", "decoder", "large", "logits", "gemv", "decode",
                                                      "beam", "attention"],
                    help="gemm: only the config-2 GEMM sweep; encoder / decoder / large: only that leg; "
                         "logits: --steps launches of config 4's tied-logits GEMV at --m rows; decode: --steps "
                         "config-4 decode steps, graphs off when RWQ_DECODER_GRAPHS=0 (short runs for profiling); "
                         "beam: the same as config 4's beam-5 steps (top-k, ranking, fork); attention: --steps "
                         "calls of the encoder attention at config 3's shape")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.only in ("logits", "gemv", "decode", "beam", "attention"):
            run_profile_driver(args)
            return
        if args.only in ("encoder", "decoder", "large"):
            import torch
            from rusty_whisper_b200 import quant
            torch.cuda.set_device(local_rank)
            quant.init(local_rank)
            dev, st = torch.device("cuda", local_rank), torch.cuda.current_stream()
            if args.only == "encoder":
                res = run_encoder(args, dev, peaks()[1], st, rank, world)
            elif args.only == "decoder":
                res = run_decoder_beams(args, dev, peaks()[0], st, rank, world)
            else:
                res = run_large_v3(args, dev, st, rank, world)
            if rank == 0:
                print(json.dumps({args.only: res}), flush=True)
            return
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
