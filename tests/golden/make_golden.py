"""Regenerate the golden fixtures under tests/golden/ from the CPU oracle.

    python tests/golden/make_golden.py

The oracle (oracle/rwq_oracle.cpp) is pinned to rusty_whisper's own tests
(tests/test_oracle_pins.py); these fixtures freeze its outputs on seeded
inputs so the GPU tests can be checked against fixed numbers on any host
(the AVX2 and VNNI tiers round differently, and a GPU box may have either).
Inputs come from rusty_whisper_b200.synth (SplitMix64, documented there).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
from rusty_whisper_b200 import synth  # noqa: E402
from rusty_whisper_b200.formats import FORMATS, NAMES  # noqa: E402

CASES = [  # (m, k, n): odd shapes as quant.rs:1238, and a decoder-like GEMV batch
    (37, 96, 41),
    (5, 256, 64),
]


def make(dtype, m, k, n, seed):
    a = synth.normal(seed, m * k).reshape(m, k)
    raw = synth.random_blocks(dtype, n, k, seed + 1)
    q, d, s = oracle.quantize_acts_i8(a)
    out = dict(
        a=a, raw=raw, m=m, k=k, n=n, dtype=dtype,
        dense=oracle.to_dense(dtype, raw, n, k),
        qa=q, da=d, sa=s,
        S=oracle.block_dots(q, dtype, raw, n),
        y_int8_scalar=oracle.int8_scalar_matmul(a, dtype, raw, n),
        y_avx2=oracle.matmul_t_q(a, dtype, raw, n, tier=oracle.TIER_AVX2),
        y_f32=oracle.matmul_t_q(a, dtype, raw, n, tier=oracle.TIER_F32),
    )
    if oracle.lib().orc_has_vnni():
        out["y_vnni"] = oracle.matmul_t_q(a, dtype, raw, n, tier=oracle.TIER_VNNI)
    return out


def main():
    oracle.lib()
    for dtype in FORMATS:
        for ci, (m, k, n) in enumerate(CASES):
            fx = make(dtype, m, k, n, seed=100 * dtype + ci)
            path = os.path.join(HERE, f"{NAMES[dtype]}_m{m}_k{k}_n{n}.npz")
            np.savez_compressed(path, **fx)
            print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
