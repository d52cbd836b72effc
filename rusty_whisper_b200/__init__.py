"""B200-native (sm_100a) quantized-matmul path of rusty_whisper.

The compute lives in ``librwq.so`` (CUDA kernels behind the C ABI of
``include/rwq.h``); this package is the host-side mirror of the
reference's ``quant`` module plus the seeded input generators.
"""
from .formats import QK, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, FORMATS, NAMES, block_bytes  # noqa: F401

__all__ = ["QK", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "FORMATS", "NAMES", "block_bytes"]
