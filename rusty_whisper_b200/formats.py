"""ggml block formats on the quantized-matmul path (quant.rs:17-131).

Every block holds ``QK = 32`` elements:

=====  ====  ==========================================  =================
dtype  code  bytes (little-endian)                       element value
=====  ====  ==========================================  =================
Q4_0   2     d:f16, qs[16]                               d*(nib-8)
Q4_1   3     d:f16, m:f16, qs[16]                        d*nib + m
Q5_0   6     d:f16, qh:u32, qs[16]                       d*((nib|h<<4)-16)
Q5_1   7     d:f16, m:f16, qh:u32, qs[16]                d*(nib|h<<4) + m
Q8_0   8     d:f16, q[32] (i8)                           d*q
=====  ====  ==========================================  =================

Element ``j < 16`` is the low nibble of ``qs[j]``; ``j >= 16`` the high
nibble of ``qs[j-16]``; bit ``j`` of ``qh`` is element ``j``'s fifth bit.
"""
from __future__ import annotations

QK = 32
Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 2, 3, 6, 7, 8
FORMATS = (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0)
NAMES = {Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1", Q8_0: "Q8_0"}
_BLOCK_BYTES = {Q4_0: 18, Q4_1: 20, Q5_0: 22, Q5_1: 24, Q8_0: 34}


def block_bytes(dtype: int) -> int:
    """Bytes per 32-element block (quant.rs:43-52).  Raises for unknown
    codes, as the reference's ``block_bytes(..).unwrap()`` panics."""
    try:
        return _BLOCK_BYTES[dtype]
    except KeyError:
        raise ValueError(f"unsupported quantized dtype {dtype}") from None


def has_min(dtype: int) -> bool:
    return dtype in (Q4_1, Q5_1)


def row_bytes(dtype: int, k: int) -> int:
    return (k // QK) * block_bytes(dtype)
