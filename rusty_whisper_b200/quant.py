"""Host-side mirror of rusty_whisper's quant interface (src/quant.rs) over
the B200 kernels of ``librwq.so``.

Same names, argument meaning and failure behaviour as the reference:

* ``block_bytes(dtype)``                     quant.rs:43
* ``QTensor(shape, dtype, raw)``             quant.rs:495-576 (``new``,
  ``row_f32``, ``to_dense``)
* ``matmul_t_q(a, b) -> C = A[m,k] . B^T``    quant.rs:754
* ``linear_w(x, w, b)``                      quant.rs:1054
* ``quantize_acts_i8(a)``                    quant.rs:690

A mismatch of inner dimensions, ``k % 32 != 0`` or an unknown dtype raise
``ValueError`` (the reference panics).  Activations that are CUDA tensors
take the asynchronous device path on torch's current stream; NumPy arrays
take the host-buffer path (copy in, compute, copy out), like the
reference's ``Tensor`` in and ``Tensor`` out.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .formats import QK, block_bytes as _bb

MODE_INT8 = _lib.MODE_INT8
MODE_F32 = _lib.MODE_F32
_MODES = {"int8": MODE_INT8, "f32": MODE_F32, MODE_INT8: MODE_INT8, MODE_F32: MODE_F32}


def block_bytes(dtype: int) -> int:
    return _bb(dtype)


def _torch():
    import torch
    return torch


def _stream_ptr(device=None) -> int:
    torch = _torch()
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


class QTensor:
    """A weight kept in ggml blocks on the GPU (``QTensor``, quant.rs:495).

    ``raw`` is the ggml byte stream (bytes, a uint8 NumPy array, or a uint8
    torch tensor on the CPU or a CUDA device)."""

    def __init__(self, shape, dtype: int, raw, device: int | None = None):
        torch = _torch()
        if len(shape) != 2:
            raise ValueError(f"QTensor needs a 2-D shape, got {shape}")
        n, k = int(shape[0]), int(shape[1])
        self.shape = [n, k]
        self.dtype = int(dtype)
        L = _lib.lib()
        if device is None:
            device = torch.cuda.current_device()
        self.device = device
        h = ctypes.c_void_p()
        with torch.cuda.device(device):
            if isinstance(raw, torch.Tensor) and raw.is_cuda:
                raw = raw.contiguous()
                rc = L.rwq_qtensor_new_device(_ptr(raw), raw.numel() * raw.element_size(), self.dtype, n, k,
                                              ctypes.c_void_p(_stream_ptr()), ctypes.byref(h))
            else:
                if isinstance(raw, torch.Tensor):
                    raw = raw.numpy()
                buf = np.ascontiguousarray(np.frombuffer(raw, np.uint8) if isinstance(raw, (bytes, bytearray))
                                           else raw, dtype=np.uint8)
                rc = L.rwq_qtensor_new(buf.ctypes.data_as(ctypes.c_void_p), buf.nbytes, self.dtype, n, k,
                                       ctypes.byref(h))
        _lib.check(rc)
        self._h = h

    @classmethod
    def _borrowed(cls, handle, shape, dtype: int, device: int, owner) -> "QTensor":
        """A view of a device weight owned by ``owner`` (a loaded model):
        never freed here, and it keeps the owner alive."""
        q = cls.__new__(cls)
        q.shape = [int(shape[0]), int(shape[1])]
        q.dtype = int(dtype)
        q.device = device
        q._h = handle
        q._owner = owner
        return q

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def prepare_gemm(self) -> None:
        torch = _torch()
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().rwq_qtensor_prepare_gemm(self._h, ctypes.c_void_p(_stream_ptr())))

    def row_f32(self, i: int, out=None):
        """Dequantize row ``i`` (quant.rs:566): a CUDA tensor of ``k`` f32."""
        return self.rows_f32([i], out)[0] if out is None else self.rows_f32([i], out.view(1, -1))[0]

    def rows_f32(self, rows, out=None):
        torch = _torch()
        with torch.cuda.device(self.device):
            if isinstance(rows, torch.Tensor) and rows.is_cuda:
                idx = rows.to(torch.int32).contiguous()
            else:
                idx = torch.as_tensor(np.asarray(rows, np.int32)).cuda()
            if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= self.shape[0]):
                raise ValueError("row index out of range")
            if out is None:
                out = torch.empty((idx.numel(), self.shape[1]), dtype=torch.float32, device="cuda")
            _lib.check(_lib.lib().rwq_dequant_rows_dev(self._h, _ptr(idx), idx.numel(), _ptr(out),
                                                       ctypes.c_void_p(_stream_ptr())))
            return out

    def to_dense(self):
        """Whole-tensor dequant (quant.rs:572): CUDA f32 ``[n, k]``."""
        torch = _torch()
        with torch.cuda.device(self.device):
            out = torch.empty(tuple(self.shape), dtype=torch.float32, device="cuda")
            _lib.check(_lib.lib().rwq_dequant_rows_dev(self._h, None, self.shape[0], _ptr(out),
                                                       ctypes.c_void_p(_stream_ptr())))
            return out

    def free(self) -> None:
        if getattr(self, "_owner", None) is not None:
            self._h = None   # borrowed: the owner frees it
            return
        if getattr(self, "_h", None):
            try:
                _lib.lib().rwq_qtensor_free(self._h)
            finally:
                self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _check_mk(a_shape, b: QTensor):
    if len(a_shape) != 2:
        raise ValueError("activations must be 2-D [m, k]")
    m, k = a_shape
    if k != b.shape[1]:
        raise ValueError(f"matmul_t_q inner dims: {k} vs {b.shape[1]}")
    if k % QK:
        raise ValueError(f"k must be a multiple of {QK}")
    return int(m), int(k)


def matmul_t_q(a, b: QTensor, mode="int8", out=None, bias=None):
    """``C = A[m,k] x B^T`` with ``B`` quantized ``[n,k]`` (quant.rs:754).

    ``mode="int8"`` reproduces the reference's x86 arithmetic (int8
    activations, integer block dots); ``mode="f32"`` its dequant-then-f32
    fallback."""
    torch = _torch()
    md = _MODES[mode]
    m, k = _check_mk(tuple(a.shape), b)
    n = b.shape[0]
    L = _lib.lib()
    if isinstance(a, torch.Tensor) and a.is_cuda:
        if a.dtype != torch.float32:
            raise ValueError("activations must be float32")
        a = a.contiguous()
        with torch.cuda.device(a.device):
            if out is None:
                out = torch.empty((m, n), dtype=torch.float32, device=a.device)
            bp = None
            if bias is not None:
                bias = bias.contiguous()
                if bias.numel() != n:
                    raise ValueError("bias length must equal n")
                bp = _ptr(bias)
            _lib.check(L.rwq_matmul_t_q_dev(_ptr(a), m, k, b.handle, bp, _ptr(out), md,
                                            ctypes.c_void_p(_stream_ptr())))
        return out
    a = np.ascontiguousarray(a, np.float32)
    if out is None:
        out = np.empty((m, n), np.float32)
    bp = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, np.float32)
        if bias.size != n:
            raise ValueError("bias length must equal n")
        bp = bias.ctypes.data_as(ctypes.c_void_p)
    with torch.cuda.device(b.device):
        _lib.check(L.rwq_matmul_t_q(a.ctypes.data_as(ctypes.c_void_p), m, k, b.handle, bp,
                                    out.ctypes.data_as(ctypes.c_void_p), md))
    return out


class QActs:
    """Activations quantized once and reused against several weights (the
    Q/K/V projections of one layernormed input).  Same results as
    ``matmul_t_q`` on the same activations."""

    def __init__(self, max_m: int, k: int, device: int | None = None):
        torch = _torch()
        if k % QK:
            raise ValueError(f"k must be a multiple of {QK}")
        self.device = torch.cuda.current_device() if device is None else device
        self.max_m, self.k, self.m = int(max_m), int(k), 0
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().rwq_qacts_new(self.max_m, self.k, ctypes.byref(h)))
        self._h = h

    def quantize(self, a) -> "QActs":
        torch = _torch()
        if not (isinstance(a, torch.Tensor) and a.is_cuda and a.dtype == torch.float32):
            raise TypeError("QActs.quantize takes a CUDA float32 tensor")
        if a.dim() != 2 or a.shape[1] != self.k:
            raise ValueError(f"expected [m, {self.k}] activations, got {tuple(a.shape)}")
        a = a.contiguous()
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().rwq_qacts_quantize(self._h, _ptr(a), a.shape[0], ctypes.c_void_p(_stream_ptr())))
        self.m = int(a.shape[0])
        return self

    def matmul(self, b: "QTensor", out=None, bias=None):
        torch = _torch()
        if b.shape[1] != self.k:
            raise ValueError(f"matmul_t_q inner dims: {self.k} vs {b.shape[1]}")
        with torch.cuda.device(self.device):
            if out is None:
                out = torch.empty((self.m, b.shape[0]), dtype=torch.float32, device="cuda")
            bp = _ptr(bias.contiguous()) if bias is not None else None
            _lib.check(_lib.lib().rwq_matmul_t_q_qacts(self._h, b.handle, bp, _ptr(out),
                                                       ctypes.c_void_p(_stream_ptr())))
        return out

    def free(self) -> None:
        if getattr(self, "_h", None):
            try:
                _lib.lib().rwq_qacts_free(self._h)
            finally:
                self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def linear_w(x, w, b=None, mode="int8"):
    """``y = x W^T + b`` (quant.rs:1054) for a quantized ``W``."""
    if not isinstance(w, QTensor):
        raise TypeError("linear_w here dispatches quantized weights only; dense weights stay on the caller's path")
    return matmul_t_q(x, w, mode=mode, bias=b)


def quantize_acts_i8(a):
    """Per-32-block int8 activations (quant.rs:690): ``(q, d, sum)``."""
    torch = _torch()
    if not (isinstance(a, torch.Tensor) and a.is_cuda):
        raise TypeError("quantize_acts_i8 takes a CUDA float32 tensor")
    m, k = a.shape
    if k % QK:
        raise ValueError(f"k must be a multiple of {QK}")
    a = a.contiguous()
    q = torch.empty((m, k), dtype=torch.int8, device=a.device)
    d = torch.empty((m, k // QK), dtype=torch.float32, device=a.device)
    s = torch.empty((m, k // QK), dtype=torch.int32, device=a.device)
    with torch.cuda.device(a.device):
        _lib.check(_lib.lib().rwq_quantize_acts_dev(_ptr(a), m, k, _ptr(q), _ptr(d), _ptr(s),
                                                    ctypes.c_void_p(_stream_ptr())))
    return q, d, s


def block_dots(a, b: QTensor, path: int = 0):
    """Exact per-block integer dots ``S[m][n][k/32]`` of the int8 path.
    ``path`` 0: the dp4a core of the GEMV kernel; 1: the tensor-core GEMM."""
    torch = _torch()
    m, k = _check_mk(tuple(a.shape), b)
    a = a.contiguous()
    S = torch.empty((m, b.shape[0], k // QK), dtype=torch.int32, device=a.device)
    with torch.cuda.device(a.device):
        _lib.check(_lib.lib().rwq_block_dots_dev(_ptr(a), m, k, b.handle, _ptr(S), path,
                                                 ctypes.c_void_p(_stream_ptr())))
    return S


def set_gemm_path(path: int) -> None:
    """Kernel path of this host thread's matmuls: 0 automatic (GEMV family
    up to 256 rows; above, 2 for the int8 tier and 4 for the f32 tier),
    1 GEMV family in row chunks, 2 tensor-core GEMM
    with the weight scales folded into the operand, 3 tensor-core GEMM with
    exact per-block integer dots, 4 tensor-core GEMM with both operands
    split into f16 hi + lo and the whole K accumulated in tensor memory."""
    _lib.check(_lib.lib().rwq_set_gemm_path(path))


def set_gemv_kernel(kind: int) -> None:
    """Kernel of the GEMV family (m <= 256): 0 automatic (row-per-lane at 1-2
    rows on wide weights, integer MMA, tiled from 32 rows on), 1 dp4a, 2
    integer MMA only, 3 tiled integer MMA only, 4 row-per-lane where it
    applies.  Kinds 0, 2, 3 and 4 give bit-identical results."""
    _lib.check(_lib.lib().rwq_set_gemv_kernel(kind))


def gemv_kernel_for(w: "QTensor", m: int) -> int:
    """The GEMV kernel (1-4, as set_gemv_kernel) that an m-row call on `w`
    runs under this thread's setting."""
    r = _lib.lib().rwq_gemv_kernel_for(w._h, int(m))
    if r < 0:
        _lib.check(r)
    return r


def stream_check(stream=None) -> None:
    """Synchronize the stream and raise if a kernel recorded a fault."""
    torch = _torch()
    s = stream.cuda_stream if stream is not None else _stream_ptr()
    _lib.check(_lib.lib().rwq_stream_check(ctypes.c_void_p(s)))


def init(device: int = 0) -> None:
    _lib.check(_lib.lib().rwq_init(device))
