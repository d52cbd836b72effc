"""ctypes binding of ``librwq.so`` (the C ABI declared in include/rwq.h).

The library is built in-tree (``python -m rusty_whisper_b200.build``).  If
it is missing this module raises: there is no CPU or eager fallback.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "librwq.so")

RWQ_OK = 0
RWQ_ERR_ARG, RWQ_ERR_DTYPE, RWQ_ERR_SHAPE, RWQ_ERR_CUDA = -1, -2, -3, -4
RWQ_ERR_NOMEM, RWQ_ERR_DEVICE, RWQ_ERR_NOGPU = -5, -6, -7
MODE_INT8, MODE_F32 = 0, 1

# Every symbol include/rwq.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_SZ = ctypes.c_size_t
SIGNATURES = {
    "rwq_block_bytes": (_I, [_I]),
    "rwq_last_error": (ctypes.c_char_p, []),
    "rwq_init": (_I, [_I]),
    "rwq_qtensor_new": (_I, [_P, _SZ, _I, _L, _L, ctypes.POINTER(_P)]),
    "rwq_qtensor_new_device": (_I, [_P, _SZ, _I, _L, _L, _P, ctypes.POINTER(_P)]),
    "rwq_qtensor_free": (_I, [_P]),
    "rwq_qtensor_shape": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_L), ctypes.POINTER(_L)]),
    "rwq_qtensor_prepare_gemm": (_I, [_P, _P]),
    "rwq_matmul_t_q": (_I, [_P, _L, _L, _P, _P, _P, _I]),
    "rwq_matmul_t_q_dev": (_I, [_P, _L, _L, _P, _P, _P, _I, _P]),
    "rwq_dequant_rows_dev": (_I, [_P, _P, _L, _P, _P]),
    "rwq_row_f32": (_I, [_P, _L, _P]),
    "rwq_quantize_acts_dev": (_I, [_P, _L, _L, _P, _P, _P, _P]),
    "rwq_block_dots_dev": (_I, [_P, _L, _L, _P, _P, _I, _P]),
    "rwq_qacts_new": (_I, [_L, _L, ctypes.POINTER(_P)]),
    "rwq_qacts_free": (_I, [_P]),
    "rwq_qacts_quantize": (_I, [_P, _P, _L, _P]),
    "rwq_matmul_t_q_qacts": (_I, [_P, _P, _P, _P, _P]),
    "rwq_matmul_t_q_noalloc": (_I, [_P, _L, _L, _P, _P, _P, _P]),
    "rwq_set_gemm_path": (_I, [_I]),
    "rwq_set_gemv_kernel": (_I, [_I]),
    "rwq_gemv_kernel_for": (_I, [_P, _L]),
    "rwq_stream_check": (_I, [_P]),
    "rwq_mma_peak": (_I, [_I, ctypes.c_longlong, _I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]),
    "rwq_model_load": (_I, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    "rwq_model_load_memory": (_I, [_P, _SZ, ctypes.POINTER(_P)]),
    "rwq_model_free": (_I, [_P]),
    "rwq_model_hparams": (_I, [_P, ctypes.POINTER(ctypes.c_int32)]),
    "rwq_model_mel_filters": (_I, [_P, ctypes.POINTER(ctypes.POINTER(ctypes.c_float)), ctypes.POINTER(_L),
                                   ctypes.POINTER(_L)]),
    "rwq_model_vocab_size": (_I, [_P, ctypes.POINTER(_L)]),
    "rwq_model_token": (_I, [_P, _L, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(_L)]),
    "rwq_model_n_tensors": (_I, [_P, ctypes.POINTER(_L)]),
    "rwq_model_find": (_I, [_P, ctypes.c_char_p, ctypes.POINTER(_L)]),
    "rwq_model_tensor": (_I, [_P, _L, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_I), ctypes.POINTER(_I),
                              ctypes.POINTER(_L)]),
    "rwq_model_tensor_raw": (_I, [_P, _L, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(_SZ)]),
    "rwq_model_qtensor": (_I, [_P, _L, ctypes.POINTER(_P)]),
    "rwq_model_dense": (_I, [_P, _L, ctypes.POINTER(ctypes.POINTER(ctypes.c_float)), ctypes.POINTER(_L)]),
    "rwq_mel_filterbank": (_I, [_I, _I, _I, _P]),
    "rwq_mel_new": (_I, [_P, _I, ctypes.POINTER(_P)]),
    "rwq_mel_free": (_I, [_P]),
    "rwq_log_mel_dev": (_I, [_P, _P, _L, _L, _P, _P]),
    "rwq_log_mel": (_I, [_P, _P, _L, _P]),
    "rwq_encoder_new": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(_P)]),
    "rwq_encoder_free": (_I, [_P]),
    "rwq_encoder_set_dense": (_I, [_P, ctypes.c_char_p, _P, _L]),
    "rwq_encoder_set_quant": (_I, [_P, ctypes.c_char_p, _I, _P, _SZ, _L, _L]),
    "rwq_encoder_encode_dev": (_I, [_P, _P, _L, _P, _P]),
    "rwq_encoder_encode": (_I, [_P, _P, _L, _P]),
    "rwq_attention_dev": (_I, [_P, _P, _P, _L, _L, _L, _L, _P, _P]),
    "rwq_conv1d_dev": (_I, [_P, _L, _L, _L, _P, _L, _P, _I, _P, _P]),
    "rwq_layer_norm_dev": (_I, [_P, _P, _P, _P, _P, _L, _L, _P, _P, _P, _P, _P]),
    "rwq_decoder_new": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(_P)]),
    "rwq_decoder_free": (_I, [_P]),
    "rwq_decoder_set_dense": (_I, [_P, ctypes.c_char_p, _P, _L]),
    "rwq_decoder_set_quant": (_I, [_P, ctypes.c_char_p, _I, _P, _SZ, _L, _L]),
    "rwq_decoder_begin": (_I, [_P, _P, _L, _L, _P, _L, _P]),
    "rwq_decoder_step": (_I, [_P, _P, _P, _P, ctypes.c_int32, _P]),
    "rwq_decoder_step_hidden": (_I, [_P, _P, _P, _P]),
    "rwq_decoder_project": (_I, [_P, _P, _L, _P, _P]),
    "rwq_decoder_fork": (_I, [_P, _P, _P]),
    "rwq_beam_topk": (_I, [_P, _L, _L, ctypes.c_int32, _I, _P, _P, _P]),
    "rwq_beam_select": (_I, [_P, _P, _I, _P, _P, _L, _I, _I, _P, _P, _P, _P, _P, _P]),
    "rwq_decoder_reset": (_I, [_P]),
    "rwq_decoder_n_past": (_I, [_P, ctypes.POINTER(_L)]),
}

_lib = None


class RwqError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"rwq status {code}: {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m rusty_whisper_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != RWQ_OK:
        msg = lib().rwq_last_error().decode(errors="replace")
        if rc in (RWQ_ERR_ARG, RWQ_ERR_SHAPE):
            raise ValueError(f"rwq status {rc}: {msg}")
        if rc == RWQ_ERR_DTYPE:
            raise ValueError(f"rwq status {rc}: {msg}")
        raise RwqError(rc, msg)
