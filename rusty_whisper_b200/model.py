"""Host-side mirror of rusty_whisper's model loading over ``librwq.so``.

* ``load_model(path)``  model.rs:145-275 (legacy ggml container) and
  gguf.rs:156-300 (GGUF v2/v3), chosen by the file's magic
* ``HParams``           model.rs:24-56 (same fields, ``model_type``,
  ``is_multilingual``)
* ``Model``             model.rs:58-68: ``hparams``, ``mel_filters``,
  ``vocab`` (token id -> bytes), ``tensors`` (name -> weight)

Parsing runs in the library without touching the GPU.  In ``tensors`` a
2-D quantized tensor is a :class:`~rusty_whisper_b200.quant.QTensor` on the
GPU (its ggml blocks uploaded verbatim on first access); everything else is
a NumPy f32 array in row-major shape, as the reference's ``Weight::Dense``.
Malformed files raise ``ValueError`` with the library's message (the
reference returns ``io::Error``).
"""
from __future__ import annotations

import ctypes
from collections.abc import Mapping
from dataclasses import dataclass

import numpy as np

from . import _lib

_FIELDS = ("n_vocab", "n_audio_ctx", "n_audio_state", "n_audio_head", "n_audio_layer", "n_text_ctx",
           "n_text_state", "n_text_head", "n_text_layer", "n_mels", "ftype")


@dataclass(frozen=True)
class HParams:
    n_vocab: int = 0
    n_audio_ctx: int = 0
    n_audio_state: int = 0
    n_audio_head: int = 0
    n_audio_layer: int = 0
    n_text_ctx: int = 0
    n_text_state: int = 0
    n_text_head: int = 0
    n_text_layer: int = 0
    n_mels: int = 0
    ftype: int = 0

    def model_type(self) -> str:
        return {4: "tiny", 6: "base", 12: "small", 24: "medium", 32: "large"}.get(self.n_audio_layer, "unknown")

    def is_multilingual(self) -> bool:
        return self.n_vocab >= 51865


class _Tensors(Mapping):
    """name -> weight, built on access (quantized matrices go to the GPU
    the first time they are read)."""

    def __init__(self, model: "Model"):
        self._m = model
        self._cache = {}

    def _index(self, name: str) -> int:
        i = ctypes.c_int64()
        if _lib.lib().rwq_model_find(self._m._h, name.encode(), ctypes.byref(i)) != _lib.RWQ_OK:
            raise KeyError(name)
        return i.value

    def info(self, name: str):
        """(dtype, row-major shape) without materialising the tensor."""
        return self._m._info(self._index(name))[1:]

    def __getitem__(self, name: str):
        if name not in self._cache:
            self._cache[name] = self._m._weight(self._index(name))
        return self._cache[name]

    def __iter__(self):
        return iter(self._m._names())

    def __len__(self) -> int:
        return len(self._m._names())


class Model:
    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle
        L = _lib.lib()
        hp = (ctypes.c_int32 * 11)()
        _lib.check(L.rwq_model_hparams(self._h, hp))
        self.hparams = HParams(*[int(v) for v in hp])
        data = ctypes.POINTER(ctypes.c_float)()
        nm, nf = ctypes.c_int64(), ctypes.c_int64()
        _lib.check(L.rwq_model_mel_filters(self._h, ctypes.byref(data), ctypes.byref(nm), ctypes.byref(nf)))
        n = nm.value * nf.value
        self.mel_filters = (np.ctypeslib.as_array(data, (n,)).copy() if n and data else np.zeros(0, np.float32))
        self.mel_shape = (nm.value, nf.value)
        nv = ctypes.c_int64()
        _lib.check(L.rwq_model_vocab_size(self._h, ctypes.byref(nv)))
        self.vocab = []
        for i in range(nv.value):
            p, ln = ctypes.c_void_p(), ctypes.c_int64()
            _lib.check(L.rwq_model_token(self._h, i, ctypes.byref(p), ctypes.byref(ln)))
            self.vocab.append(ctypes.string_at(p, ln.value) if ln.value else b"")
        self.tensors = _Tensors(self)

    def _names(self):
        n = ctypes.c_int64()
        _lib.check(_lib.lib().rwq_model_n_tensors(self._h, ctypes.byref(n)))
        seen = {}
        for i in range(n.value):
            seen[self._info(i)[0]] = i
        return list(seen)

    def _info(self, i: int):
        name, dt, nd = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_int64 * 3)()
        _lib.check(_lib.lib().rwq_model_tensor(self._h, i, ctypes.byref(name), ctypes.byref(dt), ctypes.byref(nd),
                                               shape))
        return name.value.decode(errors="replace"), dt.value, [int(shape[d]) for d in range(nd.value)]

    def raw(self, name: str) -> bytes:
        """The verbatim ggml blocks of a quantized tensor."""
        i = self.tensors._index(name)
        p, n = ctypes.c_void_p(), ctypes.c_size_t()
        _lib.check(_lib.lib().rwq_model_tensor_raw(self._h, i, ctypes.byref(p), ctypes.byref(n)))
        return ctypes.string_at(p, n.value)

    def _weight(self, i: int):
        from .quant import QTensor
        L = _lib.lib()
        _, dt, shape = self._info(i)
        if dt not in (0, 1) and len(shape) == 2:
            import torch
            h = ctypes.c_void_p()
            _lib.check(L.rwq_model_qtensor(self._h, i, ctypes.byref(h)))
            return QTensor._borrowed(h, shape, dt, torch.cuda.current_device(), self)
        data = ctypes.POINTER(ctypes.c_float)()
        n = ctypes.c_int64()
        _lib.check(L.rwq_model_dense(self._h, i, ctypes.byref(data), ctypes.byref(n)))
        return np.ctypeslib.as_array(data, (n.value,)).copy().reshape(shape)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                _lib.lib().rwq_model_free(h)
            finally:
                self._h = None


def load_model(src) -> Model:
    """Load a ggml ``.bin`` or GGUF model from a path or from bytes."""
    L = _lib.lib()
    h = ctypes.c_void_p()
    if isinstance(src, (bytes, bytearray, memoryview)):
        buf = np.frombuffer(bytes(src), np.uint8)
        _lib.check(L.rwq_model_load_memory(buf.ctypes.data_as(ctypes.c_void_p), buf.nbytes, ctypes.byref(h)))
    else:
        _lib.check(L.rwq_model_load(str(src).encode(), ctypes.byref(h)))
    return Model(h)
