"""GGUF files through the library's native reader (libinferno_b200.so).

Mirrors GGUF.read_gguf (src/GGUF.jl:119-165): metadata by key, the tensor
table in file order, raw tensor bytes straight from the read-only mapping.
``Model.from_gguf`` uses it to upload every tensor with
``inferno_engine_load_gguf`` (pinned, double-buffered staging) instead of
copying each tensor through Python.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import InfernoError, call, lib

ENOTFOUND = -7


@dataclass(frozen=True)
class TensorInfo:
    name: str
    ggml_type: int
    ne: tuple           # ggml order (ne[0] = inner / contiguous dim), trailing 1s dropped
    nbytes: int


class GgufFile:
    def __init__(self, path):
        h = C.c_void_p()
        call("inferno_gguf_open", str(path).encode(), C.byref(h))
        self.h = h
        self.path = str(path)

    def close(self):
        if getattr(self, "h", None):
            lib().inferno_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def version(self) -> int:
        return call("inferno_gguf_version", self.h)

    @property
    def data_offset(self) -> int:
        return call("inferno_gguf_data_offset", self.h)

    def __len__(self) -> int:
        return call("inferno_gguf_n_tensors", self.h)

    def keys(self) -> list:
        n = call("inferno_gguf_n_kv", self.h)
        return [lib().inferno_gguf_key(self.h, i).decode(errors="replace") for i in range(n)]

    def __contains__(self, key: str) -> bool:
        v = C.c_int64()
        rc = lib().inferno_gguf_get_int(self.h, key.encode(), C.byref(v))
        return rc != ENOTFOUND

    def get(self, key: str, default=None):
        """The value of `key`: str, int, float, or (element type, length) for arrays."""
        k = key.encode()
        L = lib()
        s = C.c_char_p()
        if L.inferno_gguf_get_string(self.h, k, C.byref(s)) == 0:
            return s.value.decode(errors="replace")
        i = C.c_int64()
        rc = L.inferno_gguf_get_int(self.h, k, C.byref(i))
        if rc == 0:
            return int(i.value)
        if rc == ENOTFOUND:
            return default
        f = C.c_double()
        if L.inferno_gguf_get_float(self.h, k, C.byref(f)) == 0:
            return float(f.value)
        et, n = C.c_int(), C.c_int64()
        call("inferno_gguf_get_array", self.h, k, C.byref(et), C.byref(n), None)
        return (int(et.value), int(n.value))

    _ARRAY_DTYPES = {0: np.uint8, 1: np.int8, 2: np.uint16, 3: np.int16, 4: np.uint32, 5: np.int32,
                     6: np.float32, 7: np.bool_, 10: np.uint64, 11: np.int64, 12: np.float64}

    def get_array(self, key: str) -> np.ndarray:
        """A numeric array value as a numpy copy (string arrays: ValueError)."""
        et, n, data = C.c_int(), C.c_int64(), C.c_void_p()
        call("inferno_gguf_get_array", self.h, key.encode(), C.byref(et), C.byref(n), C.byref(data))
        dt = self._ARRAY_DTYPES.get(int(et.value))
        if dt is None:
            raise ValueError(f"{key}: array of element type {et.value} has no numeric view")
        if n.value == 0:
            return np.zeros(0, dt)
        nbytes = int(n.value) * np.dtype(dt).itemsize
        raw = np.ctypeslib.as_array(C.cast(data, C.POINTER(C.c_uint8)), shape=(nbytes,))
        return raw.copy().view(dt)

    def tensor(self, i: int) -> TensorInfo:
        name, t, nb = C.c_char_p(), C.c_int(), C.c_uint64()
        ne = np.ones(4, np.int64)
        call("inferno_gguf_tensor_info", self.h, i, C.byref(name), C.byref(t), ne.ctypes.data_as(C.c_void_p),
             C.byref(nb), None)
        dims = [int(d) for d in ne]
        while len(dims) > 1 and dims[-1] == 1:
            dims.pop()
        return TensorInfo(name.value.decode(errors="replace"), int(t.value), tuple(dims), int(nb.value))

    def tensors(self) -> list:
        return [self.tensor(i) for i in range(len(self))]

    def tensor_bytes(self, i: int) -> np.ndarray:
        """A copy of tensor i's raw bytes."""
        nb, data = C.c_uint64(), C.c_void_p()
        call("inferno_gguf_tensor_info", self.h, i, None, None, None, C.byref(nb), C.byref(data))
        return np.ctypeslib.as_array(C.cast(data, C.POINTER(C.c_uint8)), shape=(int(nb.value),)).copy()

    def metadata(self) -> dict:
        return {k: self.get(k) for k in self.keys()}


__all__ = ["GgufFile", "TensorInfo", "InfernoError"]
