"""GGUF model files through smeai_gguf.h: tensor table, metadata, raw tensor
bytes, and Q2_K tensors loaded straight into the device tile layout."""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import QK_K, Q2K_BLOCK_BYTES, SmeaiError, check, lib

GGML_F32, GGML_F16, GGML_Q2_K, GGML_Q3_K, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_K = 0, 1, 10, 11, 12, 13, 14, 15


@dataclass
class TensorInfo:
    index: int
    name: str
    ggml_type: int
    shape: tuple          # ne[0..n_dims-1], innermost first (ggml order)
    offset: int           # relative to the data section
    nbytes: int


class GGUFFile:
    """A parsed GGUF file (smeai_gguf_open); tensor data stays in the file."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        check(lib().smeai_gguf_open(str(path).encode(), ctypes.byref(h)), f"gguf_open({path})")
        self.handle = h
        self.path = str(path)
        self.version = lib().smeai_gguf_version(h)
        self.alignment = lib().smeai_gguf_alignment(h)
        self.data_offset = lib().smeai_gguf_data_offset(h)
        self.tensors = [self._info(i) for i in range(lib().smeai_gguf_n_tensors(h))]
        self.by_name = {t.name: t for t in self.tensors}

    def _info(self, i: int) -> TensorInfo:
        name, typ, nd = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
        ne = (ctypes.c_int64 * 4)()
        off, nb = ctypes.c_uint64(), ctypes.c_uint64()
        check(lib().smeai_gguf_tensor_info(self.handle, i, ctypes.byref(name), ctypes.byref(typ), ctypes.byref(nd),
                                           ne, ctypes.byref(off), ctypes.byref(nb)), "gguf_tensor_info")
        return TensorInfo(i, name.value.decode(), typ.value, tuple(ne[d] for d in range(nd.value)), off.value,
                          nb.value)

    def find(self, name: str) -> int:
        return lib().smeai_gguf_find_tensor(self.handle, name.encode())

    def read(self, name: str) -> np.ndarray:
        """Raw bytes of a tensor (ggml's block layout), uint8."""
        t = self.by_name[name]
        out = np.empty(t.nbytes, dtype=np.uint8)
        check(lib().smeai_gguf_read_tensor(self.handle, t.index, out.ctypes.data, t.nbytes), f"gguf_read({name})")
        return out

    def load_q2k(self, name: str):
        """A 2-D Q2_K tensor as a device Q2KMatrix (rows = shape[1], k = shape[0])."""
        from .q2k import Q2KMatrix
        t = self.by_name[name]
        h = ctypes.c_void_p()
        check(lib().smeai_gguf_load_q2k(self.handle, t.index, ctypes.byref(h)), f"gguf_load_q2k({name})")
        return Q2KMatrix.from_handle(h, t.shape[1], t.shape[0])

    def load_q3k(self, name: str):
        """A 2-D Q3_K tensor as a device Q3KMatrix."""
        from .q2k import Q3KMatrix
        t = self.by_name[name]
        h = ctypes.c_void_p()
        check(lib().smeai_gguf_load_q3k(self.handle, t.index, ctypes.byref(h)), f"gguf_load_q3k({name})")
        return Q3KMatrix(None, t.shape[1], t.shape[0], handle=h)

    def load_q6k(self, name: str):
        """A 2-D Q6_K tensor as a device Q6KMatrix."""
        from .q2k import Q6KMatrix
        t = self.by_name[name]
        h = ctypes.c_void_p()
        check(lib().smeai_gguf_load_q6k(self.handle, t.index, ctypes.byref(h)), f"gguf_load_q6k({name})")
        return Q6KMatrix(None, t.shape[1], t.shape[0], handle=h)

    def key_type(self, key: str) -> int:
        return lib().smeai_gguf_key_type(self.handle, key.encode())

    def get_int(self, key: str) -> int:
        v = ctypes.c_uint64()
        check(lib().smeai_gguf_get_u64(self.handle, key.encode(), ctypes.byref(v)), f"gguf_get_u64({key})")
        return v.value

    def get_float(self, key: str) -> float:
        v = ctypes.c_double()
        check(lib().smeai_gguf_get_f64(self.handle, key.encode(), ctypes.byref(v)), f"gguf_get_f64({key})")
        return v.value

    def get_str(self, key: str) -> str:
        v = ctypes.c_char_p()
        check(lib().smeai_gguf_get_str(self.handle, key.encode(), ctypes.byref(v)), f"gguf_get_str({key})")
        return v.value.decode()

    def n_kv(self) -> int:
        return lib().smeai_gguf_n_kv(self.handle)

    def close(self):
        if getattr(self, "handle", None) and self.handle.value:
            lib().smeai_gguf_close(self.handle)
            self.handle = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["GGUFFile", "TensorInfo", "GGML_F32", "GGML_F16", "GGML_Q2_K", "GGML_Q3_K", "GGML_Q6_K", "SmeaiError"]
