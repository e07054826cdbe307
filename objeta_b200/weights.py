"""ModelWeights (crates/objeta-parser/src/lib.rs:97-330) over the library's
safetensors loader: mmap of a file or a shard directory, tensor index, raw
views, f32 conversion, and pinning so expert uploads through the
``CudaExpertCache`` (or ``to_device``) are asynchronous DMA from the mapping.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from .quant import _dev_ptr

c_size = ctypes.c_size_t
c_int = ctypes.c_int
c_void_p = ctypes.c_void_p

DTYPES = ["F32", "F16", "BF16", "I64", "I32", "I8", "U8", "F8_E8M0", "F8_E4M3", "BOOL"]
_NP = {"F32": np.float32, "F16": np.uint16, "BF16": np.uint16, "I64": np.int64, "I32": np.int32, "I8": np.int8,
       "U8": np.uint8, "F8_E8M0": np.uint8, "F8_E4M3": np.uint8, "BOOL": np.uint8}


class _InfoC(ctypes.Structure):
    _fields_ = [("dtype", c_int), ("ndim", c_int), ("shape", c_size * 8), ("offset", c_size), ("nbytes", c_size),
                ("nelem", c_size)]


_lib.register_signatures({
    "objb_weights_open": (c_int, [ctypes.c_char_p, ctypes.POINTER(c_void_p)]),
    "objb_weights_close": (None, [c_void_p]),
    "objb_weights_count": (c_int, [c_void_p, ctypes.POINTER(c_size)]),
    "objb_weights_name_at": (c_int, [c_void_p, c_size, ctypes.POINTER(ctypes.c_char_p)]),
    "objb_weights_info": (c_int, [c_void_p, ctypes.c_char_p, ctypes.POINTER(_InfoC)]),
    "objb_weights_raw": (c_int, [c_void_p, ctypes.c_char_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_size)]),
    "objb_weights_get_f32": (c_int, [c_void_p, ctypes.c_char_p, c_void_p, c_size]),
    "objb_weights_pin": (c_int, [c_void_p]),
    "objb_weights_to_device": (c_int, [c_void_p, ctypes.c_char_p, c_void_p, c_size, c_void_p]),
})


@dataclass
class TensorInfo:
    """lib.rs:21-28."""
    dtype: str
    shape: list
    offset: int
    nbytes: int
    nelem: int


class ModelWeights:
    """Lazy mmap access to safetensors weights (ModelWeights::open)."""

    def __init__(self, path):
        h = c_void_p()
        _lib.call("objb_weights_open", str(path).encode(), ctypes.byref(h))
        self._h = h

    @classmethod
    def open(cls, path) -> "ModelWeights":
        return cls(path)

    def close(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            _lib.load().objb_weights_close(h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        n = c_size()
        _lib.call("objb_weights_count", self._h, ctypes.byref(n))
        return int(n.value)

    def is_empty(self) -> bool:
        return len(self) == 0

    def keys(self) -> list:
        out = []
        for i in range(len(self)):
            p = ctypes.c_char_p()
            _lib.call("objb_weights_name_at", self._h, i, ctypes.byref(p))
            out.append(p.value.decode())
        return out

    def contains(self, name: str) -> bool:
        return self.info(name) is not None

    def info(self, name: str):
        c = _InfoC()
        st = _lib.load().objb_weights_info(self._h, name.encode(), ctypes.byref(c))
        if st != _lib.OK:
            return None
        return TensorInfo(DTYPES[c.dtype], [int(c.shape[i]) for i in range(c.ndim)], int(c.offset), int(c.nbytes),
                          int(c.nelem))

    def get_raw(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 view of the mapping."""
        p, n = c_void_p(), c_size()
        _lib.call("objb_weights_raw", self._h, name.encode(), ctypes.byref(p), ctypes.byref(n))
        if n.value == 0:
            return np.zeros(0, np.uint8)
        buf = (ctypes.c_uint8 * n.value).from_address(p.value)
        a = np.frombuffer(buf, dtype=np.uint8)
        a.flags.writeable = False
        return a

    def get_array(self, name: str) -> np.ndarray:
        """The raw tensor typed by its dtype (F16 / BF16 as uint16 bits) and shaped."""
        info = self.info(name)
        if info is None:
            raise _lib.CudaError(5, f"InvalidInput error during get tensor at objeta_b200::weights.py (weights.py): "
                                    f"missing tensor: {name}")
        return self.get_raw(name).view(_NP[info.dtype]).reshape(info.shape)

    def get_f32(self, name: str) -> np.ndarray:
        info = self.info(name)
        n = info.nbytes // {"F32": 4, "F16": 2, "BF16": 2}.get(info.dtype, 1) if info else 0
        out = np.zeros(n, np.float32)
        _lib.call("objb_weights_get_f32", self._h, name.encode(), out.ctypes.data, out.size)
        return out

    def get_matrix(self, name: str):
        """(rows, cols, row-major f32) of a 2-D tensor."""
        info = self.info(name)
        if info is None or len(info.shape) != 2:
            raise _lib.CudaError(5, f"InvalidInput error during get matrix at objeta_b200::weights.py "
                                    f"(weights.py): expected 2D tensor for {name}")
        return info.shape[0], info.shape[1], self.get_f32(name)

    def pin(self):
        """Pins the mappings for asynchronous host-to-device copies."""
        _lib.call("objb_weights_pin", self._h)

    def to_device(self, name: str, d_dst, stream=None):
        _lib.call("objb_weights_to_device", self._h, name.encode(), _dev_ptr(d_dst),
                  d_dst.numel() * d_dst.element_size(), _lib.stream_handle(stream))
        return d_dst
