"""ctypes binding of libobjeta_b200.so (the C ABI in include/objeta_b200.h).

The shared library is built in-tree by ``objeta_b200/build.py`` (nvcc, sm_100a
only).  There is deliberately no fallback: if the library is missing or
cannot be loaded, every entry point raises, and on a machine without an
sm_100 GPU every compute call fails with a Runtime error from the library.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libobjeta_b200.so")

OK = 0
ERR_DRIVER, ERR_RUNTIME, ERR_NVRTC, ERR_IO, ERR_INVALID_INPUT, ERR_UNSUPPORTED, ERR_INTERNAL = range(1, 8)
# CudaErrorKind variant names (crates/objeta-cuda/src/lib.rs:39-48).
KIND_NAMES = {1: "Driver", 2: "Runtime", 3: "Nvrtc", 4: "Io", 5: "InvalidInput",
              6: "Unsupported", 7: "Internal"}


class CudaError(RuntimeError):
    """Mirror of the reference CudaError (lib.rs:50-60): kind, action, message."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status
        self.kind = KIND_NAMES.get(status, "Internal")
        self.message = message
        # "<Kind> error during <action> at <module>:<line> (<file>): <source_message>"
        head, _, src = message.partition("): ")
        self.source_message = src if src else message
        action = head.split(" error during ", 1)[-1]
        self.action = action.rsplit(" at ", 1)[0]


_lock = threading.Lock()
_lib = None

c_size = ctypes.c_size_t
c_int = ctypes.c_int
c_void_p = ctypes.c_void_p
c_float_p = ctypes.POINTER(ctypes.c_float)


class FormatInfo(ctypes.Structure):
    _fields_ = [("block_size", ctypes.c_uint32), ("block_bytes", ctypes.c_uint32),
                ("packed_values_per_byte", ctypes.c_uint32), ("kernel_name", ctypes.c_char_p),
                ("format_label", ctypes.c_char_p), ("scale_dtype", ctypes.c_char_p),
                ("nibble_order", ctypes.c_char_p)]


class QGemvShapeC(ctypes.Structure):
    _fields_ = [(n, c_size) for n in ("rows", "cols", "block_size", "block_bytes", "blocks_per_row",
                                      "quantized_row_bytes", "quantized_matrix_bytes")]


class DeviceInfo(ctypes.Structure):
    _fields_ = [("ordinal", c_int), ("total_global_mem_bytes", c_size),
                ("compute_capability_major", c_int), ("compute_capability_minor", c_int),
                ("multiprocessor_count", c_int), ("l2_cache_bytes", c_size)]


class QGemvTelemetryC(ctypes.Structure):
    _fields_ = [("h2d_ms", ctypes.c_float), ("kernel_ms", ctypes.c_float), ("d2h_ms", ctypes.c_float),
                ("unaccounted_ms", ctypes.c_float), ("total_ms", ctypes.c_float),
                ("bytes_read", c_size), ("effective_gbps", ctypes.c_float)]


# name -> (restype, argtypes)
_SIGS = {
    "objb_last_error": (c_int, [ctypes.c_char_p, c_size]),
    "objb_abi_version": (c_int, []),
    "objb_format_info_get": (c_int, [c_int, ctypes.POINTER(FormatInfo)]),
    "objb_qgemv_shape_new": (c_int, [c_int, c_size, c_size, ctypes.POINTER(QGemvShapeC)]),
    "objb_device_info_get": (c_int, [c_int, ctypes.POINTER(DeviceInfo)]),
    "objb_device_error_take": (c_int, [c_int, ctypes.POINTER(ctypes.c_uint)]),
    "objb_host_register": (c_int, [c_void_p, c_size]),
    "objb_host_unregister": (c_int, [c_void_p]),
    "objb_quant_backend_new": (c_int, [c_int, ctypes.POINTER(c_void_p)]),
    "objb_quant_backend_free": (None, [c_void_p]),
    "objb_quant_backend_compile_format": (c_int, [c_void_p, c_int]),
    "objb_gemv_host": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_size, c_void_p, c_size,
                               c_size, c_size, c_void_p, ctypes.POINTER(QGemvTelemetryC)]),
    "objb_gemv_device": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_size, c_size, c_void_p]),
    "objb_gemv_fp4_split_device": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_size, c_size,
                                           c_void_p]),
    "objb_gemv_bf16_device": (c_int, [c_void_p, c_void_p, c_void_p, c_size, c_size, c_void_p]),
    "objb_pipe_plan_info": (c_int, [c_int, c_int, c_size, c_size, c_int, c_int, c_int,
                                    ctypes.POINTER(ctypes.c_int32), c_int]),
    "objb_compare_outputs": (c_int, [c_void_p, c_size, c_void_p, c_size, c_void_p]),
    "objb_act_quant_device": (c_int, [c_void_p, c_size, c_size, c_void_p, c_void_p, c_void_p]),
    "objb_gemv_fp8_fp4_device": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size, c_size,
                                         c_void_p]),
    "objb_gemv_fp8_fp8_device": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size, c_size,
                                         c_void_p]),
    "objb_ffn_bf16_device": (c_int, [c_void_p, c_void_p, c_void_p, c_size, c_size, c_size, c_void_p, c_void_p,
                                     c_int, ctypes.c_float, c_void_p]),
    "objb_quantize_matrix_device": (c_int, [c_int, c_void_p, c_size, c_size, c_void_p, c_void_p]),
    "objb_fp4_decode_split_device": (c_int, [c_void_p, c_void_p, c_size, c_size, c_void_p, c_void_p]),
}


def register_signatures(sigs: dict) -> None:
    """Adds signatures of entry points declared by other modules."""
    _SIGS.update(sigs)
    if _lib is not None:
        _bind(_lib, sigs)


def _bind(lib, sigs):
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def load():
    """Loads the library (once).  Raises ImportError if it is missing."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m objeta_b200.build` "
                    "(nvcc, sm_100a).  There is no CPU fallback.")
            lib = ctypes.CDLL(LIB_PATH)
            _bind(lib, _SIGS)
            _lib = lib
    return _lib


def last_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(4096)
    st = load().objb_last_error(buf, len(buf))
    return st, buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != OK:
        st, msg = last_error()
        raise CudaError(status, msg or f"status {status}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def stream_handle(stream) -> int | None:
    """Accepts None (legacy default stream), an int handle, or a torch stream."""
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    h = getattr(stream, "cuda_stream", None)
    if h is None:
        raise TypeError(f"cannot use {stream!r} as a CUDA stream")
    return int(h)
