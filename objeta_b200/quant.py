"""QuantFormat / QGemvShape / QuantBackend: the host-side mirror of objeta's
``crates/objeta-cuda/src/quant.rs`` over the C ABI of libobjeta_b200.so.

Names, argument meaning and errors follow the reference Rust API so code and
tests written against it read the same here:

* ``QuantFormat`` (quant.rs:25-96) with its metadata methods;
* ``QGemvShape`` (quant.rs:98-143);
* ``QuantBackend.new / compile_format / gemv / q4_gemv / q5_gemv``
  (quant.rs:202-322): host arrays in, host result out, H2D + kernel + D2H;
* ``QuantBackend.launch_kernel / launch_kernel_split_fp4`` (quant.rs:324-408):
  device tensors, asynchronous on a stream;
* ``QuantBackend.quantize_matrix`` (quant.rs:239-253): the reference packs on
  the CPU; here the packer runs on the GPU and is byte-identical.

All compute goes through the CUDA library; there is no CPU path.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass

import numpy as np

from . import _lib


class QuantFormat(enum.IntEnum):
    Q4_0 = 0
    Q5_0 = 1
    IQ3_0 = 2
    DeepSeekFp4E2M1 = 3

    def _info(self) -> _lib.FormatInfo:
        info = _lib.FormatInfo()
        _lib.call("objb_format_info_get", int(self), ctypes.byref(info))
        return info

    def block_size(self) -> int:
        return 32

    def block_bytes(self) -> int:
        return {0: 18, 1: 22, 2: 14, 3: 17}[int(self)]

    def kernel_name(self) -> str:
        return {0: "q4_gemv", 1: "q5_gemv", 2: "iq3_gemv", 3: "fp4_e2m1_gemv"}[int(self)]

    def format_label(self) -> str:
        return {0: "q4_0", 1: "q5_0", 2: "iq3_0", 3: "deepseek_fp4_e2m1"}[int(self)]

    def packed_values_per_byte(self) -> int:
        return 2

    def scale_dtype(self) -> str:
        return "F8_E8M0" if self == QuantFormat.DeepSeekFp4E2M1 else "F16"

    def nibble_order(self) -> str:
        return "low_first"


@dataclass(frozen=True)
class QGemvShape:
    rows: int
    cols: int
    block_size: int
    block_bytes: int

    @staticmethod
    def new(fmt: QuantFormat, rows: int, cols: int) -> "QGemvShape":
        fmt = QuantFormat(fmt)
        return QGemvShape(rows, cols, fmt.block_size(), fmt.block_bytes())

    @staticmethod
    def q4_0(rows, cols):
        return QGemvShape.new(QuantFormat.Q4_0, rows, cols)

    @staticmethod
    def q5_0(rows, cols):
        return QGemvShape.new(QuantFormat.Q5_0, rows, cols)

    @staticmethod
    def iq3_0(rows, cols):
        return QGemvShape.new(QuantFormat.IQ3_0, rows, cols)

    @staticmethod
    def deepseek_fp4(rows, cols):
        return QGemvShape.new(QuantFormat.DeepSeekFp4E2M1, rows, cols)

    def blocks_per_row(self) -> int:
        return self.cols // self.block_size

    def quantized_row_bytes(self) -> int:
        return self.blocks_per_row() * self.block_bytes

    def quantized_matrix_bytes(self) -> int:
        return self.rows * self.quantized_row_bytes()


@dataclass
class QGemvTelemetry:
    """quant.rs:145-154."""
    h2d_ms: float = 0.0
    kernel_ms: float = 0.0
    d2h_ms: float = 0.0
    unaccounted_ms: float = 0.0
    total_ms: float = 0.0
    bytes_read: int = 0
    effective_gbps: float = 0.0


def _validate_shape_metadata(fmt: QuantFormat, shape: QGemvShape) -> None:
    # quant.rs:791-812
    if shape.block_size != fmt.block_size() or shape.block_bytes != fmt.block_bytes():
        raise _lib.CudaError(
            _lib.ERR_INVALID_INPUT,
            f"InvalidInput error during validate {fmt.format_label()} shape constants at "
            f"objeta_b200::quant.py (quant.py): expected block_size={fmt.block_size()} "
            f"block_bytes={fmt.block_bytes()}, got block_size={shape.block_size} "
            f"block_bytes={shape.block_bytes}")


def _dev_ptr(t) -> int:
    """Device pointer of a contiguous CUDA torch tensor (or an int address)."""
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


class QuantBackend:
    """QuantBackend (quant.rs:192-504) bound to one CUDA device ordinal."""

    def __init__(self, device: int = 0):
        self.device = int(device)
        h = ctypes.c_void_p()
        _lib.call("objb_quant_backend_new", self.device, ctypes.byref(h))
        self._h = h

    @classmethod
    def new(cls, device: int = 0) -> "QuantBackend":
        return cls(device)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.load().objb_quant_backend_free(h)
            except Exception:
                pass
            self._h = None

    def status(self) -> None:
        return None

    def compile_format(self, fmt: QuantFormat) -> None:
        _lib.call("objb_quant_backend_compile_format", self._h, int(QuantFormat(fmt)))

    # ---- packing (quant.rs:239-253) on the device
    def quantize_matrix(self, fmt: QuantFormat, matrix, shape: QGemvShape) -> np.ndarray:
        import torch
        fmt = QuantFormat(fmt)
        _validate_shape_metadata(fmt, shape)
        if shape.cols % shape.block_size != 0:
            raise _lib.CudaError(
                _lib.ERR_INVALID_INPUT,
                f"InvalidInput error during validate {fmt.format_label()} column alignment at "
                f"objeta_b200::quant.py (quant.py): cols {shape.cols} must be a multiple of "
                f"block_size {shape.block_size}")
        m = torch.as_tensor(np.ascontiguousarray(matrix, dtype=np.float32)).reshape(-1)
        if m.numel() != shape.rows * shape.cols:
            raise _lib.CudaError(
                _lib.ERR_INVALID_INPUT,
                f"InvalidInput error during validate dense matrix size for {fmt.format_label()} at "
                f"objeta_b200::quant.py (quant.py): matrix len {m.numel()} != rows*cols "
                f"{shape.rows * shape.cols}")
        with torch.cuda.device(self.device):
            dm = m.to(f"cuda:{self.device}")
            out = self.quantize_matrix_device(fmt, dm, shape)
            return out.cpu().numpy()

    def quantize_matrix_device(self, fmt: QuantFormat, d_matrix, shape: QGemvShape, stream=None,
                               out=None):
        """Packs a device f32 matrix; returns a device uint8 tensor."""
        import torch
        fmt = QuantFormat(fmt)
        if out is None:
            out = torch.empty(shape.quantized_matrix_bytes(), dtype=torch.uint8, device=d_matrix.device)
        with torch.cuda.device(d_matrix.device):
            _lib.call("objb_quantize_matrix_device", int(fmt), _dev_ptr(d_matrix), shape.rows,
                      shape.cols, _dev_ptr(out), _lib.stream_handle(
                          stream if stream is not None else torch.cuda.current_stream()))
        return out

    def q4_quantize_matrix(self, matrix, shape):
        return self.quantize_matrix(QuantFormat.Q4_0, matrix, shape)

    def q5_quantize_matrix(self, matrix, shape):
        return self.quantize_matrix(QuantFormat.Q5_0, matrix, shape)

    # ---- host-slice GEMV (quant.rs:256-302)
    def gemv(self, fmt: QuantFormat, stream, qweights, x, shape: QGemvShape):
        fmt = QuantFormat(fmt)
        _validate_shape_metadata(fmt, shape)
        qw = np.ascontiguousarray(qweights, dtype=np.uint8).reshape(-1)
        xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        y = np.zeros(shape.rows, dtype=np.float32)
        tel = _lib.QGemvTelemetryC()
        _lib.call("objb_gemv_host", self._h, int(fmt), _lib.stream_handle(stream),
                  qw.ctypes.data, qw.size, xv.ctypes.data, xv.size, shape.rows, shape.cols,
                  y.ctypes.data, ctypes.byref(tel))
        t = QGemvTelemetry(tel.h2d_ms, tel.kernel_ms, tel.d2h_ms, tel.unaccounted_ms,
                           tel.total_ms, tel.bytes_read, tel.effective_gbps)
        return y, t

    def q4_gemv(self, stream, qweights, x, shape):
        return self.gemv(QuantFormat.Q4_0, stream, qweights, x, shape)

    def q5_gemv(self, stream, qweights, x, shape):
        return self.gemv(QuantFormat.Q5_0, stream, qweights, x, shape)

    # ---- device GEMV (quant.rs:324-408)
    def launch_kernel(self, fmt: QuantFormat, stream, d_qweights, d_x, d_y, shape: QGemvShape):
        fmt = QuantFormat(fmt)
        _lib.call("objb_gemv_device", int(fmt), _dev_ptr(d_qweights), _dev_ptr(d_x), _dev_ptr(d_y),
                  shape.rows, shape.cols, _lib.stream_handle(stream))

    def launch_kernel_split_fp4(self, stream, d_weight, d_scale, d_x, d_y, rows, cols):
        _lib.call("objb_gemv_fp4_split_device", _dev_ptr(d_weight), _dev_ptr(d_scale),
                  _dev_ptr(d_x), _dev_ptr(d_y), rows, cols, _lib.stream_handle(stream))


def gemv_device(fmt, d_qweights, d_x, d_y, rows, cols, stream=None):
    """objb_gemv_device on torch tensors."""
    _lib.call("objb_gemv_device", int(QuantFormat(fmt)), _dev_ptr(d_qweights), _dev_ptr(d_x),
              _dev_ptr(d_y), rows, cols, _lib.stream_handle(stream))


def gemv_bf16_device(d_w, d_x, d_y, rows, cols, stream=None):
    """objb_gemv_bf16_device: dense bf16 weights (any 16-bit tensor holding
    bf16 bits) times f32 x."""
    _lib.call("objb_gemv_bf16_device", _dev_ptr(d_w), _dev_ptr(d_x), _dev_ptr(d_y), rows, cols,
              _lib.stream_handle(stream))


def pipe_plan_info(fmt, rows, cols, split_fp4=False, blocks_per_lane=2, dual=False, moe_program=False):
    """How the pipelined kernel streams a rows x cols matrix (host arithmetic,
    no GPU): warps per row, row groups, rows per stage, ring slots, bytes per
    slot, dynamic shared memory, the rows per stage that keep every row group
    busy, whether an aligned x is formed in-kernel, and the ring budget."""
    import ctypes
    out = (ctypes.c_int32 * 9)()
    _lib.call("objb_pipe_plan_info", int(QuantFormat(fmt)), int(bool(split_fp4)), int(rows), int(cols),
              int(blocks_per_lane), int(bool(dual)), int(bool(moe_program)), out, 9)
    keys = ("nseg", "ngrp", "rows_per_stage", "slots", "slot_bytes", "smem_bytes", "busy_quantum",
            "x_in_kernel", "ring_budget")
    return {k: int(v) for k, v in zip(keys, out)}


def gemv_fp4_split_device(d_weight, d_scale, d_x, d_y, rows, cols, stream=None):
    _lib.call("objb_gemv_fp4_split_device", _dev_ptr(d_weight), _dev_ptr(d_scale), _dev_ptr(d_x),
              _dev_ptr(d_y), rows, cols, _lib.stream_handle(stream))


def fp4_decode_split_device(d_weight, d_scale, rows, cols, d_out, stream=None):
    """decode_deepseek_fp4_to_f32 (objeta-parser deepseek.rs:862-918) on the GPU."""
    _lib.call("objb_fp4_decode_split_device", _dev_ptr(d_weight), _dev_ptr(d_scale), rows, cols,
              _dev_ptr(d_out), _lib.stream_handle(stream))


def device_error_take(device: int = 0) -> int:
    w = ctypes.c_uint(0)
    _lib.call("objb_device_error_take", device, ctypes.byref(w))
    return int(w.value)


@dataclass
class QGemvNumerics:
    """quant.rs:156-161."""
    cosine_similarity: float
    relative_l2_error: float
    max_abs_error: float


class _NumericsC(ctypes.Structure):
    _fields_ = [("cosine_similarity", ctypes.c_float), ("relative_l2_error", ctypes.c_float),
                ("max_abs_error", ctypes.c_float)]


def compare_outputs(reference, actual) -> QGemvNumerics:
    """compare_outputs (quant.rs:676-723) through objb_compare_outputs: cosine
    and relative L2 from f64 sums in element order, f32 max-abs error."""
    r = np.ascontiguousarray(reference, dtype=np.float32).reshape(-1)
    a = np.ascontiguousarray(actual, dtype=np.float32).reshape(-1)
    out = _NumericsC()
    _lib.call("objb_compare_outputs", r.ctypes.data, r.size, a.ctypes.data, a.size, ctypes.byref(out))
    return QGemvNumerics(float(out.cosine_similarity), float(out.relative_l2_error), float(out.max_abs_error))


q4_compare = q5_compare = fp4_compare = compare_outputs


# ---------------------------------------------------- official DeepSeek activation path
def act_quant_device(d_x, rows: int, cols: int, stream=None):
    """cuda_act_quant_device (quant.rs:1229-1282): rows x cols f32 on the
    device -> (E4M3 codes uint8 [rows*cols], E8M0 scales uint8 [rows*cols/128]),
    bit-identical to the reference CPU act_quant."""
    import torch
    vals = torch.empty(rows * cols, dtype=torch.uint8, device=d_x.device)
    scales = torch.empty(max(1, rows * cols // 128), dtype=torch.uint8, device=d_x.device)
    _lib.call("objb_act_quant_device", _dev_ptr(d_x), rows, cols, _dev_ptr(vals), _dev_ptr(scales),
              _lib.stream_handle(stream))
    return vals, scales[: rows * cols // 128]


def cuda_act_quant(backend, stream, x, rows: int, cols: int):
    """cuda_act_quant (quant.rs:1119-1227), host slice in and out: returns
    (codes, scales) numpy arrays."""
    import torch
    xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if cols % 128:
        raise _lib.CudaError(5, f"InvalidInput error during cuda_act_quant at objeta_b200::quant.py (quant.py): "
                                f"cols {cols} not divisible by 128")
    if xv.size != rows * cols:
        raise _lib.CudaError(5, f"InvalidInput error during cuda_act_quant at objeta_b200::quant.py (quant.py): "
                                f"input len {xv.size} != rows {rows} * cols {cols}")
    dev = getattr(backend, "device", 0)
    with torch.cuda.device(dev):
        v, s = act_quant_device(torch.from_numpy(xv).to(f"cuda:{dev}"), rows, cols, stream)
        return v.cpu().numpy(), s.cpu().numpy()


def gemv_fp8_fp4_device(d_act, d_act_scales, d_weight, d_weight_scales, d_y, rows: int, cols: int, stream=None):
    """cuda_fp8_act_fp4_weight_gemv_device (quant.rs:1284-1326)."""
    _lib.call("objb_gemv_fp8_fp4_device", _dev_ptr(d_act), _dev_ptr(d_act_scales), _dev_ptr(d_weight),
              _dev_ptr(d_weight_scales), _dev_ptr(d_y), rows, cols, _lib.stream_handle(stream))
    return d_y


def gemv_fp8_fp8_device(d_act, d_act_scales, d_weight, d_weight_scales, d_y, rows: int, cols: int, stream=None):
    """cuda_fp8_act_fp8_weight_gemv_device (quant.rs:1328-1363)."""
    _lib.call("objb_gemv_fp8_fp8_device", _dev_ptr(d_act), _dev_ptr(d_act_scales), _dev_ptr(d_weight),
              _dev_ptr(d_weight_scales), _dev_ptr(d_y), rows, cols, _lib.stream_handle(stream))
    return d_y
