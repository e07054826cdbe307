"""objeta_b200: B200-native (sm_100a) build of objeta-cuda's quantized GEMV and
selected-expert MoE path.

The compute lives in ``libobjeta_b200.so`` (hand-written CUDA for sm_100a,
C ABI in ``include/objeta_b200.h``).  This package is the host-side mirror of
the reference Rust API (``QuantBackend``, ``MoeExecutor``, ``CudaExpertCache``,
``QuantFormat``) over that ABI.
"""
from ._lib import CudaError, LIB_PATH, load  # noqa: F401
from .quant import QGemvShape, QGemvTelemetry, QuantBackend, QuantFormat  # noqa: F401

__all__ = ["CudaError", "QGemvShape", "QGemvTelemetry", "QuantBackend", "QuantFormat", "load",
           "LIB_PATH"]
