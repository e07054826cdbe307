"""MoeExecutor / CudaExpertCache / device MoE layer: the host-side mirror of
objeta's ``crates/objeta-cuda/src/moe.rs`` over libobjeta_b200.so.

* ``ExpertTensorKind``, ``ExpertCacheKey``, ``ResidencyClass`` (moe.rs:37-68);
* ``CudaExpertCache`` (moe.rs:70-227) with the same methods and public
  counters, plus ``get_or_insert`` (README.md:121-124) and ``release``;
* ``ExpertWeights`` / ``DeepSeekFp4ExpertWeights`` (moe.rs:13-35);
* ``MoeTelemetry`` (moe.rs:229-276);
* ``MoeExecutor.execute_selected_moe_cuda`` /
  ``execute_selected_moe_native_fp4_cuda`` (moe.rs:352-1280): host arrays in,
  host output + telemetry out;
* ``MoeLayer``: a layer resident on the device, run with
  ``objb_moe_selected_device`` / ``objb_moe_forward_device``;
* ``router_topk`` (deepseek_single_layer_moe.rs:720-740) on the device.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from .quant import QuantFormat, _dev_ptr

c_size = ctypes.c_size_t
c_int = ctypes.c_int
c_void_p = ctypes.c_void_p
c_u8p = ctypes.POINTER(ctypes.c_uint8)


class ExpertTensorKind(enum.IntEnum):
    Gate = 0
    Up = 1
    Down = 2
    GateWeight = 3
    GateScale = 4
    UpWeight = 5
    UpScale = 6
    DownWeight = 7
    DownScale = 8
    SharedGateWeight = 9
    SharedGateScale = 10
    SharedUpWeight = 11
    SharedUpScale = 12
    SharedDownWeight = 13
    SharedDownScale = 14


class ResidencyClass(enum.Enum):
    RoutedDynamic = 0
    SharedPinned = 1


@dataclass(frozen=True)
class ExpertCacheKey:
    layer_id: int
    expert_id: int
    tensor_kind: ExpertTensorKind
    quant_format: QuantFormat


class _KeyC(ctypes.Structure):
    _fields_ = [("layer_id", c_size), ("expert_id", c_size), ("tensor_kind", ctypes.c_int32),
                ("quant_format", ctypes.c_int32)]


class _StatsC(ctypes.Structure):
    _fields_ = [("capacity_bytes", c_size), ("resident_bytes", c_size), ("pinned_bytes", c_size),
                ("hit_count", c_size), ("miss_count", c_size), ("eviction_count", c_size),
                ("bypass_oversized_experts", ctypes.c_int32),
                ("cache_insert_attempt_count", c_size), ("cache_insert_accept_count", c_size),
                ("cache_insert_bypass_count", c_size), ("oversized_tensor_bypass_count", c_size),
                ("oversized_expert_bypass_count", c_size), ("self_eviction_risk_count", c_size),
                ("overflow_allocations", c_size)]


class _ExpertC(ctypes.Structure):
    _fields_ = [("w_gate", c_u8p), ("w_gate_len", c_size), ("w_up", c_u8p), ("w_up_len", c_size),
                ("w_down", c_u8p), ("w_down_len", c_size)]


class _Fp4ExpertC(ctypes.Structure):
    _fields_ = [(n, t) for nm in ("gate_weight", "gate_scale", "up_weight", "up_scale", "down_weight",
                                  "down_scale") for n, t in ((nm, c_u8p), (nm + "_len", c_size))]


_TEL_SIZE_FIELDS = [
    "selected_expert_count", "logical_expert_bytes_requested", "actual_expert_bytes_loaded",
    "resident_cache_bytes_reused", "weight_bytes_loaded", "weight_bytes_reused", "scale_bytes_loaded",
    "scale_bytes_reused", "resident_cache_resident_bytes", "resident_cache_capacity_bytes",
    "resident_cache_hit_count", "resident_cache_miss_count", "resident_cache_eviction_count",
    "resident_cache_insert_attempt_count", "resident_cache_insert_accept_count",
    "resident_cache_insert_bypass_count", "resident_cache_oversized_tensor_bypass_count",
    "resident_cache_oversized_expert_bypass_count", "resident_cache_self_eviction_risk_count",
    "dequantized_scratch_bytes"]
_TEL_FLOAT_FIELDS = ["h2d_ms", "gate_up_qgemv_ms", "activation_ms", "down_qgemv_ms", "accum_ms",
                     "unaccounted_ms", "total_ms", "shared_expert_ms"]
_TEL_TAIL_FIELDS = ["bytes_gate", "bytes_up", "bytes_down", "bytes_per_expert", "selected_working_set_bytes",
                    "routed_fp4_bytes_loaded", "routed_fp4_bytes_reused", "shared_fp8_bytes_loaded",
                    "shared_fp8_bytes_reused", "total_logical_bytes", "total_loaded_bytes",
                    "total_reused_bytes"]


class _TelC(ctypes.Structure):
    _fields_ = ([(n, c_size) for n in _TEL_SIZE_FIELDS] + [(n, ctypes.c_float) for n in _TEL_FLOAT_FIELDS]
                + [(n, c_size) for n in _TEL_TAIL_FIELDS])


class _SharedFp8C(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("gate_weight", "gate_scale", "up_weight", "up_scale", "down_weight",
                                        "down_scale")]


@dataclass
class DeepSeekFp8SharedExpertWeightsDevice:
    """moe.rs:1372-1379: the FP8 shared expert, device tensors (uint8):
    E4M3 weights gate / up [inter, hidden], down [hidden, inter] and E8M0
    scales on a 128 x 128 tile grid."""
    gate_weight: object
    gate_scale: object
    up_weight: object
    up_scale: object
    down_weight: object
    down_scale: object


class _LayerC(ctypes.Structure):
    _fields_ = [("fmt", c_int), ("flags", ctypes.c_uint32), ("hidden", c_size), ("intermediate", c_size),
                ("out_dim", c_size), ("num_experts", c_size), ("d_gate", c_void_p), ("d_up", c_void_p),
                ("d_down", c_void_p), ("d_gate_scale", c_void_p), ("d_up_scale", c_void_p),
                ("d_down_scale", c_void_p)]


# objb_expert_load_fn: int (*)(void* user, const void** host_src, size_t* bytes)
_LOAD_FN = ctypes.CFUNCTYPE(c_int, c_void_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_size))

_lib.register_signatures({
    "objb_expert_cache_new": (c_int, [c_int, c_size, ctypes.POINTER(c_void_p)]),
    "objb_expert_cache_free": (None, [c_void_p]),
    "objb_expert_cache_get": (c_int, [c_void_p, ctypes.POINTER(_KeyC), ctypes.POINTER(c_void_p)]),
    "objb_expert_cache_insert": (c_int, [c_void_p, ctypes.POINTER(_KeyC), c_void_p, c_size, c_void_p,
                                         ctypes.POINTER(c_void_p), ctypes.POINTER(c_int)]),
    "objb_expert_cache_get_or_insert": (c_int, [c_void_p, ctypes.POINTER(_KeyC), c_void_p, c_size, c_void_p,
                                                ctypes.POINTER(c_void_p), ctypes.POINTER(c_int)]),
    "objb_expert_cache_get_or_load": (c_int, [c_void_p, ctypes.POINTER(_KeyC), _LOAD_FN, c_void_p, c_void_p,
                                              ctypes.POINTER(c_void_p), ctypes.POINTER(c_int)]),
    "objb_expert_cache_touch": (c_int, [c_void_p, ctypes.POINTER(_KeyC)]),
    "objb_expert_cache_evict_lru": (c_int, [c_void_p, ctypes.POINTER(_KeyC), ctypes.POINTER(c_int)]),
    "objb_expert_cache_pin": (c_int, [c_void_p, ctypes.POINTER(_KeyC)]),
    "objb_expert_cache_insert_pinned": (c_int, [c_void_p, ctypes.POINTER(_KeyC), c_void_p, c_size, c_void_p,
                                                ctypes.POINTER(c_void_p)]),
    "objb_expert_cache_clear": (c_int, [c_void_p]),
    "objb_expert_cache_reset_counters": (c_int, [c_void_p]),
    "objb_expert_cache_stats_get": (c_int, [c_void_p, ctypes.POINTER(_StatsC)]),
    "objb_expert_cache_set_bypass_oversized_experts": (c_int, [c_void_p, c_int]),
    "objb_expert_cache_count": (c_int, [c_void_p, c_int]),
    "objb_expert_cache_contains": (c_int, [c_void_p, ctypes.POINTER(_KeyC), ctypes.POINTER(c_int)]),
    "objb_expert_cache_lru_keys": (c_int, [c_void_p, ctypes.POINTER(_KeyC), c_size, ctypes.POINTER(c_size)]),
    "objb_expert_cache_release": (c_int, [c_void_p, c_void_p]),
    "objb_moe_executor_new": (c_int, [c_int, ctypes.POINTER(c_void_p)]),
    "objb_moe_executor_free": (None, [c_void_p]),
    "objb_moe_executor_compile": (c_int, [c_void_p]),
    "objb_moe_execute_selected": (c_int, [c_void_p, c_void_p, c_int, ctypes.POINTER(_ExpertC), c_size,
                                          c_void_p, c_void_p, c_size, c_void_p, c_size, c_size, c_size,
                                          c_size, c_size, c_void_p, c_void_p, ctypes.POINTER(_TelC)]),
    "objb_moe_execute_selected_native_fp4": (c_int, [c_void_p, c_void_p, ctypes.POINTER(_Fp4ExpertC), c_size,
                                                     c_void_p, c_void_p, c_size, c_void_p, c_size, c_size,
                                                     c_size, c_size, c_size, c_void_p, c_void_p,
                                                     ctypes.POINTER(_TelC)]),
    "objb_moe_execute_pairs": (c_int, [c_void_p, c_void_p, c_int, ctypes.POINTER(_ExpertC), c_size, c_void_p,
                                       c_void_p, c_void_p, c_size, c_void_p, c_size, c_size, c_size, c_size,
                                       c_size, c_void_p, c_void_p, c_size, ctypes.POINTER(_TelC)]),
    "objb_moe_scratch_bytes": (c_int, [ctypes.POINTER(_LayerC), c_size, ctypes.POINTER(c_size)]),
    "objb_moe_official_selected_device": (c_int, [ctypes.POINTER(_LayerC), c_void_p, c_void_p, c_size, c_void_p,
                                                  c_void_p, ctypes.c_float, c_void_p]),
    "objb_moe_execute_selected_official_fp4": (c_int, [c_void_p, c_void_p, ctypes.POINTER(_Fp4ExpertC), c_size,
                                                       c_void_p, c_void_p, c_size, c_void_p, c_size, c_size,
                                                       c_size, c_size, c_size, c_void_p,
                                                       ctypes.POINTER(_SharedFp8C), c_void_p,
                                                       ctypes.POINTER(_TelC)]),
    "objb_router_topk_device": (c_int, [c_void_p, c_size, c_size, c_int, c_void_p, c_void_p, c_void_p]),
    "objb_moe_selected_device": (c_int, [ctypes.POINTER(_LayerC), c_void_p, c_void_p, c_size, c_void_p,
                                         c_void_p, ctypes.c_float, c_void_p]),
    "objb_moe_forward_device": (c_int, [ctypes.POINTER(_LayerC), c_void_p, c_size, c_int, c_void_p, c_void_p,
                                        c_void_p, c_void_p, ctypes.c_float, c_void_p]),
    "objb_moe_selected_device_noalloc": (c_int, [ctypes.POINTER(_LayerC), c_void_p, c_void_p, c_size, c_void_p,
                                                 c_void_p, ctypes.c_float, c_void_p]),
})


def _key_c(key: ExpertCacheKey) -> _KeyC:
    return _KeyC(int(key.layer_id), int(key.expert_id), int(key.tensor_kind), int(key.quant_format))


def _key_py(k: _KeyC) -> ExpertCacheKey:
    return ExpertCacheKey(int(k.layer_id), int(k.expert_id), ExpertTensorKind(k.tensor_kind),
                          QuantFormat(k.quant_format))


def _host_u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8).reshape(-1)


class CudaExpertCache:
    """Device expert cache with the reference's LRU / admission semantics."""

    def __init__(self, capacity_bytes: int, device: int = 0):
        h = c_void_p()
        _lib.call("objb_expert_cache_new", int(device), int(capacity_bytes), ctypes.byref(h))
        self._h = h
        self.device = int(device)

    @classmethod
    def new(cls, capacity_bytes: int, device: int = 0) -> "CudaExpertCache":
        return cls(capacity_bytes, device)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.load().objb_expert_cache_free(h)
            except Exception:
                pass
            self._h = None

    # ---- public counters (moe.rs:70-85)
    def stats(self) -> dict:
        s = _StatsC()
        _lib.call("objb_expert_cache_stats_get", self._h, ctypes.byref(s))
        return {n: int(getattr(s, n)) for n, _ in _StatsC._fields_}

    def __getattr__(self, name):
        if name in {n for n, _ in _StatsC._fields_} and name != "bypass_oversized_experts":
            return self.stats()[name]
        raise AttributeError(name)

    @property
    def bypass_oversized_experts(self) -> bool:
        return bool(self.stats()["bypass_oversized_experts"])

    @bypass_oversized_experts.setter
    def bypass_oversized_experts(self, v: bool) -> None:
        _lib.call("objb_expert_cache_set_bypass_oversized_experts", self._h, int(bool(v)))

    # ---- methods (moe.rs:113-226)
    def get(self, key: ExpertCacheKey):
        p = c_void_p()
        _lib.call("objb_expert_cache_get", self._h, ctypes.byref(_key_c(key)), ctypes.byref(p))
        return p.value

    def insert(self, key: ExpertCacheKey, host, stream=None) -> int:
        a = _host_u8(host)
        p, r = c_void_p(), c_int()
        _lib.call("objb_expert_cache_insert", self._h, ctypes.byref(_key_c(key)), a.ctypes.data, a.size,
                  _lib.stream_handle(stream), ctypes.byref(p), ctypes.byref(r))
        return p.value

    def get_or_insert(self, key: ExpertCacheKey, load_fn, stream=None):
        """README.md:121-124: get, else insert(load_fn()).  Returns (ptr, hit).

        ``load_fn`` is a callable returning the host bytes, run only on a miss
        (objb_expert_cache_get_or_load), or the bytes themselves
        (objb_expert_cache_get_or_insert).  Counters move as the executor's
        inline get / insert (moe.rs:508-518)."""
        p, hit = c_void_p(), c_int()
        if not callable(load_fn):
            a = _host_u8(load_fn)
            _lib.call("objb_expert_cache_get_or_insert", self._h, ctypes.byref(_key_c(key)), a.ctypes.data, a.size,
                      _lib.stream_handle(stream), ctypes.byref(p), ctypes.byref(hit))
            return p.value, bool(hit.value)
        held = []
        failure = []

        def load(_user, src, nbytes):
            try:
                a = _host_u8(load_fn())
            except Exception as exc:  # reported after the C call returns
                failure.append(exc)
                return 7  # OBJB_ERR_INTERNAL + 1
            held.append(a)
            src[0] = a.ctypes.data
            nbytes[0] = a.size
            return 0

        cb = _LOAD_FN(load)
        rc = _lib.load().objb_expert_cache_get_or_load(self._h, ctypes.byref(_key_c(key)), cb, None,
                                                         _lib.stream_handle(stream), ctypes.byref(p),
                                                         ctypes.byref(hit))
        if failure:
            raise failure[0]
        _lib.check(rc)
        return p.value, bool(hit.value)

    def touch(self, key: ExpertCacheKey) -> None:
        _lib.call("objb_expert_cache_touch", self._h, ctypes.byref(_key_c(key)))

    def evict_lru(self):
        k, f = _KeyC(), c_int()
        _lib.call("objb_expert_cache_evict_lru", self._h, ctypes.byref(k), ctypes.byref(f))
        return _key_py(k) if f.value else None

    def pin(self, key: ExpertCacheKey) -> None:
        _lib.call("objb_expert_cache_pin", self._h, ctypes.byref(_key_c(key)))

    def insert_pinned(self, key: ExpertCacheKey, host, stream=None) -> int:
        a = _host_u8(host)
        p = c_void_p()
        _lib.call("objb_expert_cache_insert_pinned", self._h, ctypes.byref(_key_c(key)), a.ctypes.data, a.size,
                  _lib.stream_handle(stream), ctypes.byref(p))
        return p.value

    def clear(self) -> None:
        _lib.call("objb_expert_cache_clear", self._h)

    def reset_counters(self) -> None:
        _lib.call("objb_expert_cache_reset_counters", self._h)

    def contains(self, key: ExpertCacheKey) -> bool:
        f = c_int()
        _lib.call("objb_expert_cache_contains", self._h, ctypes.byref(_key_c(key)), ctypes.byref(f))
        return bool(f.value)

    def lru_keys(self) -> list:
        n = c_size()
        _lib.call("objb_expert_cache_lru_keys", self._h, None, 0, ctypes.byref(n))
        arr = (_KeyC * max(1, n.value))()
        _lib.call("objb_expert_cache_lru_keys", self._h, arr, n.value, ctypes.byref(n))
        return [_key_py(arr[i]) for i in range(n.value)]

    def release(self, stream=None) -> None:
        _lib.call("objb_expert_cache_release", self._h, _lib.stream_handle(stream))


@dataclass
class ExpertWeights:
    """moe.rs:13-18: packed gate / up / down of one expert (host bytes)."""
    w_gate: np.ndarray
    w_up: np.ndarray
    w_down: np.ndarray


@dataclass
class DeepSeekFp4ExpertWeights:
    """moe.rs:27-35: split FP4 weights + E8M0 scales (host bytes)."""
    gate_weight: np.ndarray
    gate_scale: np.ndarray
    up_weight: np.ndarray
    up_scale: np.ndarray
    down_weight: np.ndarray
    down_scale: np.ndarray


@dataclass
class BytesByTensorKind:
    gate: int = 0
    up: int = 0
    down: int = 0


@dataclass
class MoeTelemetry:
    """moe.rs:236-276."""
    selected_expert_count: int = 0
    logical_expert_bytes_requested: int = 0
    actual_expert_bytes_loaded: int = 0
    resident_cache_bytes_reused: int = 0
    weight_bytes_loaded: int = 0
    weight_bytes_reused: int = 0
    scale_bytes_loaded: int = 0
    scale_bytes_reused: int = 0
    resident_cache_resident_bytes: int = 0
    resident_cache_capacity_bytes: int = 0
    resident_cache_hit_count: int = 0
    resident_cache_miss_count: int = 0
    resident_cache_eviction_count: int = 0
    resident_cache_insert_attempt_count: int = 0
    resident_cache_insert_accept_count: int = 0
    resident_cache_insert_bypass_count: int = 0
    resident_cache_oversized_tensor_bypass_count: int = 0
    resident_cache_oversized_expert_bypass_count: int = 0
    resident_cache_self_eviction_risk_count: int = 0
    dequantized_scratch_bytes: int = 0
    h2d_ms: float = 0.0
    gate_up_qgemv_ms: float = 0.0
    activation_ms: float = 0.0
    down_qgemv_ms: float = 0.0
    accum_ms: float = 0.0
    unaccounted_ms: float = 0.0
    total_ms: float = 0.0
    shared_expert_ms: float = 0.0
    bytes_by_tensor_kind: BytesByTensorKind = field(default_factory=BytesByTensorKind)
    bytes_per_expert: int = 0
    selected_working_set_bytes: int = 0
    routed_fp4_bytes_loaded: int = 0
    routed_fp4_bytes_reused: int = 0
    shared_fp8_bytes_loaded: int = 0
    shared_fp8_bytes_reused: int = 0
    total_logical_bytes: int = 0
    total_loaded_bytes: int = 0
    total_reused_bytes: int = 0

    @staticmethod
    def _from_c(t: _TelC) -> "MoeTelemetry":
        m = MoeTelemetry()
        for n in _TEL_SIZE_FIELDS + _TEL_TAIL_FIELDS:
            if n in ("bytes_gate", "bytes_up", "bytes_down"):
                continue
            setattr(m, n, int(getattr(t, n)))
        for n in _TEL_FLOAT_FIELDS:
            setattr(m, n, float(getattr(t, n)))
        m.bytes_by_tensor_kind = BytesByTensorKind(int(t.bytes_gate), int(t.bytes_up), int(t.bytes_down))
        return m


def _selection(selected):
    ids = np.array([int(e) for e, _ in selected], dtype=np.int64)
    ws = np.array([float(w) for _, w in selected], dtype=np.float32)
    return ids, ws


class MoeExecutor:
    """MoeExecutor (moe.rs:284-1280) bound to one CUDA device ordinal."""

    def __init__(self, device: int = 0):
        h = c_void_p()
        _lib.call("objb_moe_executor_new", int(device), ctypes.byref(h))
        self._h = h
        self.device = int(device)

    @classmethod
    def new(cls, device: int = 0) -> "MoeExecutor":
        return cls(device)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.load().objb_moe_executor_free(h)
            except Exception:
                pass
            self._h = None

    def status(self) -> None:
        return None

    def compile(self) -> None:
        _lib.call("objb_moe_executor_compile", self._h)

    def execute_selected_moe_cuda(self, quant, stream, experts, selected_experts, x, hidden, intermediate,
                                  out_dim, layer_id, cache=None, fmt=QuantFormat.Q4_0):
        """moe.rs:352-751.  ``quant`` (a QuantBackend) is accepted for
        signature compatibility; the fused kernels do not need it."""
        keep = [(_host_u8(e.w_gate), _host_u8(e.w_up), _host_u8(e.w_down)) for e in experts]
        arr = (_ExpertC * max(1, len(keep)))()
        for i, (g, u, d) in enumerate(keep):
            arr[i] = _ExpertC(g.ctypes.data_as(c_u8p), g.size, u.ctypes.data_as(c_u8p), u.size,
                              d.ctypes.data_as(c_u8p), d.size)
        ids, ws = _selection(selected_experts)
        xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        out = np.zeros(out_dim, dtype=np.float32)
        tel = _TelC()
        _lib.call("objb_moe_execute_selected", self._h, _lib.stream_handle(stream), int(QuantFormat(fmt)), arr,
                  len(keep), ids.ctypes.data, ws.ctypes.data, ids.size, xv.ctypes.data, xv.size, hidden,
                  intermediate, out_dim, layer_id, cache._h if cache is not None else None, out.ctypes.data,
                  ctypes.byref(tel))
        return out, MoeTelemetry._from_c(tel)

    def expert_table(self, experts):
        """A C table of host expert weights for ``execute_pairs``; keep it
        (and the arrays it points into) alive while it is used."""
        keep = [(_host_u8(e.w_gate), _host_u8(e.w_up), _host_u8(e.w_down)) for e in experts]
        arr = (_ExpertC * max(1, len(keep)))()
        for i, (g, u, d) in enumerate(keep):
            arr[i] = _ExpertC(g.ctypes.data_as(c_u8p), g.size, u.ctypes.data_as(c_u8p), u.size,
                              d.ctypes.data_as(c_u8p), d.size)
        return (arr, len(keep), keep)

    def execute_pairs(self, table, pair_expert, pair_token, d_x, d_v, hidden, intermediate, out_dim, layer_id,
                      cache=None, pair_out=None, fmt=QuantFormat.Q4_0, stream=None):
        """Multi-token form of ``execute_selected_moe_cuda`` on device
        activations (objb_moe_execute_pairs): host int32 pair arrays, d_x
        [T, hidden] and d_v [V, out_dim] device tensors; each distinct expert
        is resolved through ``cache`` once per call.  Returns MoeTelemetry."""
        arr, n, _ = table
        pe = np.ascontiguousarray(pair_expert, dtype=np.int32)
        pt = np.ascontiguousarray(pair_token, dtype=np.int32)
        po = None if pair_out is None else np.ascontiguousarray(pair_out, dtype=np.int32)
        tel = _TelC()
        _lib.call("objb_moe_execute_pairs", self._h, _lib.stream_handle(stream), int(QuantFormat(fmt)), arr, n,
                  pe.ctypes.data, pt.ctypes.data, po.ctypes.data if po is not None else None, pe.size,
                  _dev_ptr(d_x), d_x.shape[0], hidden, intermediate, out_dim, layer_id,
                  cache._h if cache is not None else None, _dev_ptr(d_v), d_v.shape[0], ctypes.byref(tel))
        return MoeTelemetry._from_c(tel)

    def execute_selected_moe_official_routed_fp4_cuda(self, quant, stream, experts, selected_experts, x, hidden,
                                                      intermediate, out_dim, layer_id, cache=None,
                                                      shared_expert=None):
        """moe.rs:1393-1660: the official DeepSeek arithmetic (act_quant +
        FP8 x FP4 routed experts, optional FP8 shared expert on the device)."""
        names = ("gate_weight", "gate_scale", "up_weight", "up_scale", "down_weight", "down_scale")
        keep = [[_host_u8(getattr(e, n)) for n in names] for e in experts]
        arr = (_Fp4ExpertC * max(1, len(keep)))()
        for i, ts in enumerate(keep):
            vals = []
            for t in ts:
                vals += [t.ctypes.data_as(c_u8p), t.size]
            arr[i] = _Fp4ExpertC(*vals)
        ids, ws = _selection(selected_experts)
        xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        out = np.zeros(out_dim, dtype=np.float32)
        tel = _TelC()
        sh = None
        if shared_expert is not None:
            sh = _SharedFp8C(*[_dev_ptr(getattr(shared_expert, n)) for n in names])
        _lib.call("objb_moe_execute_selected_official_fp4", self._h, _lib.stream_handle(stream), arr, len(keep),
                  ids.ctypes.data, ws.ctypes.data, ids.size, xv.ctypes.data, xv.size, hidden, intermediate,
                  out_dim, layer_id, cache._h if cache is not None else None,
                  ctypes.byref(sh) if sh is not None else None, out.ctypes.data, ctypes.byref(tel))
        return out, MoeTelemetry._from_c(tel)

    def execute_selected_moe_native_fp4_cuda(self, quant, stream, experts, selected_experts, x, hidden,
                                             intermediate, out_dim, layer_id, cache=None):
        """moe.rs:816-1280."""
        names = ("gate_weight", "gate_scale", "up_weight", "up_scale", "down_weight", "down_scale")
        keep = [[_host_u8(getattr(e, n)) for n in names] for e in experts]
        arr = (_Fp4ExpertC * max(1, len(keep)))()
        for i, ts in enumerate(keep):
            vals = []
            for t in ts:
                vals += [t.ctypes.data_as(c_u8p), t.size]
            arr[i] = _Fp4ExpertC(*vals)
        ids, ws = _selection(selected_experts)
        xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        out = np.zeros(out_dim, dtype=np.float32)
        tel = _TelC()
        _lib.call("objb_moe_execute_selected_native_fp4", self._h, _lib.stream_handle(stream), arr, len(keep),
                  ids.ctypes.data, ws.ctypes.data, ids.size, xv.ctypes.data, xv.size, hidden, intermediate,
                  out_dim, layer_id, cache._h if cache is not None else None, out.ctypes.data, ctypes.byref(tel))
        return out, MoeTelemetry._from_c(tel)


def router_topk(d_logits, top_k: int, renormalize: bool = False, stream=None, ids=None, weights=None):
    """Device softmax + stable top-k (deepseek_single_layer_moe.rs:720-740).
    Returns (ids int32, weights f32) device tensors."""
    import torch
    n = d_logits.numel()
    if ids is None:
        ids = torch.empty(top_k, dtype=torch.int32, device=d_logits.device)
    if weights is None:
        weights = torch.empty(top_k, dtype=torch.float32, device=d_logits.device)
    _lib.call("objb_router_topk_device", _dev_ptr(d_logits), n, top_k, int(bool(renormalize)), _dev_ptr(ids),
              _dev_ptr(weights), _lib.stream_handle(stream))
    return ids, weights


def ffn_bf16_device(d_gate, d_up, d_down, hidden: int, intermediate: int, out_dim: int, d_x, d_out,
                    accumulate: bool = False, swiglu_limit: float = 0.0, stream=None):
    """The dense bf16 SwiGLU FFN (a DeepSeek-style shared expert):
    d_out = down(SwiGLU(gate x, up x)), or d_out += it with ``accumulate``."""
    _lib.call("objb_ffn_bf16_device", _dev_ptr(d_gate), _dev_ptr(d_up), _dev_ptr(d_down), hidden, intermediate,
              out_dim, _dev_ptr(d_x), _dev_ptr(d_out), int(bool(accumulate)), float(swiglu_limit),
              _lib.stream_handle(stream))
    return d_out


class MoeLayer:
    """A MoE layer resident on the device (objb_moe_layer).

    ``gate`` / ``up`` / ``down``: lists (one per expert) of uint8 CUDA tensors
    in the format's packed layout; for split FP4 also ``*_scale`` lists.
    """

    def __init__(self, fmt, hidden, intermediate, out_dim, gate, up, down, gate_scale=None, up_scale=None,
                 down_scale=None):
        import torch
        self.fmt = QuantFormat(fmt)
        self.hidden, self.intermediate, self.out_dim = int(hidden), int(intermediate), int(out_dim)
        self.num_experts = len(gate)
        self._tensors = [gate, up, down, gate_scale, up_scale, down_scale]
        dev = gate[0].device
        self.device = dev
        flags = 0
        tabs = []
        for lst in self._tensors:
            if lst is None:
                tabs.append(None)
                continue
            ptrs = [_dev_ptr(t) for t in lst]
            if any(p & 15 for p in ptrs):
                flags |= 1
            tabs.append(torch.tensor(ptrs, dtype=torch.int64, device=dev))
        self._tabs = tabs
        self._c = _LayerC(int(self.fmt), flags, self.hidden, self.intermediate, self.out_dim, self.num_experts,
                          *[t.data_ptr() if t is not None else None for t in tabs])

    def scratch_bytes(self, top_k: int) -> int:
        n = c_size()
        _lib.call("objb_moe_scratch_bytes", ctypes.byref(self._c), top_k, ctypes.byref(n))
        return int(n.value)

    def forward_selected(self, d_ids, d_weights, d_x, d_out=None, swiglu_limit: float = 0.0, stream=None):
        import torch
        if d_out is None:
            d_out = torch.empty(self.out_dim, dtype=torch.float32, device=self.device)
        _lib.call("objb_moe_selected_device", ctypes.byref(self._c), _dev_ptr(d_ids), _dev_ptr(d_weights),
                  d_ids.numel(), _dev_ptr(d_x), _dev_ptr(d_out), float(swiglu_limit), _lib.stream_handle(stream))
        return d_out

    def forward_selected_noalloc(self, d_ids, d_weights, d_x, d_out, swiglu_limit: float = 0.0, stream=None):
        """The same launch for callers that cannot let the library allocate
        device memory: scratch comes from the library's fixed 4 MiB array
        (objb_moe_selected_device_noalloc); ``d_out`` must be given.  Calls
        that overlap on the GPU share that array and race."""
        _lib.call("objb_moe_selected_device_noalloc", ctypes.byref(self._c), _dev_ptr(d_ids), _dev_ptr(d_weights),
                  d_ids.numel(), _dev_ptr(d_x), _dev_ptr(d_out), float(swiglu_limit), _lib.stream_handle(stream))
        return d_out

    def forward_official_selected(self, d_ids, d_weights, d_x, d_out=None, swiglu_limit: float = 10.0,
                                  stream=None):
        """The official DeepSeek routed arithmetic on this split-FP4 layer
        (objb_moe_official_selected_device)."""
        import torch
        if d_out is None:
            d_out = torch.empty(self.out_dim, dtype=torch.float32, device=self.device)
        _lib.call("objb_moe_official_selected_device", ctypes.byref(self._c), _dev_ptr(d_ids), _dev_ptr(d_weights),
                  d_ids.numel(), _dev_ptr(d_x), _dev_ptr(d_out), float(swiglu_limit), _lib.stream_handle(stream))
        return d_out

    def forward(self, d_logits, top_k, d_x, renormalize=False, d_out=None, swiglu_limit=0.0, stream=None,
                ids=None, weights=None):
        import torch
        if d_out is None:
            d_out = torch.empty(self.out_dim, dtype=torch.float32, device=self.device)
        if ids is None:
            ids = torch.empty(top_k, dtype=torch.int32, device=self.device)
        if weights is None:
            weights = torch.empty(top_k, dtype=torch.float32, device=self.device)
        _lib.call("objb_moe_forward_device", ctypes.byref(self._c), _dev_ptr(d_logits), top_k,
                  int(bool(renormalize)), _dev_ptr(ids), _dev_ptr(weights), _dev_ptr(d_x), _dev_ptr(d_out),
                  float(swiglu_limit), _lib.stream_handle(stream))
        return d_out, ids, weights
