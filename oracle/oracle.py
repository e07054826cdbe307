"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of the C oracle.

The C file ``objeta_oracle.c`` restates the CPU arithmetic of objeta's
``objeta-cuda`` path (quantizers, dot rows, FP4 decode, CPU MoE, router); see
its header for the rules it follows.  Only ``tests/``, ``__graft_entry__.smoke``
and ``bench.py``'s CPU-baseline legs may import this module.  The product in
``objeta_b200`` never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboro.so")
_lock = threading.Lock()
_lib = None

Q4_0, Q5_0, IQ3_0, FP4_E2M1 = 0, 1, 2, 3
BLOCK_BYTES = {Q4_0: 18, Q5_0: 22, IQ3_0: 14, FP4_E2M1: 17}

_c_u8p = ctypes.POINTER(ctypes.c_uint8)
_c_f32p = ctypes.POINTER(ctypes.c_float)
_c_i64p = ctypes.POINTER(ctypes.c_int64)
_c_u8pp = ctypes.POINTER(_c_u8p)


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc only)."""
    src = os.path.join(_HERE, "objeta_oracle.c")
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_SO)
            L.oro_f32_to_f16_bits.restype = ctypes.c_uint16
            L.oro_f32_to_f16_bits.argtypes = [ctypes.c_float]
            L.oro_f16_to_f32_bits.restype = ctypes.c_float
            L.oro_f16_to_f32_bits.argtypes = [ctypes.c_uint16]
            for n in ("oro_decode_f8_e8m0", "oro_f8e8m0_to_f32", "oro_f8e4m3_to_f32"):
                getattr(L, n).restype = ctypes.c_float
                getattr(L, n).argtypes = [ctypes.c_uint8]
            for n in ("oro_q4_quantize_block", "oro_q5_quantize_block",
                      "oro_iq3_quantize_block", "oro_fp4_quantize_block"):
                getattr(L, n).restype = None
                getattr(L, n).argtypes = [_c_f32p, _c_u8p]
            L.oro_quantize_matrix.restype = ctypes.c_int
            L.oro_quantize_matrix.argtypes = [ctypes.c_int, _c_f32p, ctypes.c_size_t,
                                              ctypes.c_size_t, _c_u8p]
            L.oro_gemv.restype = ctypes.c_int
            L.oro_gemv.argtypes = [ctypes.c_int, _c_u8p, _c_f32p, ctypes.c_size_t,
                                   ctypes.c_size_t, _c_f32p]
            L.oro_gemv_threads.restype = ctypes.c_int
            L.oro_gemv_threads.argtypes = [ctypes.c_int, _c_u8p, _c_f32p, ctypes.c_size_t,
                                           ctypes.c_size_t, _c_f32p, ctypes.c_int]
            L.oro_dequantize_matrix.restype = ctypes.c_int
            L.oro_dequantize_matrix.argtypes = [ctypes.c_int, _c_u8p, ctypes.c_size_t,
                                                ctypes.c_size_t, _c_f32p]
            L.oro_dense_gemv.restype = None
            L.oro_dense_gemv.argtypes = [_c_f32p, _c_f32p, ctypes.c_size_t,
                                         ctypes.c_size_t, _c_f32p]
            L.oro_fp4_decode_split.restype = None
            L.oro_fp4_decode_split.argtypes = [_c_u8p, _c_u8p, ctypes.c_size_t,
                                               ctypes.c_size_t, ctypes.c_size_t, _c_f32p]
            L.oro_selected_moe_q4.restype = ctypes.c_int
            L.oro_selected_moe_q4.argtypes = [_c_u8pp, _c_u8pp, _c_u8pp, ctypes.c_size_t,
                                              _c_i64p, _c_f32p, ctypes.c_size_t, _c_f32p,
                                              ctypes.c_size_t, ctypes.c_size_t,
                                              ctypes.c_size_t, _c_f32p, ctypes.c_int]
            L.oro_selected_moe_native_fp4.restype = ctypes.c_int
            L.oro_selected_moe_native_fp4.argtypes = [
                _c_u8pp, _c_u8pp, _c_u8pp, _c_u8pp, _c_u8pp, _c_u8pp, ctypes.c_size_t,
                _c_i64p, _c_f32p, ctypes.c_size_t, _c_f32p, ctypes.c_size_t,
                ctypes.c_size_t, ctypes.c_size_t, _c_f32p, ctypes.c_int]
            L.oro_router_from_logits.restype = ctypes.c_int
            L.oro_router_from_logits.argtypes = [_c_f32p, ctypes.c_size_t, ctypes.c_size_t,
                                                 ctypes.c_int, _c_i64p, _c_f32p]
            L.oro_router.restype = ctypes.c_int
            L.oro_router.argtypes = [_c_f32p, _c_f32p, ctypes.c_size_t, ctypes.c_size_t,
                                     ctypes.c_size_t, _c_i64p, _c_f32p]
            L.oro_seeded_f32s.restype = None
            L.oro_seeded_f32s.argtypes = [ctypes.c_size_t, ctypes.c_uint64, _c_f32p]
            L.oro_f32_to_f8e4m3_exact.restype = ctypes.c_uint8
            L.oro_f32_to_f8e4m3_exact.argtypes = [ctypes.c_float]
            L.oro_act_quant.restype = ctypes.c_int
            L.oro_act_quant.argtypes = [_c_f32p, ctypes.c_size_t, ctypes.c_size_t, _c_u8p, _c_u8p]
            for n in ("oro_fp8_act_fp4_weight_gemv_f32", "oro_fp8_act_fp8_weight_gemv"):
                getattr(L, n).restype = None
                getattr(L, n).argtypes = [_c_u8p, _c_u8p, _c_u8p, _c_u8p, ctypes.c_size_t, ctypes.c_size_t,
                                          _c_f32p]
            L.oro_routed_expert_fp4_official_f32.restype = ctypes.c_int
            L.oro_routed_expert_fp4_official_f32.argtypes = [_c_u8p] * 6 + [_c_f32p, ctypes.c_size_t,
                                                                            ctypes.c_size_t, ctypes.c_size_t,
                                                                            ctypes.c_float, _c_f32p]
            L.oro_shared_expert_fp8_official.restype = ctypes.c_int
            L.oro_shared_expert_fp8_official.argtypes = [_c_u8p] * 6 + [_c_f32p, ctypes.c_size_t, ctypes.c_size_t,
                                                                        ctypes.c_float, _c_f32p]
            L.oro_deepseek_gate.restype = ctypes.c_int
            L.oro_deepseek_gate.argtypes = [_c_f32p, _c_f32p, _c_i64p, ctypes.c_size_t, _c_f32p, ctypes.c_int64,
                                             ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int,
                                             ctypes.c_float, _c_i64p, _c_f32p]
            _lib = L
    return _lib


def _u8(a):
    return a.ctypes.data_as(_c_u8p)


def _f32(a):
    return a.ctypes.data_as(_c_f32p)


def _i64(a):
    return a.ctypes.data_as(_c_i64p)


def f32_to_f16_bits(v: float) -> int:
    return int(lib().oro_f32_to_f16_bits(ctypes.c_float(v)))


def f16_to_f32_bits(b: int) -> float:
    return float(lib().oro_f16_to_f32_bits(b))


def decode_f8_e8m0(raw: int) -> float:
    return float(lib().oro_decode_f8_e8m0(raw))


def f8e8m0_to_f32(raw: int) -> float:
    return float(lib().oro_f8e8m0_to_f32(raw))


def f8e4m3_to_f32(raw: int) -> float:
    return float(lib().oro_f8e4m3_to_f32(raw))


def quantize_block(fmt: int, src) -> np.ndarray:
    src = np.ascontiguousarray(src, dtype=np.float32)
    assert src.size == 32
    dst = np.zeros(BLOCK_BYTES[fmt], dtype=np.uint8)
    fn = {Q4_0: "oro_q4_quantize_block", Q5_0: "oro_q5_quantize_block",
          IQ3_0: "oro_iq3_quantize_block", FP4_E2M1: "oro_fp4_quantize_block"}[fmt]
    getattr(lib(), fn)(_f32(src), _u8(dst))
    return dst


def quantize_matrix(fmt: int, matrix, rows: int, cols: int) -> np.ndarray:
    m = np.ascontiguousarray(matrix, dtype=np.float32).reshape(-1)
    assert m.size == rows * cols
    if cols % 32 != 0:
        raise ValueError(f"cols {cols} must be a multiple of block_size 32")
    out = np.zeros(rows * (cols // 32) * BLOCK_BYTES[fmt], dtype=np.uint8)
    rc = lib().oro_quantize_matrix(fmt, _f32(m), rows, cols, _u8(out))
    if rc != 0:
        raise ValueError(f"oro_quantize_matrix failed rc={rc}")
    return out


def gemv(fmt: int, qweights, x, rows: int, cols: int, threads: int = 1) -> np.ndarray:
    qw = np.ascontiguousarray(qweights, dtype=np.uint8).reshape(-1)
    xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    y = np.zeros(rows, dtype=np.float32)
    rc = lib().oro_gemv_threads(fmt, _u8(qw), _f32(xv), rows, cols, _f32(y), threads)
    if rc != 0:
        raise ValueError(f"oro_gemv failed rc={rc}")
    return y


def dequantize_matrix(fmt: int, qweights, rows: int, cols: int) -> np.ndarray:
    qw = np.ascontiguousarray(qweights, dtype=np.uint8).reshape(-1)
    out = np.zeros(rows * cols, dtype=np.float32)
    rc = lib().oro_dequantize_matrix(fmt, _u8(qw), rows, cols, _f32(out))
    if rc != 0:
        raise ValueError("oro_dequantize_matrix failed")
    return out.reshape(rows, cols)


def row_abs_sums(fmt: int, qweights, x, rows: int, cols: int) -> np.ndarray:
    """sum_l |w_l x_l| per row (f64): the scale of the parity tolerance."""
    w = dequantize_matrix(fmt, qweights, rows, cols).astype(np.float64)
    return np.abs(w) @ np.abs(np.asarray(x, dtype=np.float64))


def dense_gemv(matrix, x, rows: int, cols: int) -> np.ndarray:
    m = np.ascontiguousarray(matrix, dtype=np.float32).reshape(-1)
    xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    y = np.zeros(rows, dtype=np.float32)
    lib().oro_dense_gemv(_f32(m), _f32(xv), rows, cols, _f32(y))
    return y


def fp4_decode_split(weight, scale, rows: int, cols: int, block_size: int = 32) -> np.ndarray:
    w = np.ascontiguousarray(weight, dtype=np.uint8).reshape(-1)
    s = np.ascontiguousarray(scale, dtype=np.uint8).reshape(-1)
    assert w.size == rows * cols // 2 and s.size == rows * cols // block_size
    out = np.zeros(rows * cols, dtype=np.float32)
    lib().oro_fp4_decode_split(_u8(w), _u8(s), rows, cols, block_size, _f32(out))
    return out


def _ptr_array(arrs):
    ptrs = (_c_u8p * len(arrs))()
    for i, a in enumerate(arrs):
        ptrs[i] = _u8(a)
    return ptrs


def selected_moe_q4(experts, selected, x, hidden, intermediate, out_dim, threads=0):
    """experts: list of (w_gate, w_up, w_down) uint8 arrays; selected: [(id, w)]."""
    g = [np.ascontiguousarray(e[0], dtype=np.uint8) for e in experts]
    u = [np.ascontiguousarray(e[1], dtype=np.uint8) for e in experts]
    d = [np.ascontiguousarray(e[2], dtype=np.uint8) for e in experts]
    ids = np.array([s[0] for s in selected], dtype=np.int64)
    ws = np.array([s[1] for s in selected], dtype=np.float32)
    xv = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(out_dim, dtype=np.float32)
    rc = lib().oro_selected_moe_q4(_ptr_array(g), _ptr_array(u), _ptr_array(d), len(experts),
                                   _i64(ids), _f32(ws), len(selected), _f32(xv), hidden,
                                   intermediate, out_dim, _f32(out), threads)
    if rc != 0:
        raise ValueError(f"oro_selected_moe_q4 failed rc={rc}")
    return out


def selected_moe_native_fp4(experts, selected, x, hidden, intermediate, out_dim, threads=0):
    """experts: list of 6-tuples (gate_w, gate_s, up_w, up_s, down_w, down_s)."""
    cols = [[np.ascontiguousarray(e[i], dtype=np.uint8) for e in experts] for i in range(6)]
    ids = np.array([s[0] for s in selected], dtype=np.int64)
    ws = np.array([s[1] for s in selected], dtype=np.float32)
    xv = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(out_dim, dtype=np.float32)
    rc = lib().oro_selected_moe_native_fp4(*[_ptr_array(c) for c in cols], len(experts),
                                           _i64(ids), _f32(ws), len(selected), _f32(xv),
                                           hidden, intermediate, out_dim, _f32(out), threads)
    if rc != 0:
        raise ValueError(f"oro_selected_moe_native_fp4 failed rc={rc}")
    return out


def router_from_logits(logits, top_k: int, renormalize: bool = False):
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    ids = np.zeros(top_k, dtype=np.int64)
    ws = np.zeros(top_k, dtype=np.float32)
    rc = lib().oro_router_from_logits(_f32(lg), lg.size, top_k, int(renormalize),
                                      _i64(ids), _f32(ws))
    if rc != 0:
        raise ValueError("router_from_logits failed")
    return ids, ws


def router(router_weights, hidden, num_experts: int, hidden_size: int, top_k: int):
    w = np.ascontiguousarray(router_weights, dtype=np.float32)
    h = np.ascontiguousarray(hidden, dtype=np.float32)
    if w.size != num_experts * hidden_size:
        raise ValueError("router weights len != num_experts * hidden_size")
    ids = np.zeros(top_k, dtype=np.int64)
    ws = np.zeros(top_k, dtype=np.float32)
    rc = lib().oro_router(_f32(w), _f32(h), num_experts, hidden_size, top_k, _i64(ids), _f32(ws))
    if rc != 0:
        raise ValueError("router failed")
    return ids, ws


def seeded_f32s(length: int, seed: int) -> np.ndarray:
    out = np.zeros(length, dtype=np.float32)
    lib().oro_seeded_f32s(length, seed & 0xFFFFFFFFFFFFFFFF, _f32(out))
    return out


def split_interleaved_fp4(interleaved, rows: int, cols: int):
    """moe.rs:2319-2331 (test helper split_interleaved_fp4): 17-byte blocks ->
    (weights [rows, cols/2], scales [rows, cols/32])."""
    a = np.ascontiguousarray(interleaved, dtype=np.uint8).reshape(rows, cols // 32, 17)
    return a[:, :, 1:].reshape(-1).copy(), a[:, :, 0].reshape(-1).copy()


def compare_outputs(reference, actual):
    """quant.rs:676-723 (compare_outputs): cosine, relative L2 (f64) and max-abs."""
    r = np.asarray(reference, dtype=np.float32).reshape(-1)
    a = np.asarray(actual, dtype=np.float32).reshape(-1)
    if r.size != a.size:
        raise ValueError(f"reference len {r.size} != actual len {a.size}")
    r64, a64 = r.astype(np.float64), a.astype(np.float64)
    dot = float(np.dot(r64, a64))
    rn = float(np.dot(r64, r64))
    an = float(np.dot(a64, a64))
    diff = (a - r).astype(np.float32)
    sq = float(np.dot(diff.astype(np.float64), diff.astype(np.float64)))
    max_abs = float(np.max(np.abs(diff))) if diff.size else 0.0
    cos = dot / (np.sqrt(rn) * np.sqrt(an)) if rn > 0 and an > 0 else 1.0
    rel = np.sqrt(sq) / np.sqrt(rn) if rn > 0 else 0.0
    return {"cosine_similarity": float(cos), "relative_l2_error": float(rel),
            "max_abs_error": max_abs}


# ---------------------------------------------------------------- official DeepSeek path
def f32_to_f8e4m3_exact(v: float) -> int:
    """deepseek.rs:1444-1481."""
    return int(lib().oro_f32_to_f8e4m3_exact(ctypes.c_float(v)))


def act_quant(x, block: int = 128):
    """deepseek.rs:1484-1525 (cpu_act_quant) -> (E4M3 codes, E8M0 scales)."""
    xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    y = np.zeros(xv.size, np.uint8)
    s = np.zeros(xv.size // block if block else 0, np.uint8)
    if lib().oro_act_quant(_f32(xv), xv.size, block, _u8(y), _u8(s)) != 0:
        raise ValueError("input length must be multiple of block_size")
    return y, s


def _u8c(a):
    return np.ascontiguousarray(a, dtype=np.uint8).reshape(-1)


def fp8_act_fp4_weight_gemv_f32(act, act_s, w, ws, rows: int, cols: int) -> np.ndarray:
    """deepseek.rs:1528-1570 (sequential f32 sum)."""
    a, as_, wv, wsv = _u8c(act), _u8c(act_s), _u8c(w), _u8c(ws)
    y = np.zeros(rows, np.float32)
    lib().oro_fp8_act_fp4_weight_gemv_f32(_u8(a), _u8(as_), _u8(wv), _u8(wsv), rows, cols, _f32(y))
    return y


def fp8_act_fp8_weight_gemv(act, act_s, w, ws, rows: int, cols: int) -> np.ndarray:
    """deepseek.rs:1630-1660 (f64 sum)."""
    a, as_, wv, wsv = _u8c(act), _u8c(act_s), _u8c(w), _u8c(ws)
    y = np.zeros(rows, np.float32)
    lib().oro_fp8_act_fp8_weight_gemv(_u8(a), _u8(as_), _u8(wv), _u8(wsv), rows, cols, _f32(y))
    return y


def routed_expert_fp4_official_f32(gw, gs, uw, us, dw, ds, x, dim: int, inter: int, out_dim: int,
                                   swiglu_limit: float) -> np.ndarray:
    """deepseek.rs:1690-1715 (cpu_routed_expert_fp4_official_f32)."""
    ts = [_u8c(t) for t in (gw, gs, uw, us, dw, ds)]
    xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.zeros(out_dim, np.float32)
    rc = lib().oro_routed_expert_fp4_official_f32(*[_u8(t) for t in ts], _f32(xv), dim, inter, out_dim,
                                                  ctypes.c_float(swiglu_limit), _f32(out))
    if rc != 0:
        raise ValueError(f"oro_routed_expert_fp4_official_f32 rc={rc}")
    return out


def shared_expert_fp8_official(w1, s1, w3, s3, w2, s2, x, dim: int, inter: int, swiglu_limit: float) -> np.ndarray:
    """deepseek.rs:1662-1688 (cpu_shared_expert_fp8_official)."""
    ts = [_u8c(t) for t in (w1, s1, w3, s3, w2, s2)]
    xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.zeros(dim, np.float32)
    rc = lib().oro_shared_expert_fp8_official(*[_u8(t) for t in ts], _f32(xv), dim, inter,
                                              ctypes.c_float(swiglu_limit), _f32(out))
    if rc != 0:
        raise ValueError(f"oro_shared_expert_fp8_official rc={rc}")
    return out


SOFTMAX, SIGMOID, SQRT_SOFTPLUS = 0, 1, 2


def deepseek_gate(gate_weight, hidden, num_experts: int, hidden_size: int, top_k: int, score_func: int,
                  route_scale: float, gate_bias=None, tid2eid=None, input_id=None):
    """dsl_moe.rs:768-881 (cpu_gate_ref) -> (ids int64 [top_k], weights f32)."""
    gw = np.ascontiguousarray(gate_weight, dtype=np.float32).reshape(-1)
    hv = np.ascontiguousarray(hidden, dtype=np.float32).reshape(-1)
    b = None if gate_bias is None else np.ascontiguousarray(gate_bias, dtype=np.float32).reshape(-1)
    t = None if tid2eid is None else np.ascontiguousarray(tid2eid, dtype=np.int64).reshape(-1)
    ids = np.zeros(top_k, np.int64)
    w = np.zeros(top_k, np.float32)
    rc = lib().oro_deepseek_gate(_f32(gw), _f32(b) if b is not None else None, _i64(t) if t is not None else None,
                                 0 if t is None else t.size, _f32(hv), -1 if input_id is None else int(input_id),
                                 num_experts, hidden_size, top_k, score_func, ctypes.c_float(route_scale),
                                 _i64(ids), _f32(w))
    if rc != 0:
        raise ValueError("input_id is required for hash layers and must be in range")
    return ids, w
