"""MoE test helpers: reference-style expert builders and the parity bound."""
import numpy as np

from oracle import oracle as O

# MoE parity: |gpu - cpu| <= bound_r, the propagated form of the GEMV bound
# (TOL * sum|w x| per dot product, through SwiGLU and the weighted combine).
TOL = 1e-5


def _silu(g):
    return g / (1.0 + np.exp(-g))


def _dsilu(g):
    s = 1.0 / (1.0 + np.exp(-g))
    return s * (1.0 + g * (1.0 - s))


def _dequant_rows(fmt, q, rows, cols, chunk=2048):
    """Yields (row0, dense f64 chunk) of a packed matrix (interleaved formats)."""
    rb = cols // 32 * O.BLOCK_BYTES[fmt]
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        yield r0, O.dequantize_matrix(fmt, q[r0 * rb:r1 * rb], r1 - r0, cols).astype(np.float64)


def _dense_split(w, s, rows, cols, chunk=2048):
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        yield r0, O.fp4_decode_split(w[r0 * cols // 2:r1 * cols // 2], s[r0 * cols // 32:r1 * cols // 32],
                                     r1 - r0, cols).reshape(r1 - r0, cols).astype(np.float64)


def _mv(chunks, v, rows):
    """(W v, |W| |v|) in f64 over row chunks."""
    y = np.zeros(rows)
    a = np.zeros(rows)
    av = np.abs(v)
    for r0, W in chunks:
        y[r0:r0 + W.shape[0]] = W @ v
        a[r0:r0 + W.shape[0]] = np.abs(W) @ av
    return y, a


def moe_bound(matrices_of, selected, x, hidden, intermediate, out_dim):
    """Per output row bound of |gpu - reference| for the selected-expert MoE.

    matrices_of(e) -> (chunks_fn(kind), ...): returns a callable giving row
    chunks of gate / up / down for expert e."""
    x = np.asarray(x, np.float64)
    bound = np.zeros(out_dim)
    for e, w in selected:
        chunks = matrices_of(e)
        g, G = _mv(chunks("gate"), x, intermediate)
        u, U = _mv(chunks("up"), x, intermediate)
        act = _silu(g) * u
        dact = np.abs(_dsilu(g)) * np.abs(u) * TOL * G + np.abs(_silu(g)) * TOL * U + 1e-6 * np.abs(act)
        _, D = _mv(chunks("down"), act, out_dim)
        _, Dd = _mv(chunks("down"), dact, out_dim)
        bound += abs(float(w)) * (TOL * D + Dd)
    return bound


def q4_matrices(experts, hidden, intermediate, out_dim, fmt=O.Q4_0):
    """experts: list of (w_gate, w_up, w_down) packed bytes."""
    def of(e):
        g, u, d = experts[e]

        def chunks(kind):
            if kind == "gate":
                return _dequant_rows(fmt, g, intermediate, hidden)
            if kind == "up":
                return _dequant_rows(fmt, u, intermediate, hidden)
            return _dequant_rows(fmt, d, out_dim, intermediate)
        return chunks
    return of


def fp4_matrices(experts, hidden, intermediate, out_dim):
    """experts: list of 6-tuples (gate_w, gate_s, up_w, up_s, down_w, down_s)."""
    def of(e):
        gw, gs, uw, us, dw, ds = experts[e]

        def chunks(kind):
            if kind == "gate":
                return _dense_split(gw, gs, intermediate, hidden)
            if kind == "up":
                return _dense_split(uw, us, intermediate, hidden)
            return _dense_split(dw, ds, out_dim, intermediate)
        return chunks
    return of


def make_q4_experts(num_experts, hidden, intermediate, out_dim, seed, fmt=O.Q4_0):
    """moe.rs:1765-1783: expert e from seeded_f32s(seed ^ e ^ 0x1111/0x2222/0x3333)."""
    experts, dense = [], []
    for e in range(num_experts):
        g = O.seeded_f32s(intermediate * hidden, seed ^ e ^ 0x1111)
        u = O.seeded_f32s(intermediate * hidden, seed ^ e ^ 0x2222)
        d = O.seeded_f32s(out_dim * intermediate, seed ^ e ^ 0x3333)
        experts.append((O.quantize_matrix(fmt, g, intermediate, hidden),
                        O.quantize_matrix(fmt, u, intermediate, hidden),
                        O.quantize_matrix(fmt, d, out_dim, intermediate)))
        dense.append((g, u, d))
    return experts, dense


def make_fp4_experts(num_experts, hidden, intermediate, out_dim, seed):
    """moe.rs:2351-2373: quantize to interleaved FP4, then split."""
    out = []
    for e in range(num_experts):
        g = O.seeded_f32s(intermediate * hidden, seed ^ e ^ 0x1111)
        u = O.seeded_f32s(intermediate * hidden, seed ^ e ^ 0x2222)
        d = O.seeded_f32s(out_dim * intermediate, seed ^ e ^ 0x3333)
        gw, gs = O.split_interleaved_fp4(O.quantize_matrix(O.FP4_E2M1, g, intermediate, hidden), intermediate, hidden)
        uw, us = O.split_interleaved_fp4(O.quantize_matrix(O.FP4_E2M1, u, intermediate, hidden), intermediate, hidden)
        dw, ds = O.split_interleaved_fp4(O.quantize_matrix(O.FP4_E2M1, d, out_dim, intermediate), out_dim,
                                         intermediate)
        out.append((gw, gs, uw, us, dw, ds))
    return out
