"""Dense bf16 GEMV and the bf16 SwiGLU FFN (the shared expert of the
DeepSeek-style layer) against the reference arithmetic: bf16 widened to f32
by a 16-bit shift (objeta-parser lib.rs:334-337), f32 dot products
(oro_dense_gemv), SwiGLU as silu_mul (kernels/moe.cu:2-22).  Bound: max
|err| <= 1e-5 * sum |w x| per row, propagated through SwiGLU for the FFN."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import TOL

pytestmark = pytest.mark.gpu


def _bf16(rng, rows, cols, scale=0.02):
    w = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
    return (w.view(np.uint32) >> 16).astype(np.uint16)          # truncated to bf16 bits


def _widen(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("rows,cols", [(256, 4096), (4096, 2048), (1000, 2080), (7, 32)])
def test_bf16_gemv_matches_reference(cuda_device, rows, cols):
    import torch
    from objeta_b200.quant import gemv_bf16_device
    rng = np.random.default_rng(rows + cols)
    w = _bf16(rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    dw = torch.from_numpy(w.view(np.int16)).cuda()
    y = torch.empty(rows, device="cuda")
    gemv_bf16_device(dw, torch.from_numpy(x).cuda(), y, rows, cols)
    torch.cuda.synchronize()
    wf = _widen(w)
    ref = O.dense_gemv(wf, x, rows, cols)
    bound = TOL * (np.abs(wf.astype(np.float64)) @ np.abs(x.astype(np.float64)))
    err = np.abs(y.cpu().numpy().astype(np.float64) - ref)
    assert np.all(err <= bound), f"max err {err.max()}"


def test_bf16_gemv_unaligned_fallback(cuda_device):
    import torch
    from objeta_b200.quant import gemv_bf16_device
    rng = np.random.default_rng(5)
    rows, cols = 64, 512
    w = _bf16(rng, rows, cols)
    buf = torch.zeros(rows * cols + 8, dtype=torch.int16, device="cuda")
    buf[1:1 + rows * cols] = torch.from_numpy(w.view(np.int16).reshape(-1)).cuda()
    x = rng.standard_normal(cols).astype(np.float32)
    y = torch.empty(rows, device="cuda")
    gemv_bf16_device(buf[1:], torch.from_numpy(x).cuda(), y, rows, cols)
    torch.cuda.synchronize()
    wf = _widen(w)
    ref = O.dense_gemv(wf, x, rows, cols)
    bound = TOL * (np.abs(wf.astype(np.float64)) @ np.abs(x.astype(np.float64)))
    assert np.all(np.abs(y.cpu().numpy() - ref) <= bound)


def _ffn_ref(wg, wu, wd, x, H, I, O_):
    g = O.dense_gemv(_widen(wg), x, I, H)
    u = O.dense_gemv(_widen(wu), x, I, H)
    act = np.array([np.float32(v / (np.float32(1) + np.exp(np.float32(-v)))) * np.float32(q)
                    for v, q in zip(g, u)], np.float32)
    return O.dense_gemv(_widen(wd), act, O_, I), g, u


@pytest.mark.parametrize("accumulate", [False, True])
def test_bf16_ffn_shared_expert(cuda_device, accumulate):
    import torch
    from objeta_b200.moe import ffn_bf16_device
    H, I, O_ = 4096, 2048, 4096
    rng = np.random.default_rng(11)
    wg, wu, wd = _bf16(rng, I, H), _bf16(rng, I, H), _bf16(rng, O_, I)
    x = rng.standard_normal(H).astype(np.float32)
    base = rng.standard_normal(O_).astype(np.float32)
    out = torch.from_numpy(base.copy()).cuda()
    t = lambda a: torch.from_numpy(a.view(np.int16)).cuda()
    ffn_bf16_device(t(wg), t(wu), t(wd), H, I, O_, torch.from_numpy(x).cuda(), out, accumulate=accumulate)
    torch.cuda.synchronize()
    ref, g, u = _ffn_ref(wg, wu, wd, x, H, I, O_)
    if accumulate:
        ref = (base + ref).astype(np.float32)
    # bound: the down bound plus the activation error pushed through |Wd|
    G = np.abs(_widen(wg).astype(np.float64)) @ np.abs(x.astype(np.float64))
    U = np.abs(_widen(wu).astype(np.float64)) @ np.abs(x.astype(np.float64))
    s = 1.0 / (1.0 + np.exp(-g.astype(np.float64)))
    ds = s * (1 + g * (1 - s))
    act = (g * s * u).astype(np.float64)
    dact = np.abs(ds * u) * TOL * G + np.abs(g * s) * TOL * U + 1e-6 * np.abs(act)
    Wd = np.abs(_widen(wd).astype(np.float64))
    bound = TOL * (Wd @ np.abs(act)) + Wd @ dact + (np.abs(ref) * 1.2e-7 if accumulate else 0)
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref)
    assert np.all(err <= bound), f"max err {err.max()}"
