"""The official DeepSeek arithmetic on the device (activations quantized to
FP8 E4M3 with E8M0 scales per 128 values) against the reference CPU
functions restated in the oracle (crates/objeta-parser/src/deepseek.rs:
1444-1715):

* act_quant codes and scales bit-exact (the reference's own CUDA kernel is
  only held to "scales exact, few code mismatches", quant.rs:1450-1510);
* FP8 x FP4 and FP8 x FP8 GEMVs within max |err| <= 1e-5 * sum |a w| per
  row, and the reference tests' cosine > 0.9999 (quant.rs:1543-1600);
* the routed MoE (device layer and executor, with the FP8 shared expert)
  at the reference's cosine bar: its intermediate activation is itself
  re-quantized to FP8, so a 1e-7 difference upstream may move one FP8 code
  by a step, which no per-row fp32 bound can absorb.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import TOL

pytestmark = pytest.mark.gpu

E4M3 = np.array([O.f8e4m3_to_f32(c) for c in range(256)], np.float64)
FP4P = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, 0, -0.5, -1, -1.5, -2, -3, -4, -6], np.float64)


def e8m0(raw):
    raw = np.asarray(raw, np.int64)
    return np.where(raw == 0, 2.0 ** -127, np.ldexp(1.0, (raw - 127).astype(np.int64)))


def _act_values(codes, scales):
    a = E4M3[np.asarray(codes, np.int64)]
    return a * np.repeat(e8m0(scales), 128)[: a.size]


def _fp4_dense(w, ws, rows, cols):
    w = np.asarray(w, np.uint8).reshape(rows, cols // 2)
    lo, hi = FP4P[w & 0xF], FP4P[w >> 4]
    d = np.empty((rows, cols))
    d[:, 0::2], d[:, 1::2] = lo, hi
    return d * np.repeat(e8m0(np.asarray(ws).reshape(rows, cols // 32)), 32, axis=1)


def _cos(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


# ------------------------------------------------------------- act_quant
def _act_inputs():
    rng = np.random.default_rng(3)
    yield np.arange(1, 129, dtype=np.float32), 1, 128                      # quant.rs:1450 input
    yield ((np.arange(256) - 128.0) * 0.5).astype(np.float32), 1, 256       # quant.rs:1479 input
    yield (np.sin(np.arange(1024, dtype=np.float32)) * 100).astype(np.float32), 4, 256  # quant.rs:1496
    mags = np.array([1e-6, 1e-3, 0.01, 1.0, 30.0, 1e4], np.float32)
    x = (rng.standard_normal((6, 2048)) * mags[:, None]).astype(np.float32)
    x[0, :128] = 0.0                                                        # an all-zero block
    x[1, 5] = 448.0 * 2 ** -7                                               # exact power-of-two cases
    yield x.reshape(-1), 6, 2048
    # values on E4M3 rounding midpoints relative to their block scale
    base = np.array([O.f8e4m3_to_f32(c) for c in range(0x08, 0x77)], np.float32)
    mid = ((base[:-1] + base[1:]) / 2).astype(np.float32)
    v = np.resize(np.concatenate([mid, -mid, base]), 1024).astype(np.float32)
    v[::128] = 448.0                                                        # pin each block's scale to 2^0
    yield v, 8, 128


@pytest.mark.parametrize("case", range(5))
def test_act_quant_bit_exact(cuda_device, case):
    import torch
    from objeta_b200.quant import act_quant_device
    x, rows, cols = list(_act_inputs())[case]
    vals, scales = act_quant_device(torch.from_numpy(x).cuda(), rows, cols)
    torch.cuda.synchronize()
    ry, rs = O.act_quant(x, 128)
    assert np.array_equal(scales.cpu().numpy(), rs)
    assert np.array_equal(vals.cpu().numpy(), ry)


def test_act_quant_rejects_non_multiple_cols(cuda_device):
    """quant.rs:1601-1608."""
    from objeta_b200._lib import CudaError
    from objeta_b200.quant import cuda_act_quant
    with pytest.raises(CudaError) as e:
        cuda_act_quant(None, None, np.ones(100, np.float32), 1, 100)
    assert e.value.kind == "InvalidInput" and "not divisible by 128" in e.value.source_message


# ----------------------------------------------------------------- GEMVs
def _fp8_fp4_fixture(rows, cols, seed):
    rng = np.random.default_rng(seed)
    x = (rng.uniform(-1, 1, cols) * 100).astype(np.float32)
    act, act_s = O.act_quant(x, 128)
    w = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
    ws = rng.integers(120, 135, rows * cols // 32, dtype=np.uint8)
    return act, act_s, w, ws


@pytest.mark.parametrize("rows,cols", [(1, 128), (2, 256), (300, 1536), (2048, 4096), (4096, 2048)])
def test_fp8_fp4_gemv(cuda_device, rows, cols):
    """quant.rs:1543-1600 shapes (small, multiblock, realistic gate / down)
    plus a non-multiple-of-512 width that takes the generic kernel."""
    import torch
    from objeta_b200.quant import gemv_fp8_fp4_device
    act, act_s, w, ws = _fp8_fp4_fixture(rows, cols, rows + cols)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    y = torch.empty(rows, device="cuda")
    gemv_fp8_fp4_device(t(act), t(act_s), t(w), t(ws), y, rows, cols)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    ref = O.fp8_act_fp4_weight_gemv_f32(act, act_s, w, ws, rows, cols).astype(np.float64)
    bound = TOL * (np.abs(_fp4_dense(w, ws, rows, cols)) @ np.abs(_act_values(act, act_s)))
    assert np.all(np.abs(got - ref) <= bound), f"max err {np.abs(got - ref).max()}"
    assert _cos(got, ref) > 0.9999


def _fp8_weights(rng, rows, cols):
    # E4M3 codes with exponent fields 1..10 (|w| <= 8), both signs, a few exponent-0 and -15 codes
    e = rng.integers(1, 11, rows * cols)
    m = rng.integers(0, 8, rows * cols)
    s = rng.integers(0, 2, rows * cols)
    c = (s << 7) | (e << 3) | m
    c[::97] = 0x7F                      # exponent 15: decodes as 448
    c[::89] = 0x05                      # exponent 0: decodes as 5 * 2^-5
    ws = rng.integers(118, 124, ((rows + 127) // 128) * ((cols + 127) // 128), dtype=np.uint8)
    return c.astype(np.uint8), ws


@pytest.mark.parametrize("rows,cols", [(256, 1024), (2048, 4096), (4096, 2048), (200, 384)])
def test_fp8_fp8_gemv(cuda_device, rows, cols):
    import torch
    from objeta_b200.quant import gemv_fp8_fp8_device
    rng = np.random.default_rng(rows)
    x = rng.standard_normal(cols).astype(np.float32)
    act, act_s = O.act_quant(x, 128)
    w, ws = _fp8_weights(rng, rows, cols)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    y = torch.empty(rows, device="cuda")
    gemv_fp8_fp8_device(t(act), t(act_s), t(w), t(ws), y, rows, cols)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    ref = O.fp8_act_fp8_weight_gemv(act, act_s, w, ws, rows, cols).astype(np.float64)
    tiles = (cols + 127) // 128
    wd = E4M3[w.reshape(rows, cols)] * np.repeat(np.repeat(e8m0(ws).reshape(-1, tiles), 128, 0)[:rows], 128, 1)[:, :cols]
    bound = TOL * (np.abs(wd) @ np.abs(_act_values(act, act_s)))
    assert np.all(np.abs(got - ref) <= bound), f"max err {np.abs(got - ref).max()}"


# ------------------------------------------------------------- routed MoE
def _official_experts(E, H, I, O_, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    t = {n: [] for n in ("gw", "gs", "uw", "us", "dw", "ds")}
    for _ in range(E):
        for wn, sn, r, c in (("gw", "gs", I, H), ("uw", "us", I, H), ("dw", "ds", O_, I)):
            t[wn].append(torch.randint(0, 256, (r * c // 2,), device="cuda", dtype=torch.uint8, generator=g))
            t[sn].append(torch.randint(119, 124, (r * c // 32,), device="cuda", dtype=torch.uint8, generator=g))
    return t


def _oracle_routed(t, sel, x, H, I, O_, limit=10.0):
    out = np.zeros(O_, np.float32)
    for e, w in sel:
        h = [t[n][e].cpu().numpy() for n in ("gw", "gs", "uw", "us", "dw", "ds")]
        v = O.routed_expert_fp4_official_f32(*h, x, H, I, O_, limit)
        out = (out + np.float32(w) * v).astype(np.float32)
    return out


def test_official_moe_layer_matches_reference(cuda_device):
    import torch
    from objeta_b200.moe import MoeLayer
    E, H, I, O_, K = 8, 1024, 512, 1024, 3
    t = _official_experts(E, H, I, O_, seed=5)
    layer = MoeLayer(O.FP4_E2M1, H, I, O_, t["gw"], t["uw"], t["dw"], t["gs"], t["us"], t["ds"])
    rng = np.random.default_rng(1)
    for trial in range(3):
        x = rng.standard_normal(H).astype(np.float32)
        ids, w = O.router_from_logits(rng.standard_normal(E).astype(np.float32), K, True)
        sel = list(zip(ids.tolist(), w.tolist()))
        got = layer.forward_official_selected(torch.from_numpy(ids.astype(np.int32)).cuda(),
                                              torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda())
        torch.cuda.synchronize()
        ref = _oracle_routed(t, sel, x, H, I, O_)
        num = O.compare_outputs(ref, got.cpu().numpy())
        assert num["cosine_similarity"] > 0.9999 and num["relative_l2_error"] < 1e-3, (trial, num)


def test_official_executor_with_fp8_shared_expert(cuda_device):
    import torch
    from objeta_b200 import QuantBackend
    from objeta_b200.moe import (CudaExpertCache, DeepSeekFp4ExpertWeights, DeepSeekFp8SharedExpertWeightsDevice,
                                 MoeExecutor, MoeLayer)
    E, H, I, O_, K = 6, 1024, 512, 1024, 2
    t = _official_experts(E, H, I, O_, seed=9)
    host = [DeepSeekFp4ExpertWeights(*[t[n][e].cpu().numpy() for n in ("gw", "gs", "uw", "us", "dw", "ds")])
            for e in range(E)]
    rng = np.random.default_rng(2)
    sw = {}
    for n, (r, c) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
        w, s = _fp8_weights(rng, r, c)
        sw[n] = (w, s)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    shared = DeepSeekFp8SharedExpertWeightsDevice(dev(sw["gate"][0]), dev(sw["gate"][1]), dev(sw["up"][0]),
                                                  dev(sw["up"][1]), dev(sw["down"][0]), dev(sw["down"][1]))
    x = rng.standard_normal(H).astype(np.float32)
    sel = [(4, 0.7), (1, 0.3)]
    ex = MoeExecutor(0)
    cache = CudaExpertCache(1 << 30, 0)
    out, tel = ex.execute_selected_moe_official_routed_fp4_cuda(QuantBackend(0), None, host, sel, x, H, I, O_, 0,
                                                               cache, shared_expert=shared)
    routed_only, _ = ex.execute_selected_moe_official_routed_fp4_cuda(QuantBackend(0), None, host, sel, x, H, I, O_,
                                                                      0, cache)
    # routed part: the device layer gives the same bits
    layer = MoeLayer(O.FP4_E2M1, H, I, O_, t["gw"], t["uw"], t["dw"], t["gs"], t["us"], t["ds"])
    lay = layer.forward_official_selected(torch.tensor([4, 1], dtype=torch.int32, device="cuda"),
                                          torch.tensor([0.7, 0.3], device="cuda"), torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(routed_only.view(np.uint32), lay.cpu().numpy().view(np.uint32))
    # shared part against the reference CPU shared expert (limit 10 as the executor)
    shared_ref = O.shared_expert_fp8_official(sw["gate"][0], sw["gate"][1], sw["up"][0], sw["up"][1],
                                              sw["down"][0], sw["down"][1], x, H, I, 10.0)
    num = O.compare_outputs(shared_ref, (out - routed_only).astype(np.float32))
    assert num["cosine_similarity"] > 0.9999, num
    ref_total = (_oracle_routed(t, sel, x, H, I, O_) + shared_ref).astype(np.float32)
    num = O.compare_outputs(ref_total, out)
    assert num["cosine_similarity"] > 0.9999 and num["relative_l2_error"] < 1e-3, num
    # telemetry (moe.rs:1612-1650)
    assert tel.shared_fp8_bytes_loaded == 2 * I * H + H * I + 2 * I * H // 128 + H * I // 128
    assert tel.routed_fp4_bytes_loaded + tel.routed_fp4_bytes_reused == tel.logical_expert_bytes_requested
    assert tel.shared_expert_ms > 0.0
