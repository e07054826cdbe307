"""The allocation-free MoE entry point (objb_moe_selected_device_noalloc).

It exists for callers that cannot let the library allocate device memory --
a serving framework that reserves all of HBM up front and forbids
allocation on its hot path, or one whose allocator must account for every
byte -- and takes its scratch from a fixed array inside the library instead
of a cudaMalloc'd per-stream workspace.  This file calls it through the C
ABI twice in a row and checks each output against the regular entry point
(objb_moe_selected_device) on the same inputs, within the MoE parity bound
the other tests use.  It is collected last so a stop-at-first-failure run has
already run everything else, and it builds all of its own inputs so it also
passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests._moe_util import moe_bound, q4_matrices, fp4_matrices

pytestmark = pytest.mark.gpu


def _q4_layer(hidden, inter, out_dim, num_experts, seed):
    import torch
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    from objeta_b200.moe import MoeLayer
    qb = QuantBackend(torch.cuda.current_device())
    g = torch.Generator(device="cuda").manual_seed(seed)
    mats = {"gate": [], "up": [], "down": []}
    for _ in range(num_experts):
        for name, (r, c) in (("gate", (inter, hidden)), ("up", (inter, hidden)), ("down", (out_dim, inter))):
            m = torch.randn(r, c, device="cuda", generator=g) * 0.02
            mats[name].append(qb.quantize_matrix_device(QuantFormat.Q4_0, m, QGemvShape.new(QuantFormat.Q4_0, r, c)))
    layer = MoeLayer(QuantFormat.Q4_0, hidden, inter, out_dim, mats["gate"], mats["up"], mats["down"])
    host = [(mats["gate"][e].cpu().numpy(), mats["up"][e].cpu().numpy(), mats["down"][e].cpu().numpy())
            for e in range(num_experts)]
    return layer, q4_matrices(host, hidden, inter, out_dim)


def _fp4_layer(hidden, inter, out_dim, num_experts, seed):
    import torch
    from objeta_b200.moe import MoeLayer
    g = torch.Generator(device="cuda").manual_seed(seed)
    t = {n: [] for n in ("gw", "gs", "uw", "us", "dw", "ds")}
    for _ in range(num_experts):
        for wn, sn, r, c in (("gw", "gs", inter, hidden), ("uw", "us", inter, hidden), ("dw", "ds", out_dim, inter)):
            t[wn].append(torch.randint(0, 256, (r * c // 2,), device="cuda", dtype=torch.uint8, generator=g))
            t[sn].append(torch.randint(119, 124, (r * c // 32,), device="cuda", dtype=torch.uint8, generator=g))
    layer = MoeLayer(O.FP4_E2M1, hidden, inter, out_dim, t["gw"], t["uw"], t["dw"], t["gs"], t["us"], t["ds"])
    host = [tuple(t[n][e].cpu().numpy() for n in ("gw", "gs", "uw", "us", "dw", "ds")) for e in range(num_experts)]
    return layer, fp4_matrices(host, hidden, inter, out_dim)


def _noalloc_call(layer, ids, weights, x, out):
    """objb_moe_selected_device_noalloc through the C ABI."""
    from objeta_b200 import _lib
    fn = _lib.load().objb_moe_selected_device_noalloc
    st = fn(ctypes.byref(layer._c), ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(weights.data_ptr()),
            ctypes.c_size_t(ids.numel()), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
            ctypes.c_float(0.0), None)
    _lib.check(st)


@pytest.mark.parametrize("kind", ["q4", "fp4"])
def test_noalloc_matches_regular_entry_point(cuda_device, kind):
    import torch
    hidden, inter, out_dim, E = (1024, 2048, 1024, 8) if kind == "q4" else (1024, 1024, 512, 8)
    layer, mats = (_q4_layer if kind == "q4" else _fp4_layer)(hidden, inter, out_dim, E, seed=17)
    sel = [(5, 0.5), (2, 0.3), (7, 0.2)]
    ids = torch.tensor([e for e, _ in sel], dtype=torch.int32, device="cuda")
    w = torch.tensor([v for _, v in sel], dtype=torch.float32, device="cuda")
    rng = np.random.default_rng(3)
    for call in range(2):  # two calls in a row through the shared array
        x = rng.standard_normal(hidden).astype(np.float32)
        dx = torch.from_numpy(x).cuda()
        ref = layer.forward_selected(ids, w, dx)
        got = torch.full((out_dim,), float("nan"), device="cuda")
        _noalloc_call(layer, ids, w, dx, got)
        torch.cuda.synchronize()
        bound = moe_bound(mats, sel, x, hidden, inter, out_dim)
        err = np.abs(got.cpu().numpy().astype(np.float64) - ref.cpu().numpy().astype(np.float64))
        assert np.all(err <= bound), f"call {call}: max err {err.max()}"


def test_noalloc_rejects_layers_beyond_its_array(cuda_device):
    import torch
    from objeta_b200._lib import CudaError
    from objeta_b200.moe import MoeLayer
    hidden, inter, out_dim = 64, 1 << 16, 64
    t = [torch.zeros(inter * hidden // 32 * 18, dtype=torch.uint8, device="cuda")]
    d = [torch.zeros(out_dim * inter // 32 * 18, dtype=torch.uint8, device="cuda")]
    layer = MoeLayer(0, hidden, inter, out_dim, t, t, d)
    ids = torch.zeros(16, dtype=torch.int32, device="cuda")
    w = torch.zeros(16, dtype=torch.float32, device="cuda")
    x = torch.zeros(hidden, device="cuda")
    out = torch.zeros(out_dim, device="cuda")
    with pytest.raises(CudaError) as ei:
        _noalloc_call(layer, ids, w, x, out)
    assert ei.value.kind == "InvalidInput" and "allocation-free" in ei.value.source_message


def test_noalloc_device_error_poisons_output_then_recovers(cuda_device):
    """An out-of-range expert id (computed as expert 0 and flagged by the
    kernel's own check) turns the whole output into NaN; the next call with
    valid ids is clean again, since each call clears the error word."""
    import torch
    hidden, inter, out_dim, E = 512, 512, 256, 4
    layer, mats = _q4_layer(hidden, inter, out_dim, E, seed=23)
    x = torch.randn(hidden, device="cuda")
    w = torch.tensor([0.6, 0.4], device="cuda")
    out = torch.zeros(out_dim, device="cuda")
    _noalloc_call(layer, torch.tensor([1, E + 3], dtype=torch.int32, device="cuda"), w, x, out)
    torch.cuda.synchronize()
    assert torch.isnan(out).all()
    ids = torch.tensor([1, 3], dtype=torch.int32, device="cuda")
    _noalloc_call(layer, ids, w, x, out)
    ref = layer.forward_selected(ids, w, x)
    torch.cuda.synchronize()
    assert not torch.isnan(out).any()
    assert torch.equal(out, ref)


def _q4_layer_offset(hidden, inter, out_dim, num_experts, seed, offset):
    """A Q4_0 layer whose expert tensors start `offset` bytes into their
    allocations (offset % 16 != 0 marks the layer unaligned: generic path)."""
    import torch
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    from objeta_b200.moe import MoeLayer
    qb = QuantBackend(torch.cuda.current_device())
    g = torch.Generator(device="cuda").manual_seed(seed)
    mats = {"gate": [], "up": [], "down": []}
    for _ in range(num_experts):
        for name, (r, c) in (("gate", (inter, hidden)), ("up", (inter, hidden)), ("down", (out_dim, inter))):
            m = torch.randn(r, c, device="cuda", generator=g) * 0.02
            q = qb.quantize_matrix_device(QuantFormat.Q4_0, m, QGemvShape.new(QuantFormat.Q4_0, r, c))
            buf = torch.zeros(q.numel() + offset, dtype=torch.uint8, device="cuda")
            buf[offset:].copy_(q)
            mats[name].append(buf[offset:])
    return MoeLayer(QuantFormat.Q4_0, hidden, inter, out_dim, mats["gate"], mats["up"], mats["down"])


def test_noalloc_unaligned_offset_x_and_side_stream(cuda_device):
    """The generic (unaligned) path, an x that is not 16-byte aligned (the x
    image launch) and a side stream: each bit-identical to the regular entry
    point on the same inputs, which runs the same kernels with other scratch."""
    import torch
    hidden, inter, out_dim, E = 1024, 1024, 512, 6
    sel = torch.tensor([4, 1, 5], dtype=torch.int32, device="cuda")
    w = torch.tensor([0.5, 0.3, 0.2], device="cuda")
    x_store = torch.randn(hidden + 1, device="cuda")
    x_off = x_store[1:]  # data_ptr + 4: not 16-byte aligned
    aligned, _ = _q4_layer(hidden, inter, out_dim, E, seed=41)
    unaligned = _q4_layer_offset(hidden, inter, out_dim, E, seed=41, offset=2)
    assert unaligned._c.flags & 1
    side = torch.cuda.Stream()
    for layer, x in ((unaligned, x_store[:hidden]), (aligned, x_off), (unaligned, x_off)):
        for s in (torch.cuda.current_stream(), side):
            got = torch.full((out_dim,), float("nan"), device="cuda")
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                ref = layer.forward_selected(sel, w, x, stream=s)
                layer.forward_selected_noalloc(sel, w, x, got, stream=s)
            torch.cuda.synchronize()
            assert torch.equal(got, ref)


def test_noalloc_sizes_unaligned_layers_by_their_own_path(cuda_device):
    """An unaligned layer runs the generic path, which needs only the
    activations: one whose aligned (fast-path) plan would not fit the fixed
    array is still accepted."""
    import torch
    from objeta_b200._lib import CudaError
    hidden, inter, out_dim, E, K = 256, 30720, 256, 24, 24
    ids = torch.arange(K, dtype=torch.int32, device="cuda")
    w = torch.full((K,), 1.0 / K, device="cuda")
    x = torch.randn(hidden, device="cuda")
    aligned, _ = _q4_layer(hidden, inter, out_dim, E, seed=5)
    assert aligned.scratch_bytes(K) > (4 << 20) - 256
    with pytest.raises(CudaError):
        aligned.forward_selected_noalloc(ids, w, x, torch.zeros(out_dim, device="cuda"))
    unaligned = _q4_layer_offset(hidden, inter, out_dim, E, seed=5, offset=2)
    assert unaligned.scratch_bytes(K) <= (4 << 20) - 256
    got = torch.full((out_dim,), float("nan"), device="cuda")
    unaligned.forward_selected_noalloc(ids, w, x, got)
    ref = unaligned.forward_selected(ids, w, x)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
