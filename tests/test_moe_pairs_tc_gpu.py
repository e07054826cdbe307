"""The tensor-core (tcgen05 kind::i8) multi-token pairs path for Q4_0 layers.

Its block sums are the exact integers of the CUDA-core digit path; only the
f32 order of the block terms differs.  So: every combined token is within the
reference MoE bound (max |err| <= 1e-5 * sum|w x| propagated) of the CPU
oracle, every pair row is close to the CUDA-core pairs row, and a pair row is
a function of (expert, token) alone -- the same bits whatever else is in the
pair list, in whichever slice of 32 it lands."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._moe_util import moe_bound, q4_matrices
from tests.test_moe_pairs_gpu import _bits_equal, _q4_layer, _routes

pytestmark = pytest.mark.gpu


def _sorted_pairs(ids):
    import torch
    T, K = ids.shape
    pe = ids.reshape(-1).astype(np.int32)
    pt = np.repeat(np.arange(T, dtype=np.int32), K)
    po = np.arange(T * K, dtype=np.int32)
    order = np.argsort(pe, kind="stable")

    def cuda(a):
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return cuda(pe[order]), cuda(pt[order]), cuda(po[order])


def _zipf_routes(T, E, K, seed, a=1.1):
    """Skewed routing: a few hot experts get runs far longer than 32."""
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, E + 1) ** a
    p /= p.sum()
    ids = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    ws = rng.random((T, K)).astype(np.float32)
    ws /= ws.sum(1, keepdims=True)
    return ids, ws


def _run_both(layer, x, pe, pt, po, rows):
    import torch
    from objeta_b200.ep import moe_pairs, moe_pairs_tc
    v_tc = torch.full((rows, layer.out_dim), float("nan"), device="cuda")
    v_cc = torch.full((rows, layer.out_dim), float("nan"), device="cuda")
    moe_pairs_tc(layer, pe, pt, x, v_tc, pair_out=po)
    moe_pairs(layer, pe, pt, x, v_cc, pair_out=po)
    torch.cuda.synchronize()
    return v_tc, v_cc


@pytest.mark.parametrize("shape", [(8, 512, 768, 544, 3, 40), (64, 2048, 512, 2048, 8, 64),
                                   (16, 1024, 256, 1152, 4, 300)])
def test_tc_pairs_within_reference_bound(cuda_device, shape):
    import torch
    from objeta_b200.ep import moe_combine
    from objeta_b200.quant import device_error_take
    E, H, I, OUT, K, T = shape
    layer, mats = _q4_layer(O.Q4_0, E, H, I, OUT, seed=E + H)
    ids, ws = _zipf_routes(T, E, K, seed=E)
    xs = np.random.default_rng(T).standard_normal((T, H)).astype(np.float32)
    x = torch.from_numpy(xs).cuda()
    pe, pt, po = _sorted_pairs(ids)
    device_error_take(cuda_device)
    v_tc, v_cc = _run_both(layer, x, pe, pt, po, T * K)
    assert device_error_take(cuda_device) == 0
    assert torch.isfinite(v_tc).all()
    scale = float(v_cc.abs().max())
    diff = float((v_tc - v_cc).abs().max())
    assert diff <= 1e-5 * scale, f"tc vs CUDA-core pairs: {diff} of {scale}"
    slot = torch.arange(T * K, dtype=torch.int32, device="cuda").reshape(T, K)
    out = torch.empty(T, OUT, device="cuda")
    moe_combine(v_tc, slot, torch.from_numpy(ws).cuda(), out)
    got = out.cpu().numpy()
    host = [(mats["gate"][e].cpu().numpy(), mats["up"][e].cpu().numpy(), mats["down"][e].cpu().numpy())
            for e in range(E)]
    for t in range(min(T, 6)):
        sel = list(zip(ids[t].tolist(), ws[t].tolist()))
        ref = O.selected_moe_q4(host, sel, xs[t], H, I, OUT)
        bound = moe_bound(q4_matrices(host, H, I, OUT), sel, xs[t], H, I, OUT)
        err = np.abs(got[t].astype(np.float64) - ref.astype(np.float64))
        assert np.all(err <= bound), f"token {t}: max err {err.max()} (bound {bound.min()})"


def test_tc_pair_rows_independent_of_grouping(cuda_device):
    """A pair's row is the same bits when it shares a slice with 31 others,
    when its run is cut at another place, and when it runs alone."""
    import torch
    from objeta_b200.ep import moe_pairs_tc
    E, H, I, OUT, K, T = 4, 1024, 512, 768, 2, 70
    layer, _ = _q4_layer(O.Q4_0, E, H, I, OUT, seed=5)
    ids, _ = _zipf_routes(T, E, K, seed=3)
    x = torch.randn(T, H, device="cuda")
    pe, pt, po = _sorted_pairs(ids)
    v_all = torch.empty(T * K, OUT, device="cuda")
    moe_pairs_tc(layer, pe, pt, x, v_all, pair_out=po)
    # the same list without its first 7 pairs: every later slice boundary moves
    v_sub = torch.empty(T * K, OUT, device="cuda")
    moe_pairs_tc(layer, pe[7:].contiguous(), pt[7:].contiguous(), x, v_sub, pair_out=po[7:].contiguous())
    torch.cuda.synchronize()
    rows = po[7:].long()
    assert _bits_equal(v_all[rows], v_sub[rows])
    for p in (0, 40, len(pe) - 1):
        v1 = torch.empty(1, OUT, device="cuda")
        moe_pairs_tc(layer, pe[p:p + 1].contiguous(), pt[p:p + 1].contiguous(), x, v1)
        torch.cuda.synchronize()
        assert _bits_equal(v1[0], v_all[int(po[p])])


def test_tc_pairs_device_count(cuda_device):
    """d_count below the array length: only the first n pairs run; rows of
    the others are untouched."""
    import torch
    from objeta_b200.ep import moe_pairs_tc
    E, H, I, OUT, K, T = 8, 1024, 512, 1024, 4, 20
    layer, _ = _q4_layer(O.Q4_0, E, H, I, OUT, seed=9)
    ids, _ = _routes(T, E, K, seed=12)
    x = torch.randn(T, H, device="cuda")
    pe, pt, po = _sorted_pairs(ids)
    n = 37
    v_full = torch.empty(T * K, OUT, device="cuda")
    moe_pairs_tc(layer, pe, pt, x, v_full, pair_out=po)
    v = torch.full((T * K, OUT), 7.0, device="cuda")
    cnt = torch.tensor([n], dtype=torch.int32, device="cuda")
    moe_pairs_tc(layer, pe, pt, x, v, pair_out=po, d_count=cnt)
    torch.cuda.synchronize()
    ran = po[:n].long()
    assert _bits_equal(v[ran], v_full[ran])
    rest = torch.ones(T * K, dtype=torch.bool, device="cuda")
    rest[ran] = False
    assert bool((v[rest] == 7.0).all())


def test_tc_pairs_bad_index_flagged(cuda_device):
    import torch
    from objeta_b200.ep import moe_pairs_tc
    from objeta_b200.quant import device_error_take
    E, H, I, OUT = 4, 256, 256, 256
    layer, _ = _q4_layer(O.Q4_0, E, H, I, OUT, seed=41)
    device_error_take(cuda_device)
    x = torch.randn(2, H, device="cuda")
    v = torch.empty(2, OUT, device="cuda")
    moe_pairs_tc(layer, torch.tensor([1, 2], dtype=torch.int32, device="cuda"),
                 torch.tensor([0, 5], dtype=torch.int32, device="cuda"), x, v)
    torch.cuda.synchronize()
    assert device_error_take(cuda_device) & 8


def test_tc_pairs_rejects_other_formats(cuda_device):
    import torch
    from objeta_b200._lib import CudaError
    from objeta_b200.ep import moe_pairs_tc
    layer, _ = _q4_layer(O.Q5_0, 2, 256, 256, 256, seed=1)
    x = torch.randn(1, 256, device="cuda")
    v = torch.empty(1, 256, device="cuda")
    with pytest.raises(CudaError):
        moe_pairs_tc(layer, torch.zeros(1, dtype=torch.int32, device="cuda"),
                     torch.zeros(1, dtype=torch.int32, device="cuda"), x, v)


def test_tc_pairs_rejects_unstaged_widths(cuda_device):
    """hidden / intermediate not a multiple of 256: rows are not whole 16-byte
    pieces per step, so the tensor-core path declines (the CUDA-core pairs
    path takes these layers)."""
    import torch
    from objeta_b200._lib import CudaError
    from objeta_b200.ep import moe_pairs_tc
    layer, _ = _q4_layer(O.Q4_0, 2, 512, 800, 256, seed=2)
    x = torch.randn(1, 512, device="cuda")
    v = torch.empty(1, 256, device="cuda")
    with pytest.raises(CudaError):
        moe_pairs_tc(layer, torch.zeros(1, dtype=torch.int32, device="cuda"),
                     torch.zeros(1, dtype=torch.int32, device="cuda"), x, v)


def test_tc_pairs_ungrouped_list_is_flagged(cuda_device):
    """A pair list that is not grouped by expert can need more slice-image
    space than the launch reserves: nothing runs, the device error word is
    flagged, and the output rows are left as they were."""
    import torch
    from objeta_b200.ep import moe_pairs_tc
    from objeta_b200.quant import device_error_take
    E, H, I, OUT, P = 2, 256, 256, 256, 96
    layer, _ = _q4_layer(O.Q4_0, E, H, I, OUT, seed=6)
    device_error_take(cuda_device)
    x = torch.randn(P, H, device="cuda")
    v = torch.full((P, OUT), 3.0, device="cuda")
    pe = (torch.arange(P, dtype=torch.int32, device="cuda") % 2).contiguous()
    pt = torch.arange(P, dtype=torch.int32, device="cuda")
    moe_pairs_tc(layer, pe, pt, x, v)
    torch.cuda.synchronize()
    assert device_error_take(cuda_device) & 8
    assert bool((v == 3.0).all())


def test_ep_grouped_matches_fused_and_plans(cuda_device):
    """ExpertParallelMoe at T * k >= GROUPED_MIN_SLOTS runs the grouped path:
    within the MoE bound of the fused single-token path (both against the
    oracle), and bit-identical between the device-sorted pair list and the
    host dispatch plan (rows depend only on (expert, token))."""
    import torch
    from objeta_b200.ep import GROUPED_MIN_SLOTS, ExpertParallelMoe
    E, H, I, OUT, K, T = 16, 1024, 512, 1024, 8, 40
    assert T * K >= GROUPED_MIN_SLOTS
    layer, mats = _q4_layer(O.Q4_0, E, H, I, OUT, seed=77)
    ids, ws = _zipf_routes(T, E, K, seed=21)
    xs = np.random.default_rng(4).standard_normal((T, H)).astype(np.float32)
    x, di, dw = torch.from_numpy(xs).cuda(), torch.from_numpy(ids).cuda(), torch.from_numpy(ws).cuda()
    a = ExpertParallelMoe(layer, E, K).forward(x, di, dw)
    b = ExpertParallelMoe(layer, E, K, plan_on_host=True).forward(x, di, dw)
    c = ExpertParallelMoe(layer, E, K, grouped="off").forward(x, di, dw)
    torch.cuda.synchronize()
    assert _bits_equal(a, b)
    assert not _bits_equal(a, c)  # the grouped path really ran
    host = [(mats["gate"][e].cpu().numpy(), mats["up"][e].cpu().numpy(), mats["down"][e].cpu().numpy())
            for e in range(E)]
    got, ref_c = a.cpu().numpy(), c.cpu().numpy()
    for t in range(0, T, 8):
        sel = list(zip(ids[t].tolist(), ws[t].tolist()))
        bound = moe_bound(q4_matrices(host, H, I, OUT), sel, xs[t], H, I, OUT)
        assert np.all(np.abs(got[t].astype(np.float64) - ref_c[t]) <= 2 * bound)
