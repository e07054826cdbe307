"""Multi-token MoE on the device: (expert, token) pairs, the slot-order
combine, the batched router, and the expert-parallel layer on one GPU and on
two (NCCL ranks, skipped with fewer than two GPUs).

Every pair output goes through the row programs of the single-token launch,
so a token's combined output must be bit-identical to the fused single-token
path (objb_moe_selected_device), which the MoE tests check against the
reference CPU MoE within max |err| <= 1e-5 * sum|w x| propagated."""
import os
import socket

import numpy as np
import pytest

from oracle import oracle as O
from tests._moe_util import moe_bound, q4_matrices

pytestmark = pytest.mark.gpu


def _q4_layer(fmt, E, H, I, OUT, seed, unaligned=False):
    import torch
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    from objeta_b200.moe import MoeLayer
    qb = QuantBackend(torch.cuda.current_device())
    g = torch.Generator(device="cuda").manual_seed(seed)
    mats = {"gate": [], "up": [], "down": []}
    keep = []
    for _ in range(E):
        for name, (r, c) in (("gate", (I, H)), ("up", (I, H)), ("down", (OUT, I))):
            m = torch.randn(r, c, device="cuda", generator=g) * 0.02
            q = qb.quantize_matrix_device(QuantFormat(fmt), m, QGemvShape.new(QuantFormat(fmt), r, c))
            if unaligned:  # shift by 4 bytes: the layer takes the generic path
                buf = torch.empty(q.numel() + 16, dtype=torch.uint8, device="cuda")
                buf[4:4 + q.numel()] = q
                keep.append(buf)
                q = buf[4:4 + q.numel()]
            mats[name].append(q)
    layer = MoeLayer(fmt, H, I, OUT, mats["gate"], mats["up"], mats["down"])
    layer._keep = keep
    return layer, mats


def _fp4_layer(E, H, I, OUT, seed):
    import torch
    from objeta_b200.moe import MoeLayer
    g = torch.Generator(device="cuda").manual_seed(seed)
    t = {n: [] for n in ("gw", "gs", "uw", "us", "dw", "ds")}
    for _ in range(E):
        for wn, sn, r, c in (("gw", "gs", I, H), ("uw", "us", I, H), ("dw", "ds", OUT, I)):
            t[wn].append(torch.randint(0, 256, (r * c // 2,), device="cuda", dtype=torch.uint8, generator=g))
            t[sn].append(torch.randint(119, 124, (r * c // 32,), device="cuda", dtype=torch.uint8, generator=g))
    return MoeLayer(O.FP4_E2M1, H, I, OUT, t["gw"], t["uw"], t["dw"], t["gs"], t["us"], t["ds"]), t


def _routes(T, E, K, seed):
    rng = np.random.default_rng(seed)
    ids, ws = [], []
    for _ in range(T):
        i, w = O.router_from_logits(rng.standard_normal(E).astype(np.float32), K, True)
        ids.append(i)
        ws.append(w)
    return np.array(ids, np.int32), np.array(ws, np.float32)


def _fused_per_token(layer, x, ids, ws):
    import torch
    outs = []
    for t in range(x.shape[0]):
        outs.append(layer.forward_selected(ids[t].contiguous(), ws[t].contiguous(), x[t].contiguous()))
    torch.cuda.synchronize()
    return torch.stack(outs)


def _pairs_then_combine(layer, x, ids, ws, permute=False):
    """All T*K (token, slot) pairs in one launch (optionally in a shuffled
    compute order with pair_out restoring the row), then the combine."""
    import torch
    from objeta_b200.ep import moe_combine, moe_pairs
    T, K = ids.shape
    pe = ids.reshape(-1).to(torch.int32)
    pt = torch.arange(T, dtype=torch.int32, device="cuda").repeat_interleave(K)
    po = None
    if permute:
        perm = torch.from_numpy(np.random.default_rng(5).permutation(T * K)).cuda()
        pe, pt, po = pe[perm], pt[perm], perm.to(torch.int32)
    v = torch.full((T * K, layer.out_dim), float("nan"), device="cuda")
    moe_pairs(layer, pe.contiguous(), pt.contiguous(), x, v, pair_out=po)
    slot = torch.arange(T * K, dtype=torch.int32, device="cuda").reshape(T, K)
    out = torch.empty(T, layer.out_dim, device="cuda")
    moe_combine(v, slot, ws, out)
    torch.cuda.synchronize()
    return out


def _bits_equal(a, b):
    return np.array_equal(a.cpu().numpy().view(np.uint32), b.cpu().numpy().view(np.uint32))


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q5_0, O.IQ3_0])
@pytest.mark.parametrize("permute", [False, True])
def test_pairs_bit_identical_to_fused(cuda_device, fmt, permute):
    import torch
    E, H, I, OUT, K, T = 8, 1024, 1536, 1024, 2, 6
    layer, _ = _q4_layer(fmt, E, H, I, OUT, seed=fmt + 11)
    ids, ws = _routes(T, E, K, seed=fmt)
    x = torch.randn(T, H, device="cuda")
    di, dw = torch.from_numpy(ids).cuda(), torch.from_numpy(ws).cuda()
    ref = _fused_per_token(layer, x, di, dw)
    got = _pairs_then_combine(layer, x, di, dw, permute=permute)
    assert _bits_equal(got, ref)


def test_pairs_fp4_split_bit_identical_to_fused(cuda_device):
    import torch
    E, H, I, OUT, K, T = 16, 2048, 1024, 2048, 4, 5
    layer, _ = _fp4_layer(E, H, I, OUT, seed=3)
    ids, ws = _routes(T, E, K, seed=9)
    x = torch.randn(T, H, device="cuda")
    di, dw = torch.from_numpy(ids).cuda(), torch.from_numpy(ws).cuda()
    assert _bits_equal(_pairs_then_combine(layer, x, di, dw, permute=True), _fused_per_token(layer, x, di, dw))


def test_pairs_generic_path_bit_identical_to_fused(cuda_device):
    import torch
    E, H, I, OUT, K, T = 4, 256, 320, 192, 2, 3
    layer, _ = _q4_layer(O.Q4_0, E, H, I, OUT, seed=21, unaligned=True)
    assert layer._c.flags & 1
    ids, ws = _routes(T, E, K, seed=2)
    x = torch.randn(T, H, device="cuda")
    di, dw = torch.from_numpy(ids).cuda(), torch.from_numpy(ws).cuda()
    assert _bits_equal(_pairs_then_combine(layer, x, di, dw, permute=True), _fused_per_token(layer, x, di, dw))


def test_pairs_within_reference_bound(cuda_device):
    import torch
    E, H, I, OUT, K, T = 8, 512, 768, 512, 3, 4
    layer, mats = _q4_layer(O.Q4_0, E, H, I, OUT, seed=31)
    ids, ws = _routes(T, E, K, seed=4)
    xs = np.random.default_rng(8).standard_normal((T, H)).astype(np.float32)
    got = _pairs_then_combine(layer, torch.from_numpy(xs).cuda(), torch.from_numpy(ids).cuda(),
                              torch.from_numpy(ws).cuda()).cpu().numpy()
    host = [(mats["gate"][e].cpu().numpy(), mats["up"][e].cpu().numpy(), mats["down"][e].cpu().numpy())
            for e in range(E)]
    for t in range(T):
        sel = list(zip(ids[t].tolist(), ws[t].tolist()))
        ref = O.selected_moe_q4(host, sel, xs[t], H, I, OUT)
        bound = moe_bound(q4_matrices(host, H, I, OUT), sel, xs[t], H, I, OUT)
        err = np.abs(got[t].astype(np.float64) - ref.astype(np.float64))
        assert np.all(err <= bound), f"token {t}: max err {err.max()}"


def test_router_batched_matches_single(cuda_device):
    import torch
    from objeta_b200.ep import router_topk_batched
    from objeta_b200.moe import router_topk
    T, E, K = 9, 256, 8
    logits = torch.randn(T, E, device="cuda")
    logits[3, 10] = logits[3, 20]  # a tie: the lower index first
    ids, w = router_topk_batched(logits, K, renormalize=True)
    for t in range(T):
        i1, w1 = router_topk(logits[t].contiguous(), K, renormalize=True)
        assert torch.equal(ids[t], i1) and _bits_equal(w[t], w1)
        ri, rw = O.router_from_logits(logits[t].cpu().numpy(), K, True)
        assert ids[t].cpu().numpy().tolist() == ri.tolist()


def test_pairs_bad_index_is_flagged(cuda_device):
    import torch
    from objeta_b200.ep import moe_pairs
    from objeta_b200.quant import device_error_take
    E, H, I, OUT = 4, 256, 256, 256
    layer, _ = _q4_layer(O.Q4_0, E, H, I, OUT, seed=41)
    device_error_take(cuda_device)
    x = torch.randn(2, H, device="cuda")
    v = torch.empty(2, OUT, device="cuda")
    moe_pairs(layer, torch.tensor([1, 2], dtype=torch.int32, device="cuda"),
              torch.tensor([0, 5], dtype=torch.int32, device="cuda"), x, v)
    torch.cuda.synchronize()
    assert device_error_take(cuda_device) & 8


def test_ep_single_rank_matches_fused(cuda_device):
    import torch
    from objeta_b200.ep import ExpertParallelMoe
    E, H, I, OUT, K, T = 16, 1024, 512, 1024, 4, 7
    layer, _ = _q4_layer(O.Q4_0, E, H, I, OUT, seed=51)
    ids, ws = _routes(T, E, K, seed=6)
    x = torch.randn(T, H, device="cuda")
    di, dw = torch.from_numpy(ids).cuda(), torch.from_numpy(ws).cuda()
    ref = _fused_per_token(layer, x, di, dw)
    for host in (False, True):  # device-only one-rank path, and the multi-rank (host plan) path
        ep = ExpertParallelMoe(layer, E, K, plan_on_host=host)
        for _ in range(2):
            got = ep.forward(x, di, dw)
            torch.cuda.synchronize()
            assert _bits_equal(got, ref)


# ------------------------------------------------------------ two ranks
def _ep_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from objeta_b200.ep import ExpertParallelMoe
    from objeta_b200.moe import MoeLayer
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        E, H, I, OUT, K, T = 16, 1024, 512, 1024, 4, 6
        full, mats = _q4_layer(O.Q4_0, E, H, I, OUT, seed=61)   # same seed: same experts on every rank
        epr = E // world
        sl = slice(rank * epr, (rank + 1) * epr)
        shard = MoeLayer(O.Q4_0, H, I, OUT, mats["gate"][sl], mats["up"][sl], mats["down"][sl])
        ids, ws = _routes(T, E, K, seed=70 + rank)
        x = torch.from_numpy(np.random.default_rng(90 + rank).standard_normal((T, H)).astype(np.float32)).cuda()
        di, dw = torch.from_numpy(ids).cuda(), torch.from_numpy(ws).cuda()
        ep = ExpertParallelMoe(shard, E, K, rank=rank, world=world)
        got = ep.forward(x, di, dw)
        ref = _fused_per_token(full, x, di, dw)
        ok = _bits_equal(got, ref)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, None))
    except Exception as exc:
        q.put((rank, False, repr(exc)))


def test_ep_two_ranks_bit_identical_to_single_gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_ep_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert ok, f"rank {rank}: EP output differs from the single-GPU fused path"
