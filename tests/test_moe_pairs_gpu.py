"""Multi-token MoE on the device: (expert, token) pairs, the slot-order
combine, the batched router, and the expert-parallel layer on one GPU and on
two (NCCL ranks, skipped with fewer than two GPUs).

Every pair output goes through the row programs of the single-token launch,
so a token's combined output must be bit-identical to the fused single-token
path (objb_moe_selected_device), which the MoE tests check against the
reference CPU MoE within max |err| <= 1e-5 * sum|w x| propagated."""
import os

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
        # one token: the fused single-token launch on the device-only path
        got1 = ep.forward(x[2:3].contiguous(), di[2:3].contiguous(), dw[2:3].contiguous())
        torch.cuda.synchronize()
        assert got1.shape == (1, OUT) and _bits_equal(got1[0], ref[2])


# ------------------------------------------------------------ two ranks
def _ep_rank(rank, world, port, q, grouped="auto", T=6, K=4):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from objeta_b200.ep import ExpertParallelMoe
    from objeta_b200.moe import MoeLayer
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        torch.cuda.set_device(rank)
        # the parent holds the rendezvous store (an OS-assigned port)
        store = dist.TCPStore("127.0.0.1", port, is_master=False, timeout=timedelta(seconds=60))
        dist.init_process_group("nccl", store=store, rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        E, H, I, OUT = 16, 1024, 512, 1024
        full, mats = _q4_layer(O.Q4_0, E, H, I, OUT, seed=61)   # same seed: same experts on every rank
        epr = E // world
        sl = slice(rank * epr, (rank + 1) * epr)
        shard = MoeLayer(O.Q4_0, H, I, OUT, mats["gate"][sl], mats["up"][sl], mats["down"][sl])
        ids, ws = _routes(T, E, K, seed=70 + rank)
        x = torch.from_numpy(np.random.default_rng(90 + rank).standard_normal((T, H)).astype(np.float32)).cuda()
        di, dw = torch.from_numpy(ids).cuda(), torch.from_numpy(ws).cuda()
        if grouped == "on":   # one GPU on the grouped path, all experts local
            ref = ExpertParallelMoe(full, E, K, grouped="on").forward(x, di, dw)
        else:
            ref = _fused_per_token(full, x, di, dw)
        # host plan: bit-identical to one GPU
        ep = ExpertParallelMoe(shard, E, K, rank=rank, world=world, exchange="host", grouped=grouped)
        ok = _bits_equal(ep.forward(x, di, dw), ref)
        # device exchange (one all-gather of the packed steps): deterministic,
        # and within the reference bound of the CPU MoE (only the combine's
        # association differs from one GPU)
        epd = ExpertParallelMoe(shard, E, K, rank=rank, world=world, exchange="device", grouped=grouped)
        g1, g2 = epd.forward(x, di, dw), epd.forward(x, di, dw)
        torch.cuda.synchronize()
        ok = ok and _bits_equal(g1, g2)
        host = [(mats["gate"][e].cpu().numpy(), mats["up"][e].cpu().numpy(), mats["down"][e].cpu().numpy())
                for e in range(E)]
        xh = x.cpu().numpy()
        for t in range(min(T, 6)):
            sel = list(zip(ids[t].tolist(), ws[t].tolist()))
            cpu = O.selected_moe_q4(host, sel, xh[t], H, I, OUT).astype(np.float64)
            bound = moe_bound(q4_matrices(host, H, I, OUT), sel, xh[t], H, I, OUT)
            ok = ok and bool(np.all(np.abs(g1[t].cpu().numpy().astype(np.float64) - cpu) <= bound))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, None))
    except Exception as exc:
        q.put((rank, False, repr(exc)))


@pytest.mark.parametrize("grouped", ["auto", "on"])
def test_ep_two_ranks_bit_identical_to_single_gpu(grouped):
    """Two NCCL ranks; with grouped="on" every rank runs the tensor-core pair
    kernel and the host-plan result must equal one GPU's grouped result bit
    for bit (grouped rows depend only on (expert, token))."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    import torch.distributed as dist
    from datetime import timedelta
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    # rendezvous store on a port the OS assigns, held here until the ranks end
    # (choosing a free port and closing it left a window another bind took)
    store = dist.TCPStore("127.0.0.1", 0, is_master=True, wait_for_workers=False, timeout=timedelta(seconds=60))
    port = store.port
    T, K = (40, 8) if grouped == "on" else (6, 4)
    procs = [ctx.Process(target=_ep_rank, args=(r, 2, port, q, grouped, T, K)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert ok, f"rank {rank}: EP output differs from the single-GPU fused path"


# ------------------------------------------- device-side expert parallelism
def test_ep_build_pairs_matches_host_plan(cuda_device):
    import torch
    from objeta_b200.ep import DispatchPlan, ep_build_pairs
    G, T, K, E = 4, 9, 4, 32
    rng = np.random.default_rng(12)
    ids_all = np.stack([np.stack([rng.choice(E, K, replace=False) for _ in range(T)]) for _ in range(G)])
    d = torch.from_numpy(ids_all.astype(np.int32)).cuda()
    for rank in range(G):
        pe, pt, po, cnt = ep_build_pairs(d, rank, E)
        torch.cuda.synchronize()
        n = int(cnt.item())
        got = sorted(zip(pe[:n].tolist(), pt[:n].tolist(), po[:n].tolist()))
        epr = E // G
        want = sorted((int(ids_all[s, t, j]) - rank * epr, s * T + t, (s * T + t) * K + j)
                      for s in range(G) for t in range(T) for j in range(K) if ids_all[s, t, j] // epr == rank)
        assert got == want
        assert np.all(np.diff(pe[:n].cpu().numpy()) >= 0)          # grouped by expert
        assert n == DispatchPlan.build(ids_all, rank, G, E).num_pairs


def test_ep_device_exchange_emulated_ranks(cuda_device):
    """Two ranks emulated on one GPU: each rank's shard runs its device-built
    pairs with a device count, its partials are exchanged by tensor slicing
    (standing in for the all-to-all), and the owner's ordered sum is checked
    against the one-GPU result (within the MoE bound; the combine's
    association differs) and for run-to-run determinism."""
    import torch
    from objeta_b200.ep import ep_build_pairs, ep_partial_combine, ep_sum_partials, moe_pairs
    from objeta_b200.moe import MoeLayer
    G, E, H, I, OUT, K, T = 2, 16, 1024, 512, 1024, 4, 5
    full, mats = _q4_layer(O.Q4_0, E, H, I, OUT, seed=71)
    epr = E // G
    shards = [MoeLayer(O.Q4_0, H, I, OUT, mats["gate"][r * epr:(r + 1) * epr], mats["up"][r * epr:(r + 1) * epr],
                       mats["down"][r * epr:(r + 1) * epr]) for r in range(G)]
    routes = [_routes(T, E, K, seed=80 + r) for r in range(G)]
    ids_all = torch.from_numpy(np.stack([r[0] for r in routes])).cuda()
    w_all = torch.from_numpy(np.stack([r[1] for r in routes])).cuda()
    xs = [torch.randn(T, H, device="cuda") for _ in range(G)]
    x_all = torch.cat(xs)

    def run():
        parts = []
        for r in range(G):
            pe, pt, po, cnt = ep_build_pairs(ids_all, r, E)
            v = torch.zeros(G * T * K, OUT, device="cuda")
            moe_pairs(shards[r], pe, pt, x_all, v, pair_out=po, d_count=cnt)
            parts.append(ep_partial_combine(ids_all, w_all, v, r, E, OUT))
        outs = []
        for s in range(G):  # all-to-all: rank s receives parts[r][s] from every r
            recv = torch.stack([parts[r][s] for r in range(G)])
            outs.append(ep_sum_partials(recv))
        torch.cuda.synchronize()
        return outs

    a, b = run(), run()
    host = [(mats["gate"][e].cpu().numpy(), mats["up"][e].cpu().numpy(), mats["down"][e].cpu().numpy())
            for e in range(E)]
    for s in range(G):
        assert _bits_equal(a[s], b[s])
        ref = _fused_per_token(full, xs[s], torch.from_numpy(routes[s][0]).cuda(),
                               torch.from_numpy(routes[s][1]).cuda()).cpu().numpy()
        xh = xs[s].cpu().numpy()
        for t in range(T):
            sel = list(zip(routes[s][0][t].tolist(), routes[s][1][t].tolist()))
            bound = moe_bound(q4_matrices(host, H, I, OUT), sel, xh[t], H, I, OUT)
            err = np.abs(a[s][t].cpu().numpy().astype(np.float64) - ref[t].astype(np.float64))
            assert np.all(err <= 2 * bound), f"rank {s} token {t}: max err {err.max()}"


@pytest.mark.parametrize("G,T,K,tc", [(3, 5, 4, False), (2, 40, 8, True), (4, 1, 8, False)])
def test_ep_packed_exchange_emulated_ranks(cuda_device, G, T, K, tc):
    """The one-all-gather exchange (objb_ep_pack_device, then the pair builder
    and partial combine reading the packed buffers) emulated on one GPU: the
    concatenated packed buffers stand in for the all-gather.  Every rank's
    partials equal, bit for bit, those of the three-all-gather layout."""
    import torch
    from objeta_b200.ep import (ep_build_pairs, ep_build_pairs_packed, ep_pack, ep_packed_rows, ep_partial_combine,
                                ep_partial_combine_packed, moe_pairs, moe_pairs_tc)
    from objeta_b200.moe import MoeLayer
    from objeta_b200.quant import device_error_take
    E, H, I, OUT = 8 * G, 1024, 512, 768
    _, mats = _q4_layer(O.Q4_0, E, H, I, OUT, seed=91 + G)
    epr = E // G
    shards = [MoeLayer(O.Q4_0, H, I, OUT, mats["gate"][r * epr:(r + 1) * epr], mats["up"][r * epr:(r + 1) * epr],
                       mats["down"][r * epr:(r + 1) * epr]) for r in range(G)]
    routes = [_routes(T, E, K, seed=300 + r) for r in range(G)]
    ids = [torch.from_numpy(r[0].astype(np.int32)).cuda() for r in routes]
    ws = [torch.from_numpy(r[1]).cuda() for r in routes]
    xs = [torch.randn(T, H, device="cuda") for _ in range(G)]
    rows = ep_packed_rows(T, K, H)
    assert rows == T + -(-2 * T * K // H)
    sends = [ep_pack(xs[r], ids[r], ws[r], torch.full((rows, H), float("nan"), device="cuda")) for r in range(G)]
    recv = torch.cat(sends)
    ids_all, w_all, x_all = torch.stack(ids), torch.stack(ws), torch.cat(xs)
    pairs = moe_pairs_tc if tc else moe_pairs
    device_error_take(cuda_device)
    for r in range(G):
        pe, pt, po, cnt = ep_build_pairs_packed(recv, G, T, K, r, E)
        v = torch.zeros(G * T * K, OUT, device="cuda")
        pairs(shards[r], pe, pt, recv, v, pair_out=po, d_count=cnt)
        got = ep_partial_combine_packed(recv, v, G, T, K, r, E, OUT)
        pe0, pt0, po0, cnt0 = ep_build_pairs(ids_all, r, E)
        v0 = torch.zeros(G * T * K, OUT, device="cuda")
        pairs(shards[r], pe0, pt0, x_all, v0, pair_out=po0, d_count=cnt0)
        want = ep_partial_combine(ids_all, w_all, v0, r, E, OUT)
        torch.cuda.synchronize()
        assert int(cnt.item()) == int(cnt0.item())
        n = int(cnt.item())
        rows_tok = pt[:n].cpu().numpy()
        assert np.all(rows_tok % rows < T)                            # token rows only, never the packed ids
        assert sorted(zip(pe[:n].tolist(), po[:n].tolist())) == sorted(zip(pe0[:n].tolist(), po0[:n].tolist()))
        assert _bits_equal(got, want), f"rank {r}"
    assert device_error_take(cuda_device) == 0
