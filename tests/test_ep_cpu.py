"""Expert-parallel MoE host logic on CPU: the dispatch plan, and the whole
exchange over world_size-2 gloo ranks with the CPU MoE (the oracle) as the
per-pair compute.  The CUDA compute of the same path is covered by the GPU
tests; here the plan and the two all-to-alls must deliver every pair output
to its token owner in slot order, so that the combined result is bit-identical
to the single-rank result and to the reference CPU MoE (moe.rs:1283-1324)."""
import os

import numpy as np
import pytest

from oracle import oracle as O
from objeta_b200.ep import DispatchPlan

H, I, OUT, E, K, T = 64, 96, 64, 8, 3, 5


def _routing(G, T, K, E, seed):
    rng = np.random.default_rng(seed)
    return np.stack([np.stack([rng.choice(E, K, replace=False) for _ in range(T)]) for _ in range(G)])


def _simulate(ids_all, E, value_of):
    """Runs the plan of every rank with numpy standing in for the two
    all-to-alls; value_of(s, t, j, e) is the pair output.  Returns per rank
    the [T, K] array of values each (t, j) slot received."""
    G = ids_all.shape[0]
    plans = [DispatchPlan.build(ids_all, r, G, E) for r in range(G)]
    # x exchange: (source rank, token) units
    x_recv = []
    for r in range(G):
        rows = []
        for s in range(G):
            off = sum(plans[s].send_counts[:r])
            rows += [(s, int(t)) for t in plans[s].send_idx[off:off + plans[s].send_counts[r]]]
        assert len(rows) == sum(plans[r].recv_counts)
        x_recv.append(rows)
    # compute on each rank (in expert order, written to pair_out rows)
    v_send = []
    for r in range(G):
        p = plans[r]
        v = [None] * sum(p.v_send_counts)
        for e, xr, o in zip(p.pair_expert, p.pair_token, p.pair_out):
            s, t = x_recv[r][xr]
            ge = int(e) + r * p.experts_per_rank
            js = [j for j in range(ids_all.shape[2]) if ids_all[s, t, j] == ge]
            assert len(js) == 1
            v[o] = value_of(s, t, js[0], ge)
        assert all(val is not None for val in v)
        v_send.append(v)
    # v exchange back to the owners, then the slot lookup
    got = []
    for s in range(G):
        recv = []
        for r in range(G):
            off = sum(plans[r].v_send_counts[:s])
            recv += v_send[r][off:off + plans[r].v_send_counts[s]]
        assert len(recv) == sum(plans[s].v_recv_counts)
        sr = plans[s].slot_row
        got.append([[recv[sr[t, j]] for j in range(sr.shape[1])] for t in range(sr.shape[0])])
    return plans, got


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_dispatch_plan_delivers_every_slot(G):
    ids_all = _routing(G, 7, 4, 16, seed=G)
    plans, got = _simulate(ids_all, 16, lambda s, t, j, e: (s, t, j, e))
    for s in range(G):
        for t in range(7):
            for j in range(4):
                assert got[s][t][j] == (s, t, j, int(ids_all[s, t, j]))
    for r in range(G):
        p = plans[r]
        # counts agree pairwise across ranks
        for s in range(G):
            assert plans[s].send_counts[r] == p.recv_counts[s]
            assert plans[s].v_recv_counts[r] == p.v_send_counts[s]
        # pairs are grouped by expert, each local
        assert np.all(np.diff(p.pair_expert) >= 0)
        assert p.pair_expert.size == 0 or (p.pair_expert.min() >= 0 and p.pair_expert.max() < 16 // G)
        assert sorted(p.pair_out.tolist()) == list(range(p.num_pairs))


def test_dispatch_plan_single_rank_is_identity_on_tokens():
    ids = _routing(1, 6, 3, 8, seed=3)
    p = DispatchPlan.build(ids, 0, 1, 8)
    assert p.send_idx.tolist() == list(range(6)) and p.recv_counts == [6]
    assert p.num_pairs == 18 and p.v_send_counts == [18]
    # slot_row enumerates (token, slot) in row-major order
    assert p.slot_row.ravel().tolist() == list(range(18))


def test_dispatch_plan_rejects_bad_tables():
    ids = _routing(2, 3, 2, 8, seed=1)
    with pytest.raises(ValueError):
        DispatchPlan.build(ids, 0, 2, 7)          # not divisible
    with pytest.raises(ValueError):
        DispatchPlan.build(ids, 0, 4, 8)          # wrong world
    bad = ids.copy()
    bad[1, 0, 0] = 8
    with pytest.raises(ValueError):
        DispatchPlan.build(bad, 0, 2, 8)


def test_exchange_bytes():
    ids = np.array([[[0, 5]], [[1, 2]]])         # rank0 token -> experts 0 (r0), 5 (r1); rank1 -> 1, 2 (r0)
    p0 = DispatchPlan.build(ids, 0, 2, 8)
    assert p0.send_counts == [1, 1] and p0.recv_counts == [1, 1]
    assert p0.exchange_bytes(10, 20) == {"dispatch": 40, "combine": 2 * 80}


# ------------------------------------------------------------- gloo ranks
def _experts():
    from tests._moe_util import make_q4_experts
    experts, _ = make_q4_experts(E, H, I, OUT, seed=77)
    return experts


def _oracle_compute(experts, plan, x_recv, n_rows, rank):
    import torch
    v = torch.zeros(n_rows, OUT)
    xs = x_recv.numpy()
    for e, xr, o in zip(plan.pair_expert, plan.pair_token, plan.pair_out):
        ge = int(e) + rank * plan.experts_per_rank
        v[int(o)] = torch.from_numpy(O.selected_moe_q4(experts, [(ge, 1.0)], xs[int(xr)], H, I, OUT))
    return v


def _np_combine(v_recv, plan, w):
    import torch
    v = v_recv.numpy()
    wn = w.numpy().astype(np.float32)
    out = np.zeros((plan.slot_row.shape[0], v.shape[1]), np.float32)
    for t in range(out.shape[0]):
        acc = np.zeros(v.shape[1], np.float32)
        for j in range(plan.slot_row.shape[1]):
            acc = (acc + np.float32(wn[t, j]) * v[plan.slot_row[t, j]]).astype(np.float32)
        out[t] = acc
    return torch.from_numpy(out)


def _inputs(rank):
    rng = np.random.default_rng(100 + rank)
    x = rng.standard_normal((T, H)).astype(np.float32)
    ids, ws = [], []
    for _ in range(T):
        i, w = O.router_from_logits(rng.standard_normal(E).astype(np.float32), K, True)
        ids.append(i)
        ws.append(w)
    return x, np.array(ids, np.int32), np.array(ws, np.float32)


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from objeta_b200.ep import ExpertParallelMoe
    try:
        store = dist.TCPStore("127.0.0.1", port, is_master=False, timeout=timedelta(seconds=60))
        dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=timedelta(seconds=60))
        experts = _experts()
        x, ids, ws = _inputs(rank)
        ep = ExpertParallelMoe(None, E, K, rank=rank, world=world, out_dim=OUT,
                               compute=lambda plan, xr, n: _oracle_compute(experts, plan, xr, n, rank),
                               combine=_np_combine)
        out = ep.forward(torch.from_numpy(x), torch.from_numpy(ids), torch.from_numpy(ws))
        q.put((rank, out.numpy(), ep.last_plan.exchange_bytes(H, OUT)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent, which fails the test
        q.put((rank, repr(exc), None))


def _parent_store():
    """A rendezvous store held by the test process on a port the OS assigns
    (no window between choosing a free port and listening on it); the ranks
    connect to it as clients."""
    import torch.distributed as dist
    from datetime import timedelta
    return dist.TCPStore("127.0.0.1", 0, is_master=True, wait_for_workers=False, timeout=timedelta(seconds=60))


def test_two_gloo_ranks_match_single_rank_and_reference():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store = _parent_store()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, store.port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, out, xb = q.get(timeout=240)
        res[r] = (out, xb)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    experts = _experts()
    for r in range(2):
        out, xb = res[r]
        assert not isinstance(out, str), out
        x, ids, ws = _inputs(r)
        for t in range(T):
            ref = O.selected_moe_q4(experts, list(zip(ids[t].tolist(), ws[t].tolist())), x[t], H, I, OUT)
            assert np.array_equal(out[t].view(np.uint32), ref.view(np.uint32)), f"rank {r} token {t}"
        assert xb["dispatch"] > 0 or xb["combine"] >= 0


def test_grouped_path_selection():
    """"auto" takes the tensor-core pairs path from GROUPED_MIN_SLOTS token
    slots on supported layers only; "on" insists on support; the choice
    depends on T * k, not on the rank count."""
    from types import SimpleNamespace
    from objeta_b200 import ep as E

    def layer(fmt=0, H=2048, I=512, flags=0, split=False):
        return SimpleNamespace(fmt=fmt, hidden=H, intermediate=I, out_dim=H, _c=SimpleNamespace(flags=flags),
                               _tensors=[None, None, None, object() if split else None, None, None])

    ok = layer()
    m = E.ExpertParallelMoe(ok, 256, 8)
    assert m._pairs_fn(E.GROUPED_MIN_SLOTS - 1) is E.moe_pairs
    assert m._pairs_fn(E.GROUPED_MIN_SLOTS) is E.moe_pairs_tc
    m2 = E.ExpertParallelMoe(ok, 256, 8, rank=1, world=2)
    assert m2._pairs_fn(E.GROUPED_MIN_SLOTS) is E.moe_pairs_tc
    assert E.ExpertParallelMoe(ok, 256, 8, grouped="off")._pairs_fn(10 ** 6) is E.moe_pairs
    assert E.ExpertParallelMoe(ok, 256, 8, grouped="on")._pairs_fn(1) is E.moe_pairs_tc
    for bad in (layer(fmt=1), layer(I=800), layer(flags=1), layer(fmt=3, split=True)):
        assert not E.grouped_supported(bad)
        assert E.ExpertParallelMoe(bad, 256, 8)._pairs_fn(10 ** 6) is E.moe_pairs
        with pytest.raises(ValueError):
            E.ExpertParallelMoe(bad, 256, 8, grouped="on")
    with pytest.raises(ValueError):
        E.ExpertParallelMoe(ok, 256, 8, grouped="yes")
