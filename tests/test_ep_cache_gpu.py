"""Multi-token MoE over host-resident experts through the expert cache
(objb_moe_execute_pairs / CachedExpertCompute): results bit-identical to the
single-token executor (execute_selected_moe_cuda, whose own tests pin it to
the reference CPU MoE), cache counters per distinct expert with the
reference's get-else-insert admission, and a cache far smaller than the
working set (evictions inside one call must not corrupt the experts that
call is still using)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._moe_util import make_q4_experts

pytestmark = pytest.mark.gpu

H, I, OUT, E, K = 1024, 512, 1024, 16, 4


def _setup(T, seed):
    from objeta_b200.moe import ExpertWeights
    experts, _ = make_q4_experts(E, H, I, OUT, seed=seed)
    ew = [ExpertWeights(g, u, d) for g, u, d in experts]
    rng = np.random.default_rng(seed)
    ids, ws = [], []
    for _ in range(T):
        i, w = O.router_from_logits(rng.standard_normal(E).astype(np.float32), K, True)
        ids.append(i)
        ws.append(w)
    x = rng.standard_normal((T, H)).astype(np.float32)
    return ew, np.array(ids, np.int32), np.array(ws, np.float32), x


def _per_token(ew, ids, ws, x):
    from objeta_b200 import QuantBackend
    from objeta_b200.moe import MoeExecutor
    ex = MoeExecutor(0)
    qb = QuantBackend(0)
    return np.stack([ex.execute_selected_moe_cuda(qb, None, ew, list(zip(ids[t].tolist(), ws[t].tolist())), x[t],
                                                  H, I, OUT, 0, None)[0] for t in range(x.shape[0])])


def _bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("capacity_experts", [E, 2])
def test_cached_ep_matches_single_token_executor(cuda_device, capacity_experts):
    import torch
    from objeta_b200.ep import CachedExpertCompute, ExpertParallelMoe
    from objeta_b200.moe import CudaExpertCache, MoeExecutor
    T = 6
    ew, ids, ws, x = _setup(T, seed=3)
    ref = _per_token(ew, ids, ws, x)
    expert_bytes = ew[0].w_gate.size + ew[0].w_up.size + ew[0].w_down.size
    cache = CudaExpertCache(capacity_experts * expert_bytes, 0)
    comp = CachedExpertCompute(MoeExecutor(0), cache, ew, H, I, OUT)
    ep = ExpertParallelMoe(None, E, K, out_dim=OUT, compute=comp)
    dx, di, dw = (torch.from_numpy(a).cuda() for a in (x, ids, ws))
    for step in range(2):
        out = ep.forward(dx, di, dw)
        torch.cuda.synchronize()
        assert _bits(out.cpu().numpy(), ref), f"step {step}"
        tel = comp.last_telemetry
        distinct = len(np.unique(ids))
        assert tel.selected_expert_count == distinct
        assert tel.logical_expert_bytes_requested == distinct * expert_bytes
        assert tel.logical_expert_bytes_requested == tel.actual_expert_bytes_loaded + tel.resident_cache_bytes_reused
        if capacity_experts == E:
            # first step loads every distinct expert, the second reuses them all
            assert (tel.resident_cache_bytes_reused == 0) if step == 0 else (tel.actual_expert_bytes_loaded == 0)
    st = cache.stats()
    if capacity_experts == E:
        assert st["miss_count"] == 3 * len(np.unique(ids)) and st["hit_count"] == 3 * len(np.unique(ids))
    else:
        assert st["eviction_count"] > 0 and st["resident_bytes"] <= st["capacity_bytes"]


def test_execute_pairs_validates_like_the_executor(cuda_device):
    import torch
    from objeta_b200._lib import CudaError
    from objeta_b200.moe import MoeExecutor
    ew, ids, ws, x = _setup(2, seed=5)
    ex = MoeExecutor(0)
    table = ex.expert_table(ew)
    dx = torch.from_numpy(x).cuda()
    v = torch.empty(8, OUT, device="cuda")
    with pytest.raises(CudaError) as e:
        ex.execute_pairs(table, [E], [0], dx, v, H, I, OUT, 0)
    assert "out of bounds" in e.value.source_message
    with pytest.raises(CudaError):
        ex.execute_pairs(table, [0], [2], dx, v, H, I, OUT, 0)       # token 2 of 2
    with pytest.raises(CudaError):
        ex.execute_pairs(table, [0], [0], dx, v, H, I, OUT, 0, pair_out=[8])


@pytest.mark.parametrize("capacity_experts", [E, 4])
def test_cached_pairs_chunked_match_oracle_and_model(cuda_device, capacity_experts):
    """256 tokens through the cache: the executor resolves the distinct
    experts in chunks of half the cache's capacity, overlapping a chunk's
    uploads with the previous chunk's kernels (16 experts: two chunks of ~512
    pairs on the tensor cores; 4 experts: eight chunks on the CUDA-core
    pairs, evicting the whole time).  Tokens match the oracle MoE within the
    reference bound, and the cache's counters and LRU order equal the
    restated cache fed the same lookups (distinct experts in first-appearance
    order, gate / up / down each)."""
    import torch
    from oracle.cache_model import CacheModel
    from objeta_b200.ep import CachedExpertCompute, ExpertParallelMoe
    from objeta_b200.moe import CudaExpertCache, MoeExecutor
    from tests._moe_util import moe_bound, q4_matrices
    T = 256
    ew, ids, ws, x = _setup(T, seed=11)
    expert_bytes = ew[0].w_gate.size + ew[0].w_up.size + ew[0].w_down.size
    cap = capacity_experts * expert_bytes
    cache = CudaExpertCache(cap, 0)
    comp = CachedExpertCompute(MoeExecutor(0), cache, ew, H, I, OUT)
    ep = ExpertParallelMoe(None, E, K, out_dim=OUT, compute=comp)
    dx, di, dw = (torch.from_numpy(a).cuda() for a in (x, ids, ws))
    model = CacheModel(cap)
    for step in range(2):
        out = ep.forward(dx, di, dw)
        torch.cuda.synchronize()
        seen = []
        for e in ep.last_plan.pair_expert.tolist():
            if e not in seen:
                seen.append(e)
        for e in seen:
            for kind, n in ((0, ew[e].w_gate.size), (1, ew[e].w_up.size), (2, ew[e].w_down.size)):
                model.get_or_insert((0, e, kind), n)
        s = cache.stats()
        for name, v in model.counters().items():
            assert s[name] == v, (step, name, s[name], v)
        assert [(q.layer_id, q.expert_id, int(q.tensor_kind)) for q in cache.lru_keys()] == model.order
    got = out.cpu().numpy()
    host = [(w.w_gate, w.w_up, w.w_down) for w in ew]
    for t in range(0, T, 37):
        sel = list(zip(ids[t].tolist(), ws[t].tolist()))
        ref = O.selected_moe_q4(host, sel, x[t], H, I, OUT)
        bound = moe_bound(q4_matrices(host, H, I, OUT), sel, x[t], H, I, OUT)
        err = np.abs(got[t].astype(np.float64) - ref.astype(np.float64))
        assert np.all(err <= bound), f"token {t}: worst err/bound {np.max(err / bound):.3f}"
    assert cache.stats()["overflow_allocations"] == 0
