"""GPU parity of the selected-expert MoE, the expert cache and the router
against the CPU oracle (reference arithmetic and counters).  Run with -m gpu."""
import random

import numpy as np
import pytest

from oracle import oracle as O
from oracle.cache_model import CacheModel
from tests._moe_util import (fp4_matrices, make_fp4_experts, make_q4_experts, moe_bound, q4_matrices)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ex(cuda_device):
    from objeta_b200.moe import MoeExecutor
    e = MoeExecutor(cuda_device)
    e.compile()
    return e


@pytest.fixture(scope="module")
def qb(cuda_device):
    from objeta_b200 import QuantBackend
    return QuantBackend(cuda_device)


def _w(experts):
    from objeta_b200.moe import ExpertWeights
    return [ExpertWeights(*e) for e in experts]


def _w4(experts):
    from objeta_b200.moe import DeepSeekFp4ExpertWeights
    return [DeepSeekFp4ExpertWeights(*e) for e in experts]


def _check(out, ref, bound, what):
    err = np.abs(out.astype(np.float64) - ref.astype(np.float64))
    bad = np.nonzero(err > bound)[0]
    assert bad.size == 0, f"{what}: row {bad[0]} err {err[bad[0]]:.3e} > bound {bound[bad[0]]:.3e}"


# ------------------------------------------------- moe.rs:1755-1889 sweeps
@pytest.mark.parametrize("seed", [0, 1, 2, 3, 4, 123])
@pytest.mark.parametrize("hidden,inter,out_dim,nsel", [(256, 512, 256, 1), (256, 512, 256, 2),
                                                       (1024, 2048, 1024, 4)])
def test_moe_correctness_sweeps(ex, qb, seed, hidden, inter, out_dim, nsel):
    experts, dense = make_q4_experts(8, hidden, inter, out_dim, seed)
    x = O.seeded_f32s(hidden, seed ^ 0xDEADBEEF)
    ws = [0.4, 0.3, 0.2, 0.1]
    sel = [((seed + i) % 8, ws[i % 4]) for i in range(nsel)]
    ref = O.selected_moe_q4(experts, sel, x, hidden, inter, out_dim)
    out, tel = ex.execute_selected_moe_cuda(qb, None, _w(experts), sel, x, hidden, inter, out_dim, 0, None)
    d = O.compare_outputs(ref, out)
    assert d["cosine_similarity"] >= 0.9999 and d["relative_l2_error"] <= 1e-4 and d["max_abs_error"] <= 1e-2
    _check(out, ref, moe_bound(q4_matrices(experts, hidden, inter, out_dim), sel, x, hidden, inter, out_dim),
           f"seed {seed}")
    # quant vs fp32 reference (moe.rs:1846-1858)
    ref32 = np.zeros(out_dim, np.float32)
    for e, w in sel:
        g = O.dense_gemv(dense[e][0], x, inter, hidden)
        u = O.dense_gemv(dense[e][1], x, inter, hidden)
        a = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)
        ref32 += np.float32(w) * O.dense_gemv(dense[e][2], a, out_dim, inter)
    assert O.compare_outputs(ref32, out)["cosine_similarity"] >= 0.98
    assert tel.selected_expert_count == nsel
    assert tel.dequantized_scratch_bytes == 0
    assert tel.resident_cache_bytes_reused == 0
    assert tel.logical_expert_bytes_requested == tel.actual_expert_bytes_loaded


# ---------------------------------------------- moe.rs:1891-2168 cache tests
H, I, OD = 256, 512, 256


@pytest.fixture(scope="module")
def four_experts():
    experts, _ = make_q4_experts(4, H, I, OD, 42)
    return experts


def _run(ex, qb, experts, sel, cache):
    x = O.seeded_f32s(H, 42 ^ 0xDEADBEEF)
    out, tel = ex.execute_selected_moe_cuda(qb, None, _w(experts), sel, x, H, I, OD, 0, cache)
    ref = O.selected_moe_q4(experts, sel, x, H, I, OD)
    _check(out, ref, moe_bound(q4_matrices(experts, H, I, OD), sel, x, H, I, OD), "cache run")
    assert tel.logical_expert_bytes_requested == tel.actual_expert_bytes_loaded + tel.resident_cache_bytes_reused
    return tel


def test_cuda_expert_cache_behavior(ex, qb, four_experts, cuda_device):
    from objeta_b200.moe import CudaExpertCache
    experts = four_experts
    eb = sum(t.size for t in experts[0])
    # 1. no cache
    tel = _run(ex, qb, experts, [(0, .5), (1, .5)], None)
    assert tel.resident_cache_bytes_reused == 0 and tel.resident_cache_capacity_bytes == 0
    assert tel.resident_cache_resident_bytes == 0
    # 2. repeated experts hit
    c = CudaExpertCache(1000 * 1024, cuda_device)
    t1 = _run(ex, qb, experts, [(0, .5), (1, .5)], c)
    assert (t1.resident_cache_bytes_reused, t1.resident_cache_hit_count, t1.resident_cache_miss_count,
            t1.resident_cache_eviction_count) == (0, 0, 6, 0)
    t2 = _run(ex, qb, experts, [(0, .5), (1, .5)], c)
    assert t2.resident_cache_bytes_reused == t2.logical_expert_bytes_requested
    assert t2.actual_expert_bytes_loaded == 0
    assert (t2.resident_cache_hit_count, t2.resident_cache_miss_count, t2.resident_cache_eviction_count) == (6, 6, 0)
    # 3. capacity fits all
    c = CudaExpertCache(4 * eb, cuda_device)
    t = _run(ex, qb, experts, [(0, .5), (1, .5), (2, .5), (3, .5)], c)
    assert t.resident_cache_eviction_count == 0 and t.resident_cache_resident_bytes == 4 * eb
    # 4. one expert of capacity: eviction
    c = CudaExpertCache(eb, cuda_device)
    t = _run(ex, qb, experts, [(0, 1.0)], c)
    assert t.resident_cache_eviction_count == 0 and t.resident_cache_resident_bytes == eb
    t = _run(ex, qb, experts, [(1, 1.0)], c)
    assert t.resident_cache_eviction_count > 0 and t.resident_cache_resident_bytes == eb
    t = _run(ex, qb, experts, [(0, 1.0)], c)
    assert t.actual_expert_bytes_loaded == eb and t.resident_cache_bytes_reused == 0
    # 5. LRU touch order
    c = CudaExpertCache(2 * eb, cuda_device)
    for e in (0, 1, 0, 2):
        _run(ex, qb, experts, [(e, 1.0)], c)
    assert _run(ex, qb, experts, [(0, 1.0)], c).resident_cache_bytes_reused == eb
    t = _run(ex, qb, experts, [(1, 1.0)], c)
    assert t.resident_cache_bytes_reused == 0 and t.actual_expert_bytes_loaded == eb


def test_oversized_tensor_bypass(ex, qb, four_experts, cuda_device):
    from objeta_b200.moe import CudaExpertCache
    e0 = four_experts[0]
    c = CudaExpertCache(e0[0].size - 1, cuda_device)
    t = _run(ex, qb, [e0], [(0, 1.0)], c)
    assert (t.resident_cache_insert_attempt_count, t.resident_cache_insert_accept_count,
            t.resident_cache_insert_bypass_count, t.resident_cache_oversized_tensor_bypass_count,
            t.resident_cache_oversized_expert_bypass_count, t.resident_cache_resident_bytes) == (3, 0, 3, 3, 0, 0)
    assert t.actual_expert_bytes_loaded == t.logical_expert_bytes_requested and t.resident_cache_bytes_reused == 0


def test_oversized_expert_bypass(ex, qb, four_experts, cuda_device):
    from objeta_b200.moe import CudaExpertCache
    e0 = four_experts[0]
    eb = sum(t.size for t in e0)
    c = CudaExpertCache(eb - 100, cuda_device)
    c.bypass_oversized_experts = True
    t = _run(ex, qb, [e0], [(0, 1.0)], c)
    assert (t.resident_cache_insert_attempt_count, t.resident_cache_insert_accept_count,
            t.resident_cache_insert_bypass_count, t.resident_cache_oversized_tensor_bypass_count,
            t.resident_cache_oversized_expert_bypass_count, t.resident_cache_self_eviction_risk_count,
            t.resident_cache_resident_bytes) == (3, 0, 3, 0, 1, 0, 0)
    c = CudaExpertCache(eb - 100, cuda_device)
    t = _run(ex, qb, [e0], [(0, 1.0)], c)
    assert t.resident_cache_self_eviction_risk_count == 1 and t.resident_cache_oversized_expert_bypass_count == 0
    assert t.resident_cache_insert_accept_count > 0


def test_self_eviction_within_one_call_is_safe(ex, qb, four_experts, cuda_device):
    """Capacity below one expert: inserting later tensors evicts earlier ones
    of the same call; the evicted slots must not be reused before the kernels
    have read them (the output must still match)."""
    from objeta_b200.moe import CudaExpertCache
    eb = sum(t.size for t in four_experts[0])
    c = CudaExpertCache(four_experts[0][0].size + 64, cuda_device)
    for sel in ([(0, .6), (1, .4)], [(2, 1.0), (0, .5), (3, .25)], [(1, .3), (1, .7)]):
        _run(ex, qb, four_experts, sel, c)
    assert c.stats()["resident_bytes"] <= eb


# ------------------------------------------- moe.rs:2333-2559 native FP4
def test_native_fp4_moe_correctness(ex, qb):
    h, i, o = 256, 512, 256
    experts = make_fp4_experts(4, h, i, o, 42)
    x = O.seeded_f32s(h, 42 ^ 0xDEADBEEF)
    sel = [(0, 0.4), (2, 0.6)]
    ref = O.selected_moe_native_fp4(experts, sel, x, h, i, o)
    out, tel = ex.execute_selected_moe_native_fp4_cuda(qb, None, _w4(experts), sel, x, h, i, o, 0, None)
    assert O.compare_outputs(ref, out)["cosine_similarity"] >= 0.9999
    _check(out, ref, moe_bound(fp4_matrices(experts, h, i, o), sel, x, h, i, o), "native fp4")
    assert tel.selected_expert_count == 2 and tel.dequantized_scratch_bytes == 0
    assert tel.resident_cache_bytes_reused == 0
    assert tel.logical_expert_bytes_requested == tel.actual_expert_bytes_loaded
    assert tel.scale_bytes_loaded == 2 * (2 * i * h // 32 + o * i // 32)


def test_native_fp4_expert_cache(ex, qb, cuda_device):
    from objeta_b200.moe import CudaExpertCache
    h, i, o = 256, 512, 256
    experts = make_fp4_experts(4, h, i, o, 42)
    x = O.seeded_f32s(h, 42 ^ 0xDEADBEEF)
    eb = sum(t.size for t in experts[0])
    assert eb == 208896
    c = CudaExpertCache(2 * eb, cuda_device)
    for e, loaded, reused, resident in [(0, eb, 0, eb), (0, 0, eb, eb), (1, eb, 0, 2 * eb), (2, eb, 0, 2 * eb),
                                        (0, eb, 0, None)]:
        out, t = ex.execute_selected_moe_native_fp4_cuda(qb, None, _w4(experts), [(e, 1.0)], x, h, i, o, 0, c)
        assert t.actual_expert_bytes_loaded == loaded and t.resident_cache_bytes_reused == reused
        if resident is not None:
            assert c.stats()["resident_bytes"] == resident
        ref = O.selected_moe_native_fp4(experts, [(e, 1.0)], x, h, i, o)
        _check(out, ref, moe_bound(fp4_matrices(experts, h, i, o), [(e, 1.0)], x, h, i, o), "fp4 cache")


# ----------------------------------------- product cache == reference model
def test_cache_matches_model_random_ops(cuda_device):
    from objeta_b200 import QuantFormat
    from objeta_b200.moe import CudaExpertCache, ExpertCacheKey, ExpertTensorKind
    rng = random.Random(7)
    cap = 10_000
    c = CudaExpertCache(cap, cuda_device)
    m = CacheModel(cap)
    keys = [(layer, e, kind) for layer in range(2) for e in range(6) for kind in (0, 1, 2)]
    sizes = {k: rng.choice([512, 1024, 2048, 3000, 12_000]) for k in keys}

    def K(k):
        return ExpertCacheKey(k[0], k[1], ExpertTensorKind(k[2]), QuantFormat.Q4_0)

    for step in range(600):
        op = rng.random()
        k = rng.choice(keys)
        if op < 0.45:
            p = c.get(K(k))
            assert (p is not None) == m.get(k), step
        elif op < 0.75:
            data = np.full(sizes[k], step % 251, np.uint8)
            p = c.insert(K(k), data)
            m.insert(k, sizes[k])
            assert p is not None
        elif op < 0.82:
            c.touch(K(k))
            m.touch(k)
        elif op < 0.88:
            got = c.evict_lru()
            want = m.evict_lru()
            assert (got is None) == (want is None), step
            if got is not None:
                assert (got.layer_id, got.expert_id, int(got.tensor_kind)) == want
        elif op < 0.92:
            c.pin(K(k))
            m.pin(k)
        elif op < 0.95:
            data = np.full(sizes[k] // 4, 3, np.uint8)
            c.insert_pinned(K(k), data)
            m.insert_pinned(k, sizes[k] // 4)
        elif op < 0.97:
            c.release()
        elif op < 0.985:
            c.reset_counters()
            m.reset_counters()
        else:
            c.clear()
            m.clear()
        s = c.stats()
        for name, v in m.counters().items():
            assert s[name] == v, (step, name, s[name], v)
        assert [(q.layer_id, q.expert_id, int(q.tensor_kind)) for q in c.lru_keys()] == m.order, step


@pytest.mark.parametrize("lazy", [True, False])
def test_get_or_insert_matches_model(cuda_device, lazy):
    """CudaExpertCache.get_or_insert through objb_expert_cache_get_or_load
    (lazy load_fn) and objb_expert_cache_get_or_insert (bytes at hand) on the
    reference's cache sequences (moe.rs:1891-2226, tensor by tensor as the
    executor looks them up, moe.rs:508-518), then random operations: hit
    flags, every counter and the LRU order after each step equal the
    restated cache (oracle/cache_model.py); the loader runs on misses only."""
    from objeta_b200 import QuantFormat
    from objeta_b200.moe import CudaExpertCache, ExpertCacheKey, ExpertTensorKind
    gate, down = 512 * 8 * 18, 256 * 16 * 18
    expert = 2 * gate + down
    sizes = {0: gate, 1: gate, 2: down}

    def K(k):
        return ExpertCacheKey(k[0], k[1], ExpertTensorKind(k[2]), QuantFormat.Q4_0)

    def step(c, m, k, nbytes, where):
        loads = []
        data = np.full(nbytes, (k[1] * 3 + k[2]) % 251, np.uint8)

        def load():
            loads.append(k)
            return data
        p, hit = c.get_or_insert(K(k), load if lazy else data)
        want_hit, _ = m.get_or_insert(k, nbytes)
        assert hit == want_hit and p is not None, where
        if lazy:
            assert len(loads) == (0 if hit else 1), where
        s = c.stats()
        for name, v in m.counters().items():
            assert s[name] == v, (where, name, s[name], v)
        assert [(q.layer_id, q.expert_id, int(q.tensor_kind)) for q in c.lru_keys()] == m.order, where

    sequences = [
        (1000 * 1024, [0, 1, 0, 1]),       # moe.rs:1950-2000: 6 misses then 6 hits
        (4 * expert, [0, 1, 2, 3]),        # moe.rs:2002-2025: no eviction
        (expert, [0, 1, 0]),               # moe.rs:2027-2082: eviction, reload
        (2 * expert, [0, 1, 0, 2, 0, 1]),  # moe.rs:2084-2166: LRU touch order
        (gate - 1, [0, 1]),                # moe.rs:2170-2226: oversized tensors bypass
    ]
    for cap, experts in sequences:
        c, m = CudaExpertCache(cap, cuda_device), CacheModel(cap)
        for i, e in enumerate(experts):
            for kind in (0, 1, 2):
                step(c, m, (0, e, kind), sizes[kind], (cap, i, kind))
            c.release()
    rng = random.Random(11)
    cap = 10_000
    c, m = CudaExpertCache(cap, cuda_device), CacheModel(cap)
    keys = [(layer, e, kind) for layer in range(2) for e in range(5) for kind in (0, 1, 2)]
    ksize = {k: rng.choice([512, 1024, 2048, 3000, 12_000]) for k in keys}
    for i in range(300):
        k = rng.choice(keys)
        r = rng.random()
        if r < 0.7:
            step(c, m, k, ksize[k], ("random", i))
        elif r < 0.8:
            c.touch(K(k))
            m.touch(k)
        elif r < 0.9:
            c.release()
        elif r < 0.95:
            c.pin(K(k))
            m.pin(k)
        else:
            c.reset_counters()
            m.reset_counters()


def test_get_or_insert_loader_error_inserts_nothing(cuda_device):
    from objeta_b200 import QuantFormat
    from objeta_b200.moe import CudaExpertCache, ExpertCacheKey, ExpertTensorKind
    c = CudaExpertCache(10_000, cuda_device)
    k = ExpertCacheKey(0, 1, ExpertTensorKind.Gate, QuantFormat.Q4_0)

    def bad():
        raise IOError("expert file missing")
    with pytest.raises(IOError):
        c.get_or_insert(k, bad)
    s = c.stats()
    assert (s["miss_count"], s["cache_insert_attempt_count"], s["resident_bytes"]) == (1, 0, 0)
    assert not c.contains(k)


def test_cache_data_roundtrip(cuda_device):
    """Resident bytes equal the uploaded host bytes, across slot reuse."""
    import ctypes
    import torch
    from objeta_b200 import QuantFormat
    from objeta_b200.moe import CudaExpertCache, ExpertCacheKey, ExpertTensorKind
    c = CudaExpertCache(4096 * 3, cuda_device)
    rng = np.random.default_rng(3)
    for r in range(12):
        k = ExpertCacheKey(0, r, ExpertTensorKind.Gate, QuantFormat.Q4_0)
        data = rng.integers(0, 256, 4096, dtype=np.uint8)
        p = c.insert(k, data)
        torch.cuda.synchronize()
        back = np.empty(4096, np.uint8)
        from cuda.bindings import runtime as rt
        err, = rt.cudaMemcpy(back.ctypes.data, p, 4096, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
        assert int(err) == 0
        assert np.array_equal(back, data), r
        c.release()
    assert c.stats()["eviction_count"] >= 9


# ------------------------------------------------------------- router
def test_router_matches_reference_selection(cuda_device):
    import torch
    from objeta_b200.moe import router_topk
    rng = np.random.default_rng(11)
    for n, k in [(8, 2), (256, 8), (4, 2), (64, 6)]:
        for t in range(40):
            logits = rng.standard_normal(n).astype(np.float32)
            if t % 7 == 0:
                logits[rng.integers(0, n, 3)] = logits[0]  # ties
            for renorm in (False, True):
                ids, w = router_topk(torch.from_numpy(logits).cuda(), k, renorm)
                rid, rw = O.router_from_logits(logits, k, renorm)
                assert ids.cpu().numpy().tolist() == rid.tolist()
                np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=0)


def test_router_reference_kat(cuda_device):
    import torch
    from objeta_b200.moe import router_topk
    # deepseek_single_layer_moe.rs:3414-3445: logits 0, 2, 0, 4 -> ids [3, 1]
    ids, w = router_topk(torch.tensor([0.0, 2.0, 0.0, 4.0], device="cuda"), 2)
    assert ids.cpu().tolist() == [3, 1] and float(w[0]) > float(w[1])


# ------------------------------------------------ device-resident layers
def _device_q4_layer(fmt, num_experts, hidden, inter, out_dim, seed):
    import torch
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    qb = QuantBackend(torch.cuda.current_device())
    g = torch.Generator(device="cuda").manual_seed(seed)
    mats = {"gate": [], "up": [], "down": []}
    for e in range(num_experts):
        for name, (r, c) in (("gate", (inter, hidden)), ("up", (inter, hidden)), ("down", (out_dim, inter))):
            m = torch.randn(r, c, device="cuda", generator=g) * 0.02
            mats[name].append(qb.quantize_matrix_device(QuantFormat(fmt), m, QGemvShape.new(QuantFormat(fmt), r, c)))
    return mats


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q5_0, O.IQ3_0])
def test_device_layer_matches_reference(cuda_device, fmt):
    """MoeLayer (objb_moe_forward_device): router + fused MoE, checked against
    the CPU MoE (gemv_cpu per expert, moe.rs:1283-1324)."""
    import torch
    from objeta_b200.moe import MoeLayer
    hidden, inter, out_dim, E, k = 1024, 1536, 1024, 16, 4
    mats = _device_q4_layer(fmt, E, hidden, inter, out_dim, seed=fmt + 5)
    layer = MoeLayer(fmt, hidden, inter, out_dim, mats["gate"], mats["up"], mats["down"])
    rng = np.random.default_rng(fmt)
    x = rng.standard_normal(hidden).astype(np.float32)
    logits = rng.standard_normal(E).astype(np.float32)
    out, ids, w = layer.forward(torch.from_numpy(logits).cuda(), k, torch.from_numpy(x).cuda(), renormalize=True)
    torch.cuda.synchronize()
    rid, rw = O.router_from_logits(logits, k, True)
    assert ids.cpu().numpy().tolist() == rid.tolist()
    host = [(mats["gate"][e].cpu().numpy(), mats["up"][e].cpu().numpy(), mats["down"][e].cpu().numpy())
            for e in range(E)]
    sel = list(zip(rid.tolist(), rw.tolist()))
    ref = np.zeros(out_dim, np.float32)
    for e, wt in sel:  # selected_moe_cpu with this format's gemv_cpu
        gg = O.gemv(fmt, host[e][0], x, inter, hidden)
        uu = O.gemv(fmt, host[e][1], x, inter, hidden)
        a = np.array([np.float32(v / (np.float32(1) + np.exp(np.float32(-v)))) * np.float32(q)
                      for v, q in zip(gg, uu)], np.float32)
        ref += np.float32(wt) * O.gemv(fmt, host[e][2], a, out_dim, inter)
    _check(out.cpu().numpy(), ref, moe_bound(q4_matrices(host, hidden, inter, out_dim, fmt), sel, x, hidden, inter,
                                             out_dim), f"layer fmt {fmt}")


def test_device_layer_fp4_baseline_shape(cuda_device):
    """BASELINE configs[3] routed part: hidden 4096, 256 experts, intermediate
    2048, top-8, FP4 codes uniform, power-of-two scales 2^-8..2^-4."""
    import torch
    from objeta_b200.moe import MoeLayer
    hidden, inter, E, k = 4096, 2048, 256, 8
    g = torch.Generator(device="cuda").manual_seed(99)
    lists = {n: [] for n in ("gw", "gs", "uw", "us", "dw", "ds")}
    for e in range(E):
        for wn, sn, r, c in (("gw", "gs", inter, hidden), ("uw", "us", inter, hidden), ("dw", "ds", hidden, inter)):
            lists[wn].append(torch.randint(0, 256, (r * c // 2,), device="cuda", dtype=torch.uint8, generator=g))
            lists[sn].append(torch.randint(119, 124, (r * c // 32,), device="cuda", dtype=torch.uint8, generator=g))
    layer = MoeLayer(O.FP4_E2M1, hidden, inter, hidden, lists["gw"], lists["uw"], lists["dw"], lists["gs"],
                     lists["us"], lists["ds"])
    rng = np.random.default_rng(5)
    for tok in range(3):
        x = rng.standard_normal(hidden).astype(np.float32)
        logits = rng.standard_normal(E).astype(np.float32)
        out, ids, w = layer.forward(torch.from_numpy(logits).cuda(), k, torch.from_numpy(x).cuda(), renormalize=True)
        torch.cuda.synchronize()
        rid, rw = O.router_from_logits(logits, k, True)
        assert ids.cpu().numpy().tolist() == rid.tolist()
        sel = list(zip(rid.tolist(), rw.tolist()))
        host = {e: tuple(lists[n][e].cpu().numpy() for n in ("gw", "gs", "uw", "us", "dw", "ds")) for e, _ in sel}
        ref = O.selected_moe_native_fp4([host.get(e, host[sel[0][0]]) for e in range(E)], sel, x, hidden, inter,
                                        hidden)
        bound = moe_bound(fp4_matrices({e: host[e] for e, _ in sel}, hidden, inter, hidden), sel, x, hidden, inter,
                          hidden)
        _check(out.cpu().numpy(), ref, bound, f"fp4 layer token {tok}")


def test_bad_expert_id_leaves_later_calls_exact(cuda_device):
    """A call with an out-of-range expert id records code 8 in the device
    error word; later calls on the regular entry point, made without
    objb_device_error_take, still wait for every stage and return the same
    bits as before (their bounded waits stop early only on a timeout of their
    own CTA, never on an older code in the device word)."""
    import torch
    from objeta_b200.moe import MoeLayer
    from objeta_b200.quant import device_error_take
    H_, I_, O_, E_ = 4096, 14336, 4096, 3
    mats = _device_q4_layer(O.Q4_0, E_, H_, I_, O_, seed=77)
    layer = MoeLayer(O.Q4_0, H_, I_, O_, mats["gate"], mats["up"], mats["down"])
    x = torch.randn(H_, device="cuda")
    ids = torch.tensor([2, 0], dtype=torch.int32, device="cuda")
    w = torch.tensor([0.75, 0.25], device="cuda")
    device_error_take(cuda_device)
    ref = layer.forward_selected(ids, w, x).clone()
    torch.cuda.synchronize()
    assert device_error_take(cuda_device) == 0
    layer.forward_selected(torch.tensor([2, 9], dtype=torch.int32, device="cuda"), w, x)
    torch.cuda.synchronize()
    for _ in range(3):
        out = layer.forward_selected(ids, w, x)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert device_error_take(cuda_device) == 8


def test_no_device_errors_recorded(cuda_device):
    from objeta_b200.quant import device_error_take
    assert device_error_take(cuda_device) == 0
