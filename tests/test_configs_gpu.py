"""BASELINE configs[2] and configs[4] at their full sizes against the CPU
oracle (selected_moe_cpu with gemv_cpu, moe.rs:1283-1324) and the propagated
reference bound.

Q4_0 layers with 8 experts of H 4096 / I 14336, top-2 of a softmax
router renormalised; one layer on two tokens, then the 4-layer stack the bench
times, each layer checked on the input the GPU gave it (the layers compose
exactly) and the stack's output compared with the oracle's own chain.
256 Q4_0 experts of H 2048 / I 512, top-8 Zipf(1.1) routing, 256
tokens through the one-rank expert-parallel layer (the tensor-core grouped
pairs), 32 of them checked against the oracle."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._moe_util import moe_bound, q4_matrices

pytestmark = pytest.mark.gpu


def _experts(n, H, I, O_, seed):
    import torch
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    qb = QuantBackend(torch.cuda.current_device())
    g = torch.Generator(device="cuda").manual_seed(seed)
    mats = {"gate": [], "up": [], "down": []}
    for _ in range(n):
        for name, (r, c) in (("gate", (I, H)), ("up", (I, H)), ("down", (O_, I))):
            m = torch.randn(r, c, device="cuda", generator=g) * 0.02
            mats[name].append(qb.quantize_matrix_device(QuantFormat.Q4_0, m, QGemvShape.new(QuantFormat.Q4_0, r, c)))
            del m
    return mats


class _HostExperts:
    """Host copies of the packed experts, fetched on first use."""

    def __init__(self, mats):
        self.mats = mats
        self.cache = {}

    def __getitem__(self, e):
        if e not in self.cache:
            self.cache[e] = tuple(self.mats[n][e].cpu().numpy() for n in ("gate", "up", "down"))
        return self.cache[e]

    def table(self, sel, n):
        first = self[sel[0][0]]
        return [self[e] if any(e == s for s, _ in sel) else first for e in range(n)]


def _check_token(host, n, sel, x, H, I, O_, got, what):
    ref = O.selected_moe_q4(host.table(sel, n), sel, x, H, I, O_)
    used = {e: host[e] for e, _ in sel}
    bound = moe_bound(q4_matrices(used, H, I, O_), sel, x, H, I, O_)
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    assert np.all(err <= bound), f"{what}: worst err/bound {np.max(err / bound):.3f}"
    return ref


C3 = dict(H=4096, I=14336, E=8, K=2, L=4)


@pytest.fixture(scope="module")
def c3_layers(cuda_device):
    import torch
    from objeta_b200.moe import MoeLayer
    layers = []
    for li in range(C3["L"]):
        m = _experts(C3["E"], C3["H"], C3["I"], C3["H"], seed=900 + li)
        layers.append((MoeLayer(O.Q4_0, C3["H"], C3["I"], C3["H"], m["gate"], m["up"], m["down"]), _HostExperts(m)))
    yield layers
    del layers
    torch.cuda.empty_cache()


def test_c3_layer_two_tokens(c3_layers):
    import torch
    H, I, E, K = C3["H"], C3["I"], C3["E"], C3["K"]
    layer, host = c3_layers[0]
    rng = np.random.default_rng(31)
    for tok in range(2):
        x = rng.standard_normal(H).astype(np.float32)
        logits = rng.standard_normal(E).astype(np.float32)
        out, ids, w = layer.forward(torch.from_numpy(logits).cuda(), K, torch.from_numpy(x).cuda(), renormalize=True)
        torch.cuda.synchronize()
        rid, rw = O.router_from_logits(logits, K, True)
        assert ids.cpu().numpy().tolist() == rid.tolist()
        np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=0)
        _check_token(host, E, list(zip(rid.tolist(), rw.tolist())), x, H, I, H, out.cpu().numpy(), f"token {tok}")


def test_c3_four_layer_stack(c3_layers):
    import torch
    H, I, E, K = C3["H"], C3["I"], C3["E"], C3["K"]
    rng = np.random.default_rng(77)
    x0 = rng.standard_normal(H).astype(np.float32)
    logits = rng.standard_normal((C3["L"], E)).astype(np.float32)
    x = torch.from_numpy(x0).cuda()
    xs_gpu, outs = [], []
    for li, (layer, _) in enumerate(c3_layers):
        out, _, _ = layer.forward(torch.from_numpy(logits[li]).cuda(), K, x, renormalize=True)
        torch.cuda.synchronize()
        xs_gpu.append(x.cpu().numpy())
        outs.append(out.cpu().numpy())
        x = out
    chain = x0
    for li, (_, host) in enumerate(c3_layers):
        rid, rw = O.router_from_logits(logits[li], K, True)
        sel = list(zip(rid.tolist(), rw.tolist()))
        # this layer on the GPU's own input: within the bound
        _check_token(host, E, sel, xs_gpu[li], H, I, H, outs[li], f"layer {li}")
        chain = O.selected_moe_q4(host.table(sel, E), sel, chain, H, I, H)
    d = O.compare_outputs(chain, outs[-1])
    assert d["cosine_similarity"] > 0.99999 and d["relative_l2_error"] < 1e-4, d


def test_c5_full_size_grouped(cuda_device):
    import torch
    from objeta_b200.ep import ExpertParallelMoe
    from objeta_b200.moe import MoeLayer
    from objeta_b200.quant import device_error_take
    H, I, E, K, T = 2048, 512, 256, 8, 256
    m = _experts(E, H, I, H, seed=4242)
    layer = MoeLayer(O.Q4_0, H, I, H, m["gate"], m["up"], m["down"])
    host = _HostExperts(m)
    perm = np.random.default_rng(7).permutation(E)
    rng = np.random.default_rng(1256)
    p = 1.0 / np.arange(1, E + 1) ** 1.1
    p /= p.sum()
    ids = np.stack([perm[rng.choice(E, K, replace=False, p=p)] for _ in range(T)]).astype(np.int32)
    lg = rng.standard_normal((T, K))
    ws = np.exp(lg - lg.max(1, keepdims=True))
    ws = (ws / ws.sum(1, keepdims=True)).astype(np.float32)
    xs = rng.standard_normal((T, H)).astype(np.float32)
    ep = ExpertParallelMoe(layer, E, K)
    device_error_take(cuda_device)
    out = ep.forward(torch.from_numpy(xs).cuda(), torch.from_numpy(ids).cuda(), torch.from_numpy(ws).cuda())
    torch.cuda.synchronize()
    assert device_error_take(cuda_device) == 0
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    for t in range(0, T, T // 32):
        sel = list(zip(ids[t].tolist(), ws[t].tolist()))
        _check_token(host, E, sel, xs[t], H, I, H, got[t], f"token {t}")
