"""The DeepSeek V4 gate on the device against cpu_gate_ref (oracle
restatement of dsl_moe.rs:768-881): selected ids bit-exact, weights within
4 ulp (exp / log1p are evaluated in double and rounded; glibc's f32
functions may differ by an ulp), on the reference's gate tests
(dsl_moe.rs:883-1000) and on random gates for all three score functions."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _run(gate, hidden, k, sf, rs, bias=None, tid2eid=None, input_ids=None):
    import torch
    from objeta_b200.ep import deepseek_gate
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dtype=dt)).cuda()
    ids, w = deepseek_gate(t(gate, np.float32), t(hidden, np.float32), k, sf, rs,
                           None if bias is None else t(bias, np.float32),
                           None if tid2eid is None else t(tid2eid, np.int64),
                           None if input_ids is None else t(input_ids, np.int64))
    torch.cuda.synchronize()
    return ids.cpu().numpy(), w.cpu().numpy()


def _check(gate, hidden, E, H, k, sf, rs, bias=None, tid2eid=None, input_ids=None):
    hid = np.asarray(hidden, np.float32).reshape(-1, H)
    ids, w = _run(gate, hid, k, sf, rs, bias, tid2eid, input_ids)
    for t in range(hid.shape[0]):
        rid, rw = O.deepseek_gate(gate, hid[t], E, H, k, sf, rs, gate_bias=bias, tid2eid=tid2eid,
                                  input_id=None if input_ids is None else int(input_ids[t]))
        assert ids[t].tolist() == rid.tolist(), (t, ids[t], rid)
        same = (np.abs(w[t] - rw) <= 4 * np.spacing(np.abs(rw))) | (np.isnan(w[t]) & np.isnan(rw))
        assert np.all(same), (t, w[t], rw)
    return ids, w


def test_gate_reference_cases(cuda_device):
    z = np.zeros((256, 4096), np.float32)
    ids, w = _check(z, np.full(4096, 0.1), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5)
    assert abs(float(w.sum()) - 1.5) < 1e-4
    g = z.copy()
    g[10], g[20], g[30] = 3.0, 2.0, 1.0
    ids, _ = _check(g, np.ones(4096), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5)
    assert ids[0, :3].tolist() == [10, 20, 30]
    g = z.copy()
    g[0] = 0.5
    g[100] = 2.0
    tid2eid = np.arange(129280 * 6) % 256
    ia, wa = _check(g, np.ones(4096), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5, tid2eid=tid2eid, input_ids=[0])
    # logit -2048 takes the reference's ln_1p(exp(-v)) branch: an infinite
    # score, so the normalised weights are [NaN, 0, ...] on both sides
    ib, wb = _check(g, -np.ones(4096), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5, tid2eid=tid2eid, input_ids=[0])
    assert ia.tolist() == ib.tolist() == [[0, 1, 2, 3, 4, 5]] and not np.array_equal(wa, wb, equal_nan=True)


@pytest.mark.parametrize("sf", [O.SOFTMAX, O.SIGMOID, O.SQRT_SOFTPLUS])
def test_gate_random(cuda_device, sf):
    rng = np.random.default_rng(sf)
    E, H, T, k = 256, 4096, 5, 8
    gate = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    hid = rng.standard_normal((T, H)).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    _check(gate, hid, E, H, k, sf, 1.5)
    _check(gate, hid, E, H, k, sf, 2.5, bias=bias)


def test_gate_hash_out_of_range_is_flagged(cuda_device):
    from objeta_b200.quant import device_error_take
    device_error_take(cuda_device)
    ids, w = _run(np.zeros((16, 64), np.float32), np.ones((1, 64)), 2, O.SQRT_SOFTPLUS, 1.5,
                  tid2eid=np.arange(10 * 2) % 16, input_ids=[10])
    assert ids.tolist() == [[-1, -1]] and np.isnan(w).all()
    assert device_error_take(cuda_device) & 8
