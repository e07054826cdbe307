"""Experts read from a safetensors file (mmap, pinned) through the expert
cache give the same bits as the same experts held in ordinary memory."""
import json
import struct

import numpy as np
import pytest

from tests._moe_util import make_q4_experts

pytestmark = pytest.mark.gpu


def test_pinned_safetensors_experts_feed_the_cache(cuda_device, tmp_path):
    import torch
    from objeta_b200 import QuantBackend
    from objeta_b200.moe import CudaExpertCache, ExpertWeights, MoeExecutor
    from objeta_b200.weights import ModelWeights
    E, H, I, O_ = 4, 512, 256, 512
    experts, _ = make_q4_experts(E, H, I, O_, seed=21)
    header, blobs, off = {}, [], 0
    for e, (g, u, d) in enumerate(experts):
        for n, a in (("w1", g), ("w3", u), ("w2", d)):
            header[f"layers.0.experts.{e}.{n}.weight"] = {"dtype": "U8", "shape": [a.size],
                                                          "data_offsets": [off, off + a.size]}
            blobs.append(a.tobytes())
            off += a.size
    h = json.dumps(header).encode()
    p = tmp_path / "experts.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + b"".join(blobs))
    w = ModelWeights(p)
    w.pin()
    mapped = [ExpertWeights(w.get_raw(f"layers.0.experts.{e}.w1.weight"), w.get_raw(f"layers.0.experts.{e}.w3.weight"),
                            w.get_raw(f"layers.0.experts.{e}.w2.weight")) for e in range(E)]
    plain = [ExpertWeights(g, u, d) for g, u, d in experts]
    x = np.random.default_rng(4).standard_normal(H).astype(np.float32)
    sel = [(2, 0.6), (0, 0.4)]
    ex, qb = MoeExecutor(0), QuantBackend(0)
    a, _ = ex.execute_selected_moe_cuda(qb, None, plain, sel, x, H, I, O_, 0, CudaExpertCache(1 << 28, 0))
    b, tel = ex.execute_selected_moe_cuda(qb, None, mapped, sel, x, H, I, O_, 0, CudaExpertCache(1 << 28, 0))
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert tel.actual_expert_bytes_loaded == 2 * (2 * experts[0][0].size + experts[0][2].size)
    # a tensor straight to the device
    d = torch.empty(experts[1][2].size, dtype=torch.uint8, device="cuda")
    w.to_device("layers.0.experts.1.w2.weight", d)
    torch.cuda.synchronize()
    assert np.array_equal(d.cpu().numpy(), experts[1][2])
    w.close()
