"""Outlier vectors on the GPU: blocks whose largest |x| dwarfs their other
values (the "wide" blocks of the integer digit images) against the CPU oracle
with the reference bound, max |err| <= 1e-5 * sum|w x| per row (propagated
through SwiGLU and the combine for the MoE paths).

Outliers of 1e3, 1e4 and 1e5 (and a block of seven of 3e4) sit in the
vector, and half of every matrix's
rows weigh them by the zero code (their dense weight is set to 0 before the
reference packer quantizes it), which is the case the integer path alone
misses.  Covered: the GEMV at the BASELINE configs[1] shapes (in-kernel image
up to 4096 columns, image launch at 14336 and for a misaligned x), the fused
single-token MoE (outliers in x and, through scaled gate / up rows, in the
activations the down rows read), the CUDA-core pairs and the tensor-core
pairs."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._moe_util import moe_bound, q4_matrices
from tests._util import assert_rows_within

pytestmark = pytest.mark.gpu

DIGIT_FORMATS = [O.Q4_0, O.Q5_0, O.IQ3_0]
MAGS = (1e3, -1e4, 1e5)


def _outlier_x(cols, seed, per_block=(1, 1, 2)):
    """N(0,1) with outlier groups: one value of 1e3 in one block, one of -1e4
    in another, two of 1e5 in a third (and a block with 7 outliers of 3e4,
    the most one block may hold)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(cols).astype(np.float32)
    nb = cols // 32
    blocks = rng.choice(nb, 4, replace=False)
    cols_out = []
    for b, mag, n in zip(blocks[:3], MAGS, per_block):
        for c in rng.choice(32, n, replace=False):
            x[b * 32 + c] = mag
            cols_out.append(b * 32 + c)
    for c in rng.choice(32, 7, replace=False):
        x[blocks[3] * 32 + c] = 3e4
        cols_out.append(blocks[3] * 32 + c)
    return x, np.array(cols_out)


def _quantize_zeroing(fmt, rows, cols, zero_cols, seed, scale_rows=None):
    """Device weights N(0, 0.02^2) packed by the byte-exact device packer; rows
    [0, rows/2) get weight 0 at zero_cols; scale_rows are multiplied by 200."""
    import torch
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    qb = QuantBackend(torch.cuda.current_device())
    g = torch.Generator(device="cuda").manual_seed(seed)
    m = torch.randn(rows, cols, device="cuda", generator=g) * 0.02
    if zero_cols is not None and len(zero_cols):
        zc = torch.from_numpy(np.asarray(zero_cols, np.int64)).cuda()
        m[: rows // 2, zc] = 0.0
    if scale_rows is not None:
        m[torch.from_numpy(np.asarray(scale_rows, np.int64)).cuda()] *= 200.0
    return qb.quantize_matrix_device(QuantFormat(fmt), m, QGemvShape.new(QuantFormat(fmt), rows, cols))


@pytest.mark.parametrize("fmt", DIGIT_FORMATS)
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096), (4096, 14336), (151936, 2048)])
def test_gemv_outliers_at_baseline_shapes(cuda_device, fmt, rows, cols):
    import torch
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    x, oc = _outlier_x(cols, seed=rows + cols + fmt)
    dq = _quantize_zeroing(fmt, rows, cols, oc, seed=fmt * 31 + cols)
    qb = QuantBackend(cuda_device)
    shape = QGemvShape.new(QuantFormat(fmt), rows, cols)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(rows, device="cuda")
    qb.launch_kernel(QuantFormat(fmt), torch.cuda.current_stream(), dq, dx, dy, shape)
    # a misaligned x takes the image launch instead of the in-kernel image
    buf = torch.zeros(cols + 4, device="cuda")
    buf[1:1 + cols] = dx
    dy2 = torch.empty(rows, device="cuda")
    qb.launch_kernel(QuantFormat(fmt), torch.cuda.current_stream(), dq, buf[1:1 + cols], dy2, shape)
    torch.cuda.synchronize()
    q = dq.cpu().numpy()
    ref = O.gemv(fmt, q, x, rows, cols, threads=0)
    sums = O.row_abs_sums(fmt, q, x, rows, cols)
    assert_rows_within(dy.cpu().numpy(), ref, sums, what=f"fmt={fmt} {rows}x{cols}")
    assert_rows_within(dy2.cpu().numpy(), ref, sums, what=f"fmt={fmt} {rows}x{cols} misaligned x")
    # the two image builders mark the same blocks: the rows are the same bits
    assert torch.equal(dy, dy2)


@pytest.mark.parametrize("fmt", DIGIT_FORMATS)
def test_gemv_outliers_host_api(cuda_device, fmt):
    """QuantBackend.gemv (host slices) on the reference packer's bytes."""
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    rows, cols = 1024, 4096
    x, oc = _outlier_x(cols, seed=5 + fmt)
    rng = np.random.default_rng(fmt)
    m = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    m[: rows // 2, oc] = 0.0
    q = O.quantize_matrix(fmt, m, rows, cols)
    y, _ = QuantBackend(cuda_device).gemv(QuantFormat(fmt), None, q, x, QGemvShape.new(QuantFormat(fmt), rows, cols))
    assert_rows_within(y, O.gemv(fmt, q, x, rows, cols), O.row_abs_sums(fmt, q, x, rows, cols),
                       what=f"host api fmt={fmt}")


def _layer(fmt, E, H, I, OUT, x_outlier_cols, act_rows, seed):
    from objeta_b200.moe import MoeLayer
    mats = {"gate": [], "up": [], "down": []}
    for e in range(E):
        mats["gate"].append(_quantize_zeroing(fmt, I, H, x_outlier_cols, seed * 7 + 3 * e, act_rows))
        mats["up"].append(_quantize_zeroing(fmt, I, H, x_outlier_cols, seed * 7 + 3 * e + 1, act_rows))
        mats["down"].append(_quantize_zeroing(fmt, OUT, I, act_rows, seed * 7 + 3 * e + 2))
    return MoeLayer(fmt, H, I, OUT, mats["gate"], mats["up"], mats["down"]), mats


def _host(mats, E):
    return [(mats["gate"][e].cpu().numpy(), mats["up"][e].cpu().numpy(), mats["down"][e].cpu().numpy())
            for e in range(E)]


def _moe_ref(fmt, host, sel, x, H, I, OUT):
    """selected_moe_cpu (moe.rs:1283-1324) with this format's gemv_cpu."""
    ref = np.zeros(OUT, np.float32)
    for e, wt in sel:
        gg = O.gemv(fmt, host[e][0], x, I, H)
        uu = O.gemv(fmt, host[e][1], x, I, H)
        a = np.array([np.float32(v / (np.float32(1) + np.exp(np.float32(-v)))) * np.float32(q)
                      for v, q in zip(gg, uu)], np.float32)
        ref += np.float32(wt) * O.gemv(fmt, host[e][2], a, OUT, I)
    return ref


@pytest.mark.parametrize("fmt", DIGIT_FORMATS)
def test_moe_selected_outliers(cuda_device, fmt):
    """objb_moe_selected_device: outliers in x (gate / up rows) and in the
    activations (down rows)."""
    import torch
    with np.errstate(over="ignore"):
        E, H, I, OUT, K = 6, 1024, 2048, 1024, 3
        x, oc = _outlier_x(H, seed=11 + fmt)
        act_rows = np.array([5, 6, 300, 301, 302, 1500])
        layer, mats = _layer(fmt, E, H, I, OUT, oc, act_rows, seed=fmt + 1)
        host = _host(mats, E)
        for sel in ([(1, 0.5), (4, 0.3), (0, 0.2)], [(5, 1.0), (2, 0.25), (3, -0.5)]):
            ids = torch.tensor([e for e, _ in sel], dtype=torch.int32, device="cuda")
            w = torch.tensor([v for _, v in sel], dtype=torch.float32, device="cuda")
            out = layer.forward_selected(ids, w, torch.from_numpy(x).cuda())
            torch.cuda.synchronize()
            ref = _moe_ref(fmt, host, sel, x, H, I, OUT)
            bound = moe_bound(q4_matrices(host, H, I, OUT, fmt), sel, x, H, I, OUT)
            err = np.abs(out.cpu().numpy().astype(np.float64) - ref)
            assert np.all(err <= bound), f"fmt {fmt}: worst err/bound {np.max(err / bound):.3f}"


def _pairs(T, K, E, seed):
    import torch
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    ws = rng.random((T, K)).astype(np.float32)
    pe = ids.reshape(-1)
    pt = np.repeat(np.arange(T, dtype=np.int32), K)
    po = np.arange(T * K, dtype=np.int32)
    order = np.argsort(pe, kind="stable")

    def cuda(a):
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return ids, ws, cuda(pe[order]), cuda(pt[order]), cuda(po[order])


@pytest.mark.parametrize("path", ["cuda_core", "tensor_core"])
def test_pairs_outliers(cuda_device, path):
    """Multi-token pairs (objb_moe_pairs_device / objb_moe_pairs_tc_device):
    tokens with and without outliers in one launch, every token against the
    oracle MoE; configs[4]'s expert shape (H 2048, I 512)."""
    import torch
    from objeta_b200.ep import moe_combine, moe_pairs, moe_pairs_tc
    from objeta_b200.quant import device_error_take
    with np.errstate(over="ignore"):
        E, H, I, OUT, K, T = 8, 2048, 512, 2048, 4, 40
        xs = np.random.default_rng(1).standard_normal((T, H)).astype(np.float32)
        xo, oc = _outlier_x(H, seed=3)
        for t in range(0, T, 3):
            xs[t] = xo if t % 2 == 0 else -xo
        act_rows = np.array([7, 8, 9, 200, 201, 450])
        layer, mats = _layer(O.Q4_0, E, H, I, OUT, oc, act_rows, seed=9)
        ids, ws, pe, pt, po = _pairs(T, K, E, seed=4)
        v = torch.full((T * K, OUT), float("nan"), device="cuda")
        device_error_take(cuda_device)
        (moe_pairs_tc if path == "tensor_core" else moe_pairs)(layer, pe, pt, torch.from_numpy(xs).cuda(), v,
                                                               pair_out=po)
        slot = torch.arange(T * K, dtype=torch.int32, device="cuda").reshape(T, K)
        out = torch.empty(T, OUT, device="cuda")
        moe_combine(v, slot, torch.from_numpy(ws).cuda(), out)
        torch.cuda.synchronize()
        assert device_error_take(cuda_device) == 0
        got = out.cpu().numpy()
        host = _host(mats, E)
        for t in range(T):
            sel = list(zip(ids[t].tolist(), ws[t].tolist()))
            ref = _moe_ref(O.Q4_0, host, sel, xs[t], H, I, OUT)
            bound = moe_bound(q4_matrices(host, H, I, OUT), sel, xs[t], H, I, OUT)
            err = np.abs(got[t].astype(np.float64) - ref)
            assert np.all(err <= bound), f"{path} token {t}: worst err/bound {np.max(err / bound):.3f}"


@pytest.mark.parametrize("rows,cols", [(2048, 4096), (4096, 2048), (512, 7168)])
def test_split_fp4_gemv_outliers(cuda_device, rows, cols):
    """Split FP4 rows (objb_gemv_fp4_split_device) on the integer digit path:
    outliers over zero codes (both zero codes, 0 and 8, appear) against the
    interleaved-FP4 gemv_cpu of the same bytes."""
    import torch
    from objeta_b200.quant import gemv_fp4_split_device
    rng = np.random.default_rng(rows + 3 * cols)
    w = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
    s = rng.integers(119, 124, rows * cols // 32, dtype=np.uint8)
    x, oc = _outlier_x(cols, seed=cols + 1)
    W = w.reshape(rows, cols // 2)
    for i, c in enumerate(oc):   # rows [0, rows/2): code 0 or 8 at every outlier column
        zero = 0x0 if i % 2 else 0x8
        if c % 2 == 0:
            W[: rows // 2, c // 2] = (W[: rows // 2, c // 2] & 0xF0) | zero
        else:
            W[: rows // 2, c // 2] = (W[: rows // 2, c // 2] & 0x0F) | (zero << 4)
    dy = torch.empty(rows, device="cuda")
    gemv_fp4_split_device(torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(x).cuda(), dy,
                          rows, cols)
    torch.cuda.synchronize()
    inter = np.concatenate([s.reshape(rows, cols // 32, 1), w.reshape(rows, cols // 32, 16)], axis=2).reshape(-1)
    ref = O.gemv(O.FP4_E2M1, inter, x, rows, cols, threads=0)
    assert_rows_within(dy.cpu().numpy(), ref, O.row_abs_sums(O.FP4_E2M1, inter, x, rows, cols),
                       what=f"split fp4 {rows}x{cols} outliers")
