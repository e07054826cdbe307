"""GPU parity of the batch-1 GEMV, the device packers and the FP4 decode
against the CPU oracle (reference arithmetic).  Run with -m gpu on a B200."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import TOL, assert_rows_within

pytestmark = pytest.mark.gpu

FORMATS = [O.Q4_0, O.Q5_0, O.IQ3_0, O.FP4_E2M1]
# quant.rs:1714-1857 cosine thresholds of the reference's own sweeps
COS_MIN = {O.Q4_0: 0.990, O.Q5_0: 0.995, O.IQ3_0: 0.970, O.FP4_E2M1: 0.9999}


@pytest.fixture(scope="module")
def qb(cuda_device):
    from objeta_b200 import QuantBackend
    return QuantBackend(cuda_device)


def _torch():
    import torch
    return torch


# ---------------------------------------------------------- reference sweep
@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("rows,cols", [(1, 32), (16, 32), (128, 256), (1024, 4096)])
def test_run_case_seed_sweep(qb, fmt, rows, cols):
    """quant.rs:1622-1662 run_case + the *_correctness_and_seed_sweep tests:
    host-slice QuantBackend.gemv vs gemv_cpu on the reference's LCG inputs."""
    from objeta_b200 import QGemvShape, QuantFormat
    for seed in (0, 1, 2, 3, 4, 123):
        m = O.seeded_f32s(rows * cols, seed ^ 0xA5A5_5A5A_1234_5678)
        x = O.seeded_f32s(cols, seed ^ 0xD00D_F00D_1234_5678)
        q = O.quantize_matrix(fmt, m, rows, cols)
        ref = O.gemv(fmt, q, x, rows, cols)
        shape = QGemvShape.new(QuantFormat(fmt), rows, cols)
        y, tel = qb.gemv(QuantFormat(fmt), None, q, x, shape)
        assert_rows_within(y, ref, O.row_abs_sums(fmt, q, x, rows, cols), what=f"fmt={fmt} seed={seed}")
        assert O.compare_outputs(ref, y)["cosine_similarity"] > COS_MIN[fmt]
        assert tel.bytes_read == q.size + 4 * cols
        assert tel.kernel_ms > 0 and tel.total_ms >= tel.kernel_ms


# ----------------------------------------------------- device packers exact
def _edge_matrix(rows, cols, rng):
    m = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    m[0, :32] = 0.0                                   # all-zero block -> 1e-10 scale
    m[0, 32:64] = 0.0
    m[0, 40] = 3.5                                    # single spike
    m[1, :32] = np.linspace(-1, 1, 32, dtype=np.float32)
    m[1, 32:64] = np.float32(2.0 ** -140)             # subnormal scale path
    m[1, 64:96] = np.float32(6.0) * np.arange(32, dtype=np.float32) / 31  # FP4 exact grid
    m[2, :32] = np.float32(1e30)
    m[2, 32:64] = -np.float32(7.0) * (np.arange(32) % 15 - 7) / 7  # ties for Q4 rounding
    m[2, 64:96] = np.float32(-0.0)
    m[3, :32] = np.float32(6.0) * np.float32(2.0 ** 7) * (1 + np.float32(2.0 ** -23))  # log2 edge
    m[3, 32:64] = np.float32(np.nan)
    m[3, 32] = 1.0
    return m


@pytest.mark.parametrize("fmt", FORMATS)
def test_device_quantizer_is_byte_exact(cuda_device, fmt):
    torch = _torch()
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    qb = QuantBackend(cuda_device)
    rng = np.random.default_rng(1234 + fmt)
    for rows, cols in [(4, 128), (257, 512), (64, 4096)]:
        m = _edge_matrix(rows, cols, rng)
        shape = QGemvShape.new(QuantFormat(fmt), rows, cols)
        got = qb.quantize_matrix(QuantFormat(fmt), m, shape)
        ref = O.quantize_matrix(fmt, m, rows, cols)
        assert got.dtype == np.uint8 and got.size == ref.size
        diff = np.nonzero(got != ref)[0]
        assert diff.size == 0, f"first differing byte {diff[:8]} got {got[diff[:8]]} ref {ref[diff[:8]]}"
    # the reference LCG data too
    m = O.seeded_f32s(128 * 256, 77)
    assert np.array_equal(qb.quantize_matrix(QuantFormat(fmt), m, QGemvShape.new(QuantFormat(fmt), 128, 256)),
                          O.quantize_matrix(fmt, m, 128, 256))
    torch.cuda.synchronize()


def test_fp4_log2_ceiling_edges(cuda_device):
    """ceil(log2(amax/6)) at and one ulp around powers of two, for every
    exponent the E8M0 byte can hold."""
    from objeta_b200 import QGemvShape, QuantBackend, QuantFormat
    qb = QuantBackend(cuda_device)
    vals = []
    for e in range(-140, 128):
        base = np.float32(6.0) * np.float32(2.0) ** np.float32(e) if e > -126 else np.float32(6.0 * 2.0 ** e)
        for d in (-2, -1, 0, 1, 2, 3):
            v = np.nextafter(base, np.float32(np.inf)) if d > 0 else base
            for _ in range(max(d - 1, 0)):
                v = np.nextafter(v, np.float32(np.inf))
            if d < 0:
                v = base
                for _ in range(-d):
                    v = np.nextafter(v, np.float32(0))
            vals.append(np.float32(v))
    vals = np.array([v for v in vals if np.isfinite(v) and v > 0], np.float32)
    n = (vals.size + 31) // 32 * 32
    m = np.zeros(n * 32, np.float32)
    m[::32][: vals.size] = vals  # one value per 32-block
    m = m[: n * 32]
    rows = n // 32
    got = qb.quantize_matrix(QuantFormat.DeepSeekFp4E2M1, m, QGemvShape.deepseek_fp4(rows, 32 * 32))
    ref = O.quantize_matrix(O.FP4_E2M1, m, rows, 32 * 32)
    assert np.array_equal(got, ref)


# ------------------------------------------------------------ FP4 decode
def test_fp4_decode_split_bit_exact(cuda_device):
    torch = _torch()
    from objeta_b200.quant import fp4_decode_split_device
    scales = [0, 1, 100, 119, 123, 127, 128, 200, 253, 254, 255]
    rows, cols = len(scales), 512
    w = np.tile(np.arange(256, dtype=np.uint8), rows)
    s = np.repeat(np.array(scales, np.uint8), cols // 32)
    dw = torch.from_numpy(w).cuda()
    ds = torch.from_numpy(s).cuda()
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    fp4_decode_split_device(dw, ds, rows, cols, out)
    got = out.cpu().numpy()
    ref = O.fp4_decode_split(w, s, rows, cols, 32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), "decode must be bit-exact (incl. +0.0 for code 8, NaN for 0*inf)"


# --------------------------------------------- full-size shapes (device API)
def _device_case(fmt, rows, cols, seed):
    torch = _torch()
    from objeta_b200.quant import QuantBackend, QGemvShape, QuantFormat
    g = torch.Generator(device="cuda").manual_seed(seed)
    dm = torch.randn(rows, cols, device="cuda", generator=g) * 0.02
    dx = torch.randn(cols, device="cuda", generator=g)
    qb = QuantBackend(torch.cuda.current_device())
    shape = QGemvShape.new(QuantFormat(fmt), rows, cols)
    dq = qb.quantize_matrix_device(QuantFormat(fmt), dm, shape)
    del dm
    dy = torch.empty(rows, device="cuda")
    qb.launch_kernel(QuantFormat(fmt), torch.cuda.current_stream(), dq, dx, dy, shape)
    torch.cuda.synchronize()
    return dq, dx, dy


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096), (4096, 14336), (151936, 2048)])
def test_baseline_sweep_shapes(cuda_device, fmt, rows, cols):
    dq, dx, dy = _device_case(fmt, rows, cols, seed=rows * 7 + cols + fmt)
    q = dq.cpu().numpy()
    x = dx.cpu().numpy()
    ref = O.gemv(fmt, q, x, rows, cols, threads=0)
    assert_rows_within(dy.cpu().numpy(), ref, O.row_abs_sums(fmt, q, x, rows, cols),
                       what=f"fmt={fmt} {rows}x{cols}")


@pytest.mark.parametrize("rows,cols", [(2048, 4096), (4096, 2048), (512, 7168), (3, 512), (40, 96)])
def test_split_fp4_gemv(cuda_device, rows, cols):
    torch = _torch()
    from objeta_b200.quant import gemv_fp4_split_device
    rng = np.random.default_rng(rows + cols)
    w = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
    s = rng.integers(119, 124, rows * cols // 32, dtype=np.uint8)
    x = rng.standard_normal(cols).astype(np.float32)
    dy = torch.empty(rows, device="cuda")
    gemv_fp4_split_device(torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda(),
                          torch.from_numpy(x).cuda(), dy, rows, cols)
    torch.cuda.synchronize()
    # the split layout is the interleaved layout with the scale byte moved out
    inter = np.concatenate([s.reshape(rows, cols // 32, 1), w.reshape(rows, cols // 32, 16)],
                           axis=2).reshape(-1)
    ref = O.gemv(O.FP4_E2M1, inter, x, rows, cols, threads=0)
    assert_rows_within(dy.cpu().numpy(), ref, O.row_abs_sums(O.FP4_E2M1, inter, x, rows, cols),
                       what=f"split fp4 {rows}x{cols}")


# ------------------------------------------------------ fallback + edges
@pytest.mark.parametrize("fmt", FORMATS)
def test_fallback_misaligned_and_ragged(cuda_device, fmt):
    torch = _torch()
    from objeta_b200.quant import gemv_device
    bb = O.BLOCK_BYTES[fmt]
    for rows, cols, offset in [(37, 96, 0), (64, 4096, 1), (5, 32, 3), (300, 2080, 0)]:
        m = O.seeded_f32s(rows * cols, rows * 31 + cols)
        x = O.seeded_f32s(cols, cols)
        q = O.quantize_matrix(fmt, m, rows, cols)
        buf = torch.zeros(q.size + 64, dtype=torch.uint8, device="cuda")
        buf[offset:offset + q.size] = torch.from_numpy(q).cuda()
        view = buf[offset:offset + q.size]
        dy = torch.empty(rows, device="cuda")
        gemv_device(fmt, view.data_ptr(), torch.from_numpy(x).cuda(), dy, rows, cols)
        torch.cuda.synchronize()
        ref = O.gemv(fmt, q, x, rows, cols)
        assert_rows_within(dy.cpu().numpy(), ref, O.row_abs_sums(fmt, q, x, rows, cols),
                           what=f"fmt={fmt} {rows}x{cols}+{offset}")
        assert q.size == rows * cols // 32 * bb


@pytest.mark.parametrize("fmt", FORMATS + ["split"])
def test_inline_x_matches_ximage_launch(cuda_device, fmt):
    """With x 16-byte aligned the GEMV kernel forms its x registers itself
    (digit images up to 4096 columns built in shared memory, interleaved FP4
    quads loaded from x); with x misaligned an ximage launch builds them
    first.  Both give the same bits, including blocks of zeros, tiny and huge
    magnitudes, Inf and NaN.  The 14336-column digit shapes and split FP4 rows
    take the image launch either way (the case still checks alignment does not
    change their bits)."""
    torch = _torch()
    from objeta_b200.quant import gemv_device, gemv_fp4_split_device
    for rows, cols in [(4096, 4096), (300, 14336), (64, 2048), (7, 96)]:
        rng = np.random.default_rng(rows + cols)
        x = rng.standard_normal(cols).astype(np.float32)
        x[32:64] = 0.0
        x[64:96] *= 1e-39
        if cols >= 512:
            x[96:128] *= 1e30
            x[130] = np.inf
            x[200] = np.nan
        if fmt == "split":
            w = torch.from_numpy(rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)).cuda()
            sc = torch.from_numpy(rng.integers(119, 124, rows * cols // 32, dtype=np.uint8)).cuda()
            run = lambda xv, y: gemv_fp4_split_device(w, sc, xv, y, rows, cols)
        else:
            m = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
            q = torch.from_numpy(O.quantize_matrix(fmt, m, rows, cols)).cuda()
            run = lambda xv, y: gemv_device(fmt, q, xv, y, rows, cols)
        xa = torch.from_numpy(x).cuda()
        assert xa.data_ptr() % 16 == 0
        buf = torch.zeros(cols + 4, device="cuda")
        buf[1:1 + cols] = xa
        xm = buf[1:1 + cols]
        ya = torch.empty(rows, device="cuda")
        ym = torch.empty(rows, device="cuda")
        run(xa, ya)
        run(xm, ym)
        torch.cuda.synchronize()
        assert torch.equal(ya.view(torch.int32), ym.view(torch.int32)), (fmt, rows, cols)


def test_gemv_is_deterministic(cuda_device):
    torch = _torch()
    dq, dx, dy = _device_case(O.Q4_0, 14336, 4096, seed=5)
    from objeta_b200.quant import gemv_device
    dy2 = torch.empty_like(dy)
    gemv_device(O.Q4_0, dq, dx, dy2, 14336, 4096)
    torch.cuda.synchronize()
    assert torch.equal(dy, dy2)


def test_rejects_non_multiple_cols(qb):
    import objeta_b200
    from objeta_b200 import QGemvShape, QuantFormat
    shape = QGemvShape.q4_0(4, 33)
    with pytest.raises(objeta_b200.CudaError) as ei:
        qb.gemv(QuantFormat.Q4_0, None, np.zeros(4 * 18, np.uint8), np.zeros(33, np.float32), shape)
    assert "multiple of block_size" in ei.value.source_message


def test_rejects_size_mismatch(qb):
    import objeta_b200
    from objeta_b200 import QGemvShape, QuantFormat
    shape = QGemvShape.q4_0(4, 64)
    with pytest.raises(objeta_b200.CudaError) as ei:
        qb.gemv(QuantFormat.Q4_0, None, np.zeros(10, np.uint8), np.zeros(64, np.float32), shape)
    assert "qweights len 10 != expected 144" in ei.value.source_message


def test_no_pipeline_timeouts_recorded(cuda_device):
    from objeta_b200.quant import device_error_take
    assert device_error_take(cuda_device) == 0
