"""A numpy model of the integer ("digit image") block sums of the Q4_0 / Q5_0 /
IQ3_0 GEMV kernels, checked against the CPU oracle (gemv_cpu, quant.rs:627-1019)
with the 1e-5 * sum|w x| row bound, on vectors with outlier values.

The kernels hold each 32-value block of x as X = rint(x * 2^(20-E)) (2^E above
the block's largest |x|) and form sum_l (q_l - off) X_l exactly in integers;
a block whose few largest values dwarf the others ("wide": the half-step
rounding of its values can exceed 2^-14 of their mass, each value capped at
2^-5 of the block scale) is left out of the integer sum and added in fp32
instead.  This file states
that arithmetic in numpy (integer sums exact, per-block fp32 products as the
kernel rounds them, the sum over blocks in f64) so the rule can be judged on
the CPU: with it every row holds the bound for outliers from 30 to 3e6 times
the ordinary values; without
it, outliers of 1e4 over zero-weight columns break the bound.  The GPU tests
(test_gemv_gpu.py, test_moe_gpu.py, test_moe_pairs_tc_gpu.py) run the real
kernels on the same kind of inputs.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import TOL

OFFSET = {O.Q4_0: 8, O.Q5_0: 16, O.IQ3_0: 4}


def unpack_codes(fmt, q, rows, cols):
    """(q - off) as int64 [rows, nb, 32] and the f16 block scales as f32."""
    bb = O.BLOCK_BYTES[fmt]
    nb = cols // 32
    blk = np.asarray(q, np.uint8).reshape(rows, nb, bb)
    s = blk[:, :, 0].astype(np.uint16) | (blk[:, :, 1].astype(np.uint16) << 8)
    scale = s.view(np.float16).astype(np.float32)
    lane = np.arange(32)
    if fmt == O.Q4_0:
        by = blk[:, :, 2 + lane // 2].astype(np.int64)
        code = (by >> (4 * (lane & 1))) & 0xF
    elif fmt == O.Q5_0:
        lo = (blk[:, :, 6 + lane // 2].astype(np.int64) >> (4 * (lane & 1))) & 0xF
        hi = (blk[:, :, 2 + lane // 8].astype(np.int64) >> (lane & 7)) & 1
        code = lo | (hi << 4)
    else:
        lo = (blk[:, :, 2 + lane // 4].astype(np.int64) >> (2 * (lane & 3))) & 3
        hi = (blk[:, :, 10 + lane // 8].astype(np.int64) >> (lane & 7)) & 1
        code = lo | (hi << 2)
    return code - OFFSET[fmt], scale


def digit_X(xb):
    """X = rint(x * 2^(20-E)) per block (E: frexp exponent of the block max)."""
    m = np.abs(xb).max(axis=1)
    _, E = np.frexp(m)
    with np.errstate(invalid="ignore", over="ignore"):
        X = np.rint(np.ldexp(xb.astype(np.float64), (20 - E)[:, None]))
        X = np.where(np.isfinite(X), X, 0).astype(np.int64)
    return X, E, m


def wide_blocks(xb):
    """The kernels' wide-block rule on x blocks [nb, 32] (f32): with
    y = x 2^(20-E), c = #{|y| >= 2^-8} and R = sum min(|X|, 2^15),
    wide <=> c >= 2 and c * 2^13 > R."""
    X, E, m = digit_X(xb)
    with np.errstate(invalid="ignore", over="ignore"):
        y = np.nan_to_num(np.abs(np.ldexp(xb.astype(np.float64), (20 - E)[:, None])))
    c = (y >= 2.0 ** -8).sum(axis=1)
    R = np.minimum(np.abs(X), 1 << 15).sum(axis=1)
    return np.isfinite(m) & (c >= 2) & (c * 8192 > R)


def digit_gemv(fmt, q, x, rows, cols, wide_rule=True):
    codes, scale = unpack_codes(fmt, q, rows, cols)
    nb = cols // 32
    xb = np.asarray(x, np.float32).reshape(nb, 32)
    X, E, _ = digit_X(xb)
    wide = wide_blocks(xb) if wide_rule else np.zeros(nb, bool)
    X[wide] = 0
    T = np.einsum("rbl,bl->rb", codes, X)                      # exact block sums
    word = np.ldexp(np.float32(1.0), E - 20).astype(np.float32)
    blockval = T.astype(np.float32) * (scale * word[None, :])  # f32, as the kernel
    y = blockval.astype(np.float64).sum(axis=1)
    if wide.any():
        w = (codes[:, wide, :].astype(np.float32) * scale[:, wide, None]).astype(np.float32)
        terms = (w * xb[wide][None, :, :]).astype(np.float32)
        y += terms.astype(np.float64).sum(axis=(1, 2))
    return y


def _case(fmt, rows, cols, outliers, seed, zero_frac=0.5):
    rng = np.random.default_rng(seed)
    m = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    for c, v in outliers:
        x[c] = v
        m[: int(rows * zero_frac), c] = 0.0   # those rows weigh the outlier by code `off` (zero)
    q = O.quantize_matrix(fmt, m, rows, cols)
    return q, x


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q5_0, O.IQ3_0])
@pytest.mark.parametrize("mag", [30.0, 100.0, 300.0, 1e3, 1e4, 1e5, 1e6, -3e6])
def test_wide_rule_holds_the_bound(fmt, mag):
    """Outliers of every size over zero-weight columns, one per block and
    several in one block, at 1024 and 4096 columns (the row bound grows with
    the row, so the narrow rows are the harder case)."""
    for cols, seed in ((1024, 1), (4096, 2), (1024, 3)):
        rows = 512
        outs = [(37, mag), (300, -mag / 3), (301, mag / 7), (640, mag), (641, mag), (642, -mag)]
        outs += [(96 + i, mag * (1 - 0.1 * i)) for i in range(7)]   # seven in one block
        q, x = _case(fmt, rows, cols, outs, seed=fmt * 100 + seed + int(abs(np.log10(abs(mag)))))
        ref = O.gemv(fmt, q, x, rows, cols).astype(np.float64)
        bound = TOL * O.row_abs_sums(fmt, q, x, rows, cols)
        err = np.abs(digit_gemv(fmt, q, x, rows, cols) - ref)
        assert np.all(err <= bound), f"cols {cols}: worst err/bound {np.max(err / bound):.3f}"


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q5_0, O.IQ3_0])
def test_integer_path_alone_misses_the_bound_on_outliers(fmt):
    """Without the wide rule the 1e4 outliers break the bound on the rows that
    weigh them by zero: the inputs above do exercise the rule."""
    rows, cols = 512, 1024
    q, x = _case(fmt, rows, cols, [(37, 1e4), (640, 1e5)], seed=7 + fmt)
    ref = O.gemv(fmt, q, x, rows, cols).astype(np.float64)
    bound = TOL * O.row_abs_sums(fmt, q, x, rows, cols)
    err = np.abs(digit_gemv(fmt, q, x, rows, cols, wide_rule=False) - ref)
    assert np.any(err > bound)


def test_wide_rule_leaves_ordinary_vectors_alone():
    """N(0,1) vectors, SwiGLU activations and vectors with moderate (20x)
    spikes flag no block: the integer path keeps them.  SwiGLU activations at
    a large scale (half of a block is silu of a large negative gate: tiny,
    and spread over many decades) flag at most a block in a thousand; those
    take the exact fp32 path, which only costs time.  (A spike a few hundred
    times the block's typical value does flag its block.)"""
    rng = np.random.default_rng(3)
    flagged = blocks = 0
    with np.errstate(over="ignore"):
        for _ in range(20):
            g = rng.standard_normal(14336).astype(np.float32)
            u = rng.standard_normal(14336).astype(np.float32)
            act = (g / (1 + np.exp(-g)) * u).astype(np.float32)
            big = (40 * g / (1 + np.exp(-40 * g)) * 40 * u).astype(np.float32)
            spiky = rng.standard_normal(4096).astype(np.float32)
            spiky[rng.integers(0, 4096, 16)] *= 20
            for v in (g, act, spiky):
                assert not wide_blocks(v.reshape(-1, 32)).any()
            flagged += int(wide_blocks(big.reshape(-1, 32)).sum())
            blocks += big.size // 32
    assert flagged <= blocks // 1000, (flagged, blocks)


def test_wide_rule_edges():
    b = np.zeros((8, 32), np.float32)
    b[0, 0] = 1e4                           # one value, the rest zero: exact anyway
    b[1, 0], b[1, 1] = 1e4, 1.0             # one ordinary value keeps 7 bits: integer path
    b[2, 0], b[2, 1:] = 1e3, 1.0            # an outlier over 31 ordinary values: wide
    b[3, :16], b[3, 16:] = 1e4, 1.0         # half outliers: no longer "a few", integer path
    b[4, 0], b[4, 1:] = np.inf, 1.0         # not finite: NaN path, not wide
    b[5] = np.float32(2.0 ** -140)          # subnormal block: exact digits, not wide
    b[6, 0], b[6, 1] = 1e4, 3.0             # two values far apart: the small one keeps 12 bits
    b[7] = np.float32(1.0)                  # ordinary
    assert wide_blocks(b).tolist() == [False, False, True, False, False, False, False, False]
