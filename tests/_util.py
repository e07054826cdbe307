"""Shared test helpers: the parity bound and seeded input builders."""
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent

# GEMV / MoE fp32 parity bound: max |err| <= TOL * sum_l |w_l x_l| per row.
TOL = 1e-5


def assert_rows_within(actual, reference, abs_sums, tol=TOL, what=""):
    a = np.asarray(actual, np.float64).reshape(-1)
    r = np.asarray(reference, np.float64).reshape(-1)
    s = np.asarray(abs_sums, np.float64).reshape(-1)
    assert a.shape == r.shape == s.shape, (a.shape, r.shape, s.shape)
    err = np.abs(a - r)
    bound = tol * s
    bad = np.nonzero(err > bound)[0]
    if bad.size:
        i = bad[0]
        raise AssertionError(
            f"{what}: {bad.size} rows exceed {tol}*sum|w*x|; first row {i}: "
            f"actual={a[i]!r} reference={r[i]!r} err={err[i]:.3e} bound={bound[i]:.3e}")
    return float(np.max(err / np.maximum(s, 1e-300))) if s.size else 0.0


def header_functions():
    """Names of every function declared in include/*.h."""
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(?:int|void|size_t|const char\s*\*)\s+\*?\s*(objb_\w+)\s*\(", text):
            names.append(m.group(1))
    return sorted(set(names))
