"""Shared helpers for the parity tests."""
import numpy as np

# Tolerance of the FP32 aggregation: the path's target is a maximum relative
# error of 1e-5 with FP32 accumulation.  Summation order differs from the reference
# for split rows (atomic merge order) and for single-row tasks whose nonzeros
# are spread over lane groups, so the bound is relative to the condition of
# each output element: |gpu - ref64| <= REL_TOL * max(|ref64|, cond), where
# ref64 is the exact (double) mean and cond = (1/deg) * sum |a_ij * x_jk|.
REL_TOL = 1e-5


def rel_errors(out, ref64, cond):
    err = np.abs(out.astype(np.float64) - ref64)
    scale = np.maximum(np.abs(ref64), cond)
    with np.errstate(divide="ignore", invalid="ignore"):
        rel = np.where(scale > 0, err / scale, np.where(err > 0, np.inf, 0.0))
    return rel


def assert_mean_close(out, ref64, cond, tol=REL_TOL, what=""):
    rel = rel_errors(out, ref64, cond)
    worst = float(rel.max()) if rel.size else 0.0
    assert worst <= tol, f"{what}: max condition-relative error {worst:.3e} > {tol:.0e}"
    return worst


def random_csr(rng, n, maxdeg, n_cols=None, p_zero=0.1, hubs=1, hub_factor=7, values="normal"):
    n_cols = n if n_cols is None else n_cols
    deg = rng.integers(0, maxdeg + 1, n)
    deg[rng.random(n) < p_zero] = 0
    for _ in range(hubs if n > 3 else 0):
        deg[rng.integers(0, n)] = maxdeg * hub_factor
    rowoff = np.zeros(n + 1, np.int64)
    np.cumsum(deg, out=rowoff[1:])
    col = rng.integers(0, n_cols, rowoff[-1]).astype(np.int32)
    if values == "ones":
        val = np.ones(rowoff[-1], np.float32)
    else:
        val = rng.standard_normal(rowoff[-1]).astype(np.float32)
    return rowoff.astype(np.int32), col, val


def sorted_rowoff_from_degrees(degrees):
    d = np.sort(np.asarray(degrees, np.int64))
    ro = np.zeros(len(d) + 1, np.int64)
    np.cumsum(d, out=ro[1:])
    return ro.astype(np.int32)
