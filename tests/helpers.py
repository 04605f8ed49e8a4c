"""Shared test helpers: the reference's compare() and scale-relative metrics."""
import numpy as np


def compare(got, want, abs_tol, rel_tol):
    """compare (test/helpers/tensors.ts:81-105): an element fails only when it
    exceeds BOTH the absolute and the relative tolerance. Returns
    (max_abs, max_rel, worst-8 list)."""
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    assert got.shape == want.shape, (got.shape, want.shape)
    abs_err = np.abs(got - want)
    rel_err = abs_err / np.maximum(1e-6, np.abs(want))
    bad = np.nonzero((abs_err > abs_tol) & (rel_err > rel_tol) | ~np.isfinite(got))[0]
    worst = sorted(bad, key=lambda i: -abs_err[i])[:8]
    return float(abs_err.max(initial=0)), float(rel_err.max(initial=0)), \
        [(int(i), float(got[i]), float(want[i])) for i in worst]


def scale_metrics(got, want):
    """(max_abs / max|want|, rel-L2) -- the per-layer tolerance metrics."""
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    scale = max(np.abs(want).max(initial=0), 1e-30)
    rel_l2 = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    return float(np.abs(got - want).max(initial=0) / scale), float(rel_l2)
