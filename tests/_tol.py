"""Tolerance helpers shared by the parity tests."""

import numpy as np


def assert_rel_close(actual, ref, rtol, floor_frac=1e-3, what=""):
    """Elementwise |a - r| <= rtol * max(|r|, floor_frac * max|r|).

    Elementwise relative error is ill-posed where the reference is ~0, so the bound uses a
    floor of floor_frac of the largest reference magnitude.
    """
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    assert a.shape == r.shape, (a.shape, r.shape)
    scale = np.maximum(np.abs(r), floor_frac * max(np.max(np.abs(r)), 1e-30))
    err = np.abs(a - r) / scale
    worst = float(np.max(err)) if err.size else 0.0
    assert worst <= rtol, f"{what} max scaled error {worst:.3e} > {rtol:.1e}"
    return worst


def assert_norm_close(actual, ref, rtol, what=""):
    """Max-normalized error: max |a - r| <= rtol * max |r| (the fp32-path check: fp32
    accumulation error is relative to the magnitude of the terms, not of each result)."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    assert a.shape == r.shape, (a.shape, r.shape)
    worst = float(np.max(np.abs(a - r)) / max(np.max(np.abs(r)), 1e-30))
    assert worst <= rtol, f"{what} max-normalized error {worst:.3e} > {rtol:.1e}"
    return worst
