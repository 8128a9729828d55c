"""Helpers shared by the GPU parity tests."""
from __future__ import annotations

import numpy as np


def within(out, ref, tol: float) -> None:
    """|out - ref| <= tol * max(|ref|, 1), element-wise (the parity metric)."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    assert out.shape == ref.shape, (out.shape, ref.shape)
    assert np.isfinite(out).all(), "non-finite output"
    err = np.abs(out - ref)
    bound = tol * np.maximum(np.abs(ref), 1.0)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err / bound), err.shape)
        raise AssertionError(f"{bad.sum()} elements beyond tol {tol}: worst at {i} "
                             f"out={out[i]!r} ref={ref[i]!r} err={err[i]:.3e}")


def max_rel(out, ref) -> float:
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    return float((np.abs(out - ref) / np.maximum(np.abs(ref), 1.0)).max())
