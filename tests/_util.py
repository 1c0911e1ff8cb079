"""Shared helpers for the parity tests."""

from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"

# BASELINE tolerances (fp32 kernels against the fp64 oracle):
FWD_TOL = 1e-4   # forward: max |a - b| / max |b|
GRAD_TOL = 1e-3  # gradients: max |a - b| / max |b|


def rel_err(a, b) -> float:
    """Normwise max relative error max|a-b| / max|b| (0 when both are 0)."""
    a = np.asarray(a)
    b = np.asarray(b)
    if a.shape != b.shape:
        raise AssertionError(f"shape mismatch {a.shape} vs {b.shape}")
    denom = float(np.max(np.abs(b))) if b.size else 0.0
    num = float(np.max(np.abs(a - b))) if a.size else 0.0
    if denom == 0.0:
        return num
    return num / denom


def assert_close(a, b, tol, what=""):
    e = rel_err(a, b)
    assert e <= tol, f"{what}: normwise max relative error {e:.3e} > {tol:.1e}"


def golden(name: str):
    return np.load(GOLDEN / f"{name}.npz")
