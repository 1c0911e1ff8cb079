"""Shared helpers for the parity tests."""

from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"

# The benchmark's stated tolerances (fp32 kernels against the fp64 oracle):
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


# Element-wise relative error with a floor: max_i |a_i - b_i| / (|b_i| + f),
# f = ELEM_FLOOR * max|b|.  Elements far below the tensor's scale (decayed
# states, small gradients) are held to a relative bound instead of hiding under
# the normwise one; the floor keeps exact zeros of b meaningful.
ELEM_FLOOR = 1e-3
FWD_ELEM_TOL = 1e-2
GRAD_ELEM_TOL = 5e-2


def elem_rel_err(a, b, floor: float = ELEM_FLOOR) -> float:
    a = np.asarray(a)
    b = np.asarray(b)
    if a.shape != b.shape:
        raise AssertionError(f"shape mismatch {a.shape} vs {b.shape}")
    if not a.size:
        return 0.0
    mag = np.abs(b)
    f = floor * float(np.max(mag))
    if f == 0.0:
        return float(np.max(np.abs(a - b)))
    return float(np.max(np.abs(a - b) / (mag + f)))


def assert_close(a, b, tol, what="", elem_tol=None):
    """Normwise bound `tol`; the element-wise error (floor ELEM_FLOOR) is
    reported beside it and, when `elem_tol` is given, bounded too."""
    e = rel_err(a, b)
    ee = elem_rel_err(a, b)
    assert e <= tol, (f"{what}: normwise max relative error {e:.3e} > {tol:.1e} "
                      f"(element-wise {ee:.3e})")
    if elem_tol is not None:
        assert ee <= elem_tol, (f"{what}: element-wise relative error {ee:.3e} > "
                                f"{elem_tol:.1e} (floor {ELEM_FLOOR:g} x max; normwise {e:.3e})")
    return e, ee


def golden(name: str):
    return np.load(GOLDEN / f"{name}.npz")
