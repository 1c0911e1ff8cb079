"""numpy front end of the double-precision C oracle (oracle/rqf_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for tests/, __graft_entry__.smoke() and
the CPU baseline of bench.py.  Parity of these functions with the reference
is pinned by tests/test_oracle_golden.py against vectors generated from the
reference implementation (tests/golden/make_golden.py).

Layouts: "btf" = (batch, time, filters), "fbt" = (filters, batch, time).
All complex arrays are numpy complex128; inputs of other dtypes are converted.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "librqf_oracle.so"
_LIB = None

_LAYOUT = {"btf": 0, "fbt": 1}


def build(force: bool = False) -> Path:
    """Compile oracle/rqf_oracle.c with the system gcc (make)."""
    if force or not _LIB_PATH.exists():
        subprocess.run(["make", "-C", str(_HERE)], check=True, capture_output=True)
    return _LIB_PATH


def _lib():
    global _LIB
    if _LIB is None:
        build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        ci = ctypes.c_int
        lib.rqfo_two_tap_forward.argtypes = [ci, i64, i64, i64, p, p, p, p, p, ci, ci]
        lib.rqfo_two_tap_backward.argtypes = [ci, i64, i64, i64, p, p, p, p, p, ci, p, p, p, p, ci]
        lib.rqfo_tbptt_backward.argtypes = [ci, i64, i64, i64, p, p, p, p, p, ci, p, p, p, p, p, ci]
        lib.rqfo_two_tap_backward_masked.argtypes = [ci, i64, i64, i64, p, p, p, p, p, ci, p, p, p,
                                                     p, p, ci]
        lib.rqfo_two_tap_backward_masked.restype = ci
        lib.rqfo_max_threads.restype = ci
        for fn in (lib.rqfo_two_tap_forward, lib.rqfo_two_tap_backward, lib.rqfo_tbptt_backward):
            fn.restype = ci
        _LIB = lib
    return _LIB


def max_threads() -> int:
    return int(_lib().rqfo_max_threads())


def _c128(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a), dtype=np.complex128)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _threads(nthreads: int | None) -> int:
    if nthreads is None:
        return int(os.environ.get("RQF_ORACLE_THREADS", "0"))
    return int(nthreads)


def two_tap_forward(c1, tap0, tap1, x, layout: str = "btf", fuse_act: bool = False,
                    nthreads: int | None = None) -> np.ndarray:
    """y[t] = c1*y[t-1] + tap0*x[t] + tap1*x[t-1]; tap1=None gives the
    single-tap scan y = c1*y + c2*x (pass c2 as tap0)."""
    c1, tap0 = _c128(c1), _c128(tap0)
    tap1 = None if tap1 is None else _c128(tap1)
    x = _c128(x)
    y = np.empty_like(x)
    d0, d1, d2 = x.shape
    st = _lib().rqfo_two_tap_forward(_LAYOUT[layout], d0, d1, d2, _ptr(c1), _ptr(tap0),
                                     _ptr(tap1), _ptr(x), _ptr(y), int(fuse_act),
                                     _threads(nthreads))
    if st:
        raise RuntimeError("oracle forward failed")
    return y


def two_tap_backward(c1, tap0, tap1, x, gy, layout: str = "btf", fuse_act: bool = False,
                     nthreads: int | None = None, mask=None):
    """Full-BPTT VJP of two_tap_forward: returns (gx, gc1, gtap0, gtap1)
    (gtap1 is None when tap1 is None).  With fuse_act, `mask` (bool array of
    x.shape + (2,), [..., 0] for Re and [..., 1] for Im) overrides the sign
    test of split-ReLU'."""
    c1, tap0 = _c128(c1), _c128(tap0)
    tap1 = None if tap1 is None else _c128(tap1)
    x, gy = _c128(x), _c128(gy)
    gx = np.empty_like(x)
    nf = c1.shape[0]
    gc1 = np.zeros(nf, np.complex128)
    gt0 = np.zeros(nf, np.complex128)
    gt1 = None if tap1 is None else np.zeros(nf, np.complex128)
    d0, d1, d2 = x.shape
    m = None
    if mask is not None:
        m = np.ascontiguousarray(mask, dtype=np.uint8)
        if m.shape != x.shape + (2,):
            raise ValueError(f"mask must have shape {x.shape + (2,)}")
    st = _lib().rqfo_two_tap_backward_masked(_LAYOUT[layout], d0, d1, d2, _ptr(c1), _ptr(tap0),
                                             _ptr(tap1), _ptr(x), _ptr(gy), int(fuse_act),
                                             _ptr(m), _ptr(gx), _ptr(gc1), _ptr(gt0), _ptr(gt1),
                                             _threads(nthreads))
    if st:
        raise RuntimeError("oracle backward failed")
    return gx, gc1, gt0, gt1


def relu_mask_from_output(act) -> np.ndarray:
    """Split-ReLU decisions implied by a split-ReLU output (act > 0 per part)."""
    act = np.asarray(act)
    return np.stack([act.real > 0, act.imag > 0], axis=-1)


def mask_disagreement(mask, y_ref) -> float:
    """Largest |component| of the fp64 state where `mask` disagrees with its
    sign, relative to max |y_ref| (0 when they agree everywhere)."""
    ref = np.stack([y_ref.real > 0, y_ref.imag > 0], axis=-1)
    bad = mask != ref
    if not bad.any():
        return 0.0
    parts = np.stack([y_ref.real, y_ref.imag], axis=-1)
    return float(np.max(np.abs(parts[bad])) / max(np.max(np.abs(parts)), 1e-300))


def tbptt_backward(c1, tap0, tap1, x, gy, layout: str = "btf", fuse_act: bool = False,
                   nthreads: int | None = None):
    """TBPTT(1) surrogate VJP: returns (gz, gzw, gc1, gtap0, gtap1)."""
    c1, tap0, tap1 = _c128(c1), _c128(tap0), _c128(tap1)
    x, gy = _c128(x), _c128(gy)
    gz = np.empty_like(x)
    gzw = np.empty_like(x)
    nf = c1.shape[0]
    gc1, gt0, gt1 = (np.zeros(nf, np.complex128) for _ in range(3))
    d0, d1, d2 = x.shape
    st = _lib().rqfo_tbptt_backward(_LAYOUT[layout], d0, d1, d2, _ptr(c1), _ptr(tap0),
                                    _ptr(tap1), _ptr(x), _ptr(gy), int(fuse_act), _ptr(gz),
                                    _ptr(gzw), _ptr(gc1), _ptr(gt0), _ptr(gt1),
                                    _threads(nthreads))
    if st:
        raise RuntimeError("oracle tbptt backward failed")
    return gz, gzw, gc1, gt0, gt1


# --- convenience wrappers named after the reference callables -------------

def chunked_scan(c1, c2, u):
    """Forward of scan.py:sequential_scan / _triton_chunked_scan, (B,T,F)."""
    return two_tap_forward(c1, c2, None, u, "btf")


def chunked_scan_backward(c1, c2, u, gy):
    """(gc1, gc2, gu) of chunked_scan_kernel.py:_chunked_scan_backward_raw."""
    gu, gc1, gc2, _ = two_tap_backward(c1, c2, None, u, gy, "btf")
    return gc1, gc2, gu
