"""Pin the numpy selective-scan oracle (oracle/selective.py) to the
reference: tests/golden/selective_*.npz hold outputs and gradients of the
reference's reference_layer_scan (selective_scan.py:71-104) in fp64 with
autograd, on inputs built by the reference's own SelectiveController.  CPU."""

import numpy as np
import pytest

from _util import GOLDEN, assert_close, golden
from oracle import selective

CASES = sorted(int(p.stem.split("_")[1]) for p in GOLDEN.glob("selective_*.npz"))
TOL = 1e-9


def load(i):
    g = golden(f"selective_{i}")
    z = g["z"]
    F, B, T = z.shape
    opt = selective.options(g["options"])

    def logits(k, n):
        a = g[k]
        return a if a.size else np.zeros((n, B, T))

    ins = dict(gl=logits("gamma_logits", F), dl=logits("warp_logits", 0),
               wl=logits("write_logits", F), bias=g["bias"], theta=g["theta"],
               groups=g["groups"], lo=g["minimum"], span=g["span"], step=g["step"],
               horizon=g["horizon"], th_lo=g["theta_minimum"], th_hi=g["theta_maximum"], opt=opt)
    return g, z, ins, bool(g["truncated"])


@pytest.mark.parametrize("i", CASES)
def test_selective_oracle_matches_reference(i):
    g, z, ins, truncated = load(i)
    y, co = selective.forward(z, **ins)
    assert_close(y, g["raw"], TOL, "raw")
    act = np.maximum(y.real, 0) + 1j * np.maximum(y.imag, 0)
    assert_close(act, g["act"], TOL, "act")
    dz, dzw, dG, dD, dW, dbias, dtheta = selective.backward(
        z, y, co, g["gy"], g["gx"], truncated=truncated, **ins)
    assert_close(dz, g["dz"], TOL, "dz")
    F = z.shape[0]
    dweight = dzw.reshape(F, -1) @ z.reshape(F, -1).conj().T
    assert_close(dweight, g["dweight"], TOL, "dweight (lag cotangent)")
    opt = ins["opt"]
    if opt[0]:
        assert_close(dG, g["dG"], TOL, "dG")
    if opt[1]:
        assert_close(dD, g["dD"], TOL, "dD (group-reduced)")
    if opt[2]:
        assert_close(dW, g["dW"], TOL, "dW")
    assert_close(dbias, g["dbias"], TOL, "dbias")
    assert_close(dtheta, g["dtheta"], TOL, "dtheta")
