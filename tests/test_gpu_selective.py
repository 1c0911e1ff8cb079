"""GPU parity of the selective scan kernels (through the C ABI) against the
reference's golden vectors and the pinned fp64 numpy oracle.  Tolerances:
forward normwise max relative error <= 1e-4, gradients <= 1e-3."""

import numpy as np
import pytest
import torch

from _util import FWD_TOL, GOLDEN, GRAD_TOL, assert_close, golden
from oracle import oracle as core_oracle
from oracle import selective

pytestmark = pytest.mark.gpu

CASES = sorted(int(p.stem.split("_")[1]) for p in GOLDEN.glob("selective_*.npz"))
MASK_EDGE = 1e-4


@pytest.fixture(scope="module", autouse=True)
def _device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import prospective_rqf_b200 as rqf

    rqf.read_device_error(clear=True)
    yield
    rqf.check_device_errors()


def rqf():
    import prospective_rqf_b200

    return prospective_rqf_b200


def cuda(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dtype)


def host(t):
    return None if t is None else t.detach().cpu().numpy()


def as_inputs(d, opt, B, T):
    """SelectiveScanInputs-like 13-tuple of device tensors from numpy arrays."""
    F = d["bias"].shape[0]

    def logits(a, n):
        return cuda(a if a.size else np.zeros((n, B, T)), torch.float32)

    return (logits(d["gl"], 0), logits(d["dl"], 0), logits(d["wl"], 0),
            cuda(d["bias"], torch.float32), cuda(d["theta"], torch.float32),
            cuda(d["groups"], torch.int64) if d["groups"].size else None,
            cuda(d["lo"], torch.float32), cuda(d["span"], torch.float32),
            cuda(d["step"], torch.float32), cuda(d["horizon"], torch.float32),
            cuda(d["th_lo"], torch.float32), cuda(d["th_hi"], torch.float32), opt)


def run_kernel(z, d, opt, gy, gx, truncated):
    F, B, T = z.shape
    inputs = as_inputs(d, opt, B, T)
    zt = cuda(z, torch.complex64)
    raw, act, entries = rqf().selective_forward(zt, inputs, True, True, None)
    out = rqf().selective_backward(zt, inputs, entries, cuda(gy, torch.complex64),
                                   cuda(gx, torch.complex64), True, truncated, None)
    return host(raw), host(act), [host(o) for o in out]


def check(z, d, opt, gy, gx, truncated, ref_fwd, ref_bwd, use_kernel_mask):
    raw, act, (dz, dzw, dG, dD, dW, dbias, dtheta) = run_kernel(z, d, opt, gy, gx, truncated)
    assert_close(raw, ref_fwd[0], FWD_TOL, "raw")
    assert_close(act, ref_fwd[1], FWD_TOL, "act")
    if use_kernel_mask:
        mask = core_oracle.relu_mask_from_output(act)
        edge = core_oracle.mask_disagreement(mask, ref_fwd[0])
        assert edge < MASK_EDGE, f"split-ReLU decision differs at |state| = {edge:.2e} max"
        ref_bwd = ref_bwd(mask)
    rdz, rdzw, rdG, rdD, rdW, rdbias, rdtheta = ref_bwd
    assert_close(dz, rdz, GRAD_TOL, "dz")
    assert_close(dzw, rdzw, GRAD_TOL, "dzw")
    if opt[0]:
        assert_close(dG, rdG, GRAD_TOL, "dG")
    if opt[1]:
        assert_close(dD, rdD, GRAD_TOL, "dD (group)")
    if opt[2]:
        assert_close(dW, rdW, GRAD_TOL, "dW")
    assert_close(dbias, rdbias, GRAD_TOL, "dbias")
    assert_close(dtheta, rdtheta, GRAD_TOL, "dtheta")


@pytest.mark.parametrize("i", CASES)
def test_selective_matches_reference_goldens(i):
    g = golden(f"selective_{i}")
    z = g["z"]
    F, B, T = z.shape
    opt = selective.options(g["options"])
    d = dict(gl=g["gamma_logits"], dl=g["warp_logits"], wl=g["write_logits"], bias=g["bias"],
             theta=g["theta"], groups=g["groups"], lo=g["minimum"], span=g["span"],
             step=g["step"], horizon=g["horizon"], th_lo=g["theta_minimum"],
             th_hi=g["theta_maximum"])
    truncated = bool(g["truncated"])
    raw, act, (dz, dzw, dG, dD, dW, dbias, dtheta) = run_kernel(z, d, opt, g["gy"], g["gx"],
                                                                truncated)
    assert_close(raw, g["raw"], FWD_TOL, "raw")
    assert_close(act, g["act"], FWD_TOL, "act")
    assert_close(dz, g["dz"], GRAD_TOL, "dz")
    dweight = dzw.astype(np.complex128).reshape(F, -1) @ z.reshape(F, -1).conj().T
    assert_close(dweight, g["dweight"], GRAD_TOL, "dweight (lag cotangent)")
    if opt[0]:
        assert_close(dG, g["dG"], GRAD_TOL, "dG")
    if opt[1]:
        assert_close(dD, g["dD"], GRAD_TOL, "dD")
    if opt[2]:
        assert_close(dW, g["dW"], GRAD_TOL, "dW")
    assert_close(dbias, g["dbias"], GRAD_TOL, "dbias")
    assert_close(dtheta, g["dtheta"], GRAD_TOL, "dtheta")


def random_case(rng, F, B, T, opt, ngroups=3):
    """Seeded inputs with the ranges the reference's controller produces
    (resonant recipe: gamma band ~[0, 1], theta = omega*tau, h = dt/tau)."""
    c32 = lambda a: np.asarray(a, np.float32).astype(np.float64)  # noqa: E731
    theta = c32(rng.uniform(0.05, 2.5, F))
    d = dict(
        gl=c32(rng.standard_normal((F, B, T))) if opt[0] else np.zeros(0),
        dl=c32(rng.standard_normal((ngroups, B, T))) if opt[1] else np.zeros(0),
        wl=c32(rng.standard_normal((F, B, T))) if opt[2] else np.zeros(0),
        # bias is logit(resting gamma) for the sigmoid link, log(gamma) for the
        # log-shift link, and gamma itself without gamma control (gamma in (0, 1))
        bias=c32(rng.standard_normal(F) if opt[0] and not opt[3]
                 else np.log(rng.uniform(0.05, 0.5, F)) if opt[0]
                 else rng.uniform(0.05, 0.9, F)),
        theta=theta, groups=rng.integers(0, ngroups, F) if opt[1] else np.zeros(0, np.int64),
        lo=c32(np.full(F, 1e-6)), span=c32(np.full(F, 1 - 2e-6)), step=c32(np.full(F, 0.2)),
        horizon=c32(np.full(F, 1.0)), th_lo=c32(theta * 0.4), th_hi=c32(theta * 1.6))
    if opt[1]:
        d["groups"][:ngroups] = np.arange(ngroups)
    z = rng.standard_normal((F, B, T)) + 1j * rng.standard_normal((F, B, T))
    z = z.astype(np.complex64).astype(np.complex128)
    gy = rng.standard_normal((F, B, T)) + 1j * rng.standard_normal((F, B, T))
    gx = rng.standard_normal((F, B, T)) + 1j * rng.standard_normal((F, B, T))
    return z, d, gy.astype(np.complex64).astype(np.complex128), \
        gx.astype(np.complex64).astype(np.complex128)


OPTS = {
    # (has_gamma, has_warp, has_write, log_shift, gscale, wscale, prospective,
    #  gamma_horizon, write_sigmoid, write_max, write_bias, bound_warp)
    "gamma_sigmoid": (True, False, False, False, 0.223, 0.223, True, False, False, 2.0, 0.0,
                      False),
    "all_grouped": (True, True, True, False, 0.223, 0.223, True, False, True, 2.0, 0.0, True),
    "logshift_write": (True, False, True, True, 0.223, 0.223, True, True, True, 2.0, 0.0, False),
    "warp_only_plain": (False, True, False, False, 0.223, 0.223, False, False, False, 2.0, 0.0,
                        False),
}


@pytest.mark.parametrize("T", [1, 2, 1023, 1024, 1025, 3000])
@pytest.mark.parametrize("name", sorted(OPTS))
@pytest.mark.parametrize("truncated", [False, True])
def test_selective_vs_oracle(T, name, truncated):
    rng = np.random.default_rng(T * 7 + len(name) + int(truncated))
    opt = OPTS[name]
    F, B = 6, 3
    z, d, gy, gx = random_case(rng, F, B, T, opt)
    ins = dict(gl=d["gl"] if d["gl"].size else np.zeros((F, B, T)),
               dl=d["dl"] if d["dl"].size else np.zeros((1, B, T)),
               wl=d["wl"] if d["wl"].size else np.zeros((F, B, T)), bias=d["bias"],
               theta=d["theta"], groups=d["groups"], lo=d["lo"], span=d["span"], step=d["step"],
               horizon=d["horizon"], th_lo=d["th_lo"], th_hi=d["th_hi"], opt=opt)
    y, co = selective.forward(z, **ins)
    act = np.maximum(y.real, 0) + 1j * np.maximum(y.imag, 0)

    def ref_bwd(mask):
        return selective.backward(z, y, co, gy, gx, truncated=truncated, mask=mask, **ins)

    check(z, d, opt, gy, gx, truncated, (y, act), ref_bwd, use_kernel_mask=True)


def test_selective_config3_rows():
    """Config-3 sequence length (T=4096) and width, on a 64-channel slice:
    sigmoid gamma, sigmoid write, 8-group frequency warp, prospective."""
    rng = np.random.default_rng(3)
    opt = (True, True, True, False, 0.223, 0.223, True, False, True, 2.0, 0.0, True)
    F, B, T = 64, 8, 4096
    z, d, gy, gx = random_case(rng, F, B, T, opt, ngroups=8)
    ins = dict(gl=d["gl"], dl=d["dl"], wl=d["wl"], bias=d["bias"], theta=d["theta"],
               groups=d["groups"], lo=d["lo"], span=d["span"], step=d["step"],
               horizon=d["horizon"], th_lo=d["th_lo"], th_hi=d["th_hi"], opt=opt)
    y, co = selective.forward(z, **ins)
    act = np.maximum(y.real, 0) + 1j * np.maximum(y.imag, 0)

    def ref_bwd(mask):
        return selective.backward(z, y, co, gy, gx, truncated=False, mask=mask, **ins)

    check(z, d, opt, gy, gx, False, (y, act), ref_bwd, use_kernel_mask=True)


# ------------------------------------------------------ bf16 storage mode
# Tolerances of the bf16 storage mode (no pinned parity: the reference has no
# such mode).  Stored bf16 values carry half a bf16 ulp of rounding, 2^-9 of
# their magnitude, so raw / act and the logit cotangents are held to 5e-3
# normwise against the fp64 oracle; dz, dzw, dbias and dtheta stay fp32 and keep
# the fp32 bounds.  Against the fp32 kernel on the same (bf16-valued) logits
# the mode must agree to the bf16 rounding of the fp32 kernel's outputs.
BF16_TOL = 5e-3


def _bf16_values(d):
    """The logits rounded to bf16 (both modes and the oracle see these values)."""
    out = dict(d)
    for k in ("gl", "dl", "wl"):
        if d[k].size:
            out[k] = torch.from_numpy(d[k]).to(torch.bfloat16).to(torch.float64).numpy()
    return out


@pytest.mark.parametrize("T", [1, 1023, 1025, 4096])
@pytest.mark.parametrize("truncated", [False, True])
def test_selective_bf16_storage_mode(T, truncated):
    from prospective_rqf_b200 import ops

    rng = np.random.default_rng(500 + T + int(truncated))
    opt = (True, True, True, False, 0.223, 0.223, True, False, True, 2.0, 0.0, True)
    F, B = 24, 4
    z, d, gy, gx = random_case(rng, F, B, T, opt, ngroups=4)
    d = _bf16_values(d)
    inputs = as_inputs(d, opt, B, T)
    zt = cuda(z, torch.complex64)
    raw16, act16, ent16 = ops.selective_forward_bf16(zt, inputs, True, True)
    out16 = ops.selective_backward_bf16(zt, inputs, ent16, cuda(gy, torch.complex64),
                                        cuda(gx, torch.complex64), True, truncated)
    raw32, act32, ent32 = ops.selective_forward(zt, inputs, True, True)
    out32 = ops.selective_backward(zt, inputs, ent32, cuda(gy, torch.complex64),
                                   cuda(gx, torch.complex64), True, truncated)

    def c16(t):  # (F,B,T,2) bf16 -> complex128
        a = t.float().cpu().numpy().astype(np.float64)
        return a[..., 0] + 1j * a[..., 1]

    def as_bf16_pairs(t):
        return c16(torch.view_as_real(t).to(torch.bfloat16))

    # same arithmetic: the bf16 outputs are the fp32 kernel's, rounded once
    assert np.array_equal(c16(raw16), as_bf16_pairs(raw32))
    assert np.array_equal(c16(act16), as_bf16_pairs(act32))
    for i, name in ((0, "dz"), (1, "dzw"), (5, "dbias"), (6, "dtheta")):
        assert torch.equal(out16[i], out32[i]), f"{name} differs from the fp32 mode"
    for i, name in ((2, "dG"), (3, "dD"), (4, "dW")):
        if out32[i] is not None:
            assert torch.equal(out16[i], out32[i].to(torch.bfloat16)), f"{name} rounding differs"

    # against the fp64 oracle, with the stated bf16-storage tolerance
    ins = dict(gl=d["gl"], dl=d["dl"], wl=d["wl"], bias=d["bias"], theta=d["theta"],
               groups=d["groups"], lo=d["lo"], span=d["span"], step=d["step"],
               horizon=d["horizon"], th_lo=d["th_lo"], th_hi=d["th_hi"], opt=opt)
    y, co = selective.forward(z, **ins)
    act = np.maximum(y.real, 0) + 1j * np.maximum(y.imag, 0)
    assert_close(c16(raw16), y, BF16_TOL, "raw (bf16)")
    assert_close(c16(act16), act, BF16_TOL, "act (bf16)")
    mask = core_oracle.relu_mask_from_output(c16(act16))
    assert core_oracle.mask_disagreement(mask, y) < MASK_EDGE
    rdz, rdzw, rdG, rdD, rdW, rdbias, rdtheta = selective.backward(
        z, y, co, gy, gx, truncated=truncated, mask=mask, **ins)
    dz, dzw, dG, dD, dW, dbias, dtheta = (None if t is None else t.float().cpu().numpy()
                                          if t.dtype == torch.bfloat16 else host(t)
                                          for t in out16)
    assert_close(dz, rdz, GRAD_TOL, "dz")
    assert_close(dzw, rdzw, GRAD_TOL, "dzw")
    assert_close(dG, rdG, BF16_TOL, "dG (bf16)")
    assert_close(dD, rdD, BF16_TOL, "dD (bf16)")
    assert_close(dW, rdW, BF16_TOL, "dW (bf16)")
    assert_close(dbias, rdbias, GRAD_TOL, "dbias")
    assert_close(dtheta, rdtheta, GRAD_TOL, "dtheta")
