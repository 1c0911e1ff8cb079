"""The RQF coefficient producer against the reference's own RQF module.

rqf_filter_two_tap_coefficients (through ops.filter_two_tap_coefficients, the
drop-in that install() binds to RQF.compute_two_tap_coefficients) is compared
with rqf_models/backbones/rqf/filter.py:RQF.compute_two_tap_coefficients
(:510-664) of the reference module itself, from its offline install in
baseline/_ref, over every branch: Euler / ZOH / FOH (FOH also
non-prospective), tau and gamma mode, prospective_tau (none, a scalar, a
per-filter tensor that needs a gradient), the dynamic gamma clamp, and the log
and sigmoid leaf parametrizations, with log_tau learned.

The oracle is the reference module converted to float64 (its own torch
expressions, run in double): outputs must agree to 1e-6 and every leaf
gradient (a fixed random complex cotangent on each output) to 1e-5, normwise,
the kernel computing in double from the same fp32 leaves.  Against the
reference's own fp32 run the outputs agree to the forward tolerance 1e-4 for
Euler and ZOH; FOH is held to 5e-4 there, because the reference evaluates
(e^a - 1 - a)/a^2 in fp32 with the cancellation of e^a - 1 - a just above its
Taylor threshold (|a| = 1e-3): its own fp32 result is up to ~1e-4 away from
its fp64 one.
"""

import copy
import itertools
import sys
import zlib
from pathlib import Path

import numpy as np
import pytest
import torch

from _util import FWD_TOL, assert_close

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
if not (REF / "rqf_models").exists():
    pytest.skip("reference install (baseline/_ref) absent", allow_module_level=True)
if str(REF) not in sys.path:
    sys.path.insert(0, str(REF))

F = 96
DT, TAU = 1.0 / 16000.0, 0.0003125


def _module(disc, space, clamp, seed, saturated=False):
    from rqf_models.backbones.rqf.filter import RQF

    kw = dict(num_filters=F, tau=TAU, dt=DT, learn_tau=True, discretization=disc,
              param_space=space, clamp_gamma=clamp)
    if space == "log":
        kw["seq_duration"] = 1.0
    else:
        kw.update(min_freq=1.0, max_freq=3000.0, min_gamma=0.01, max_gamma=0.9)
    r = RQF(**kw)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():  # leaves spread over the band, off any clamp boundary by chance
        r.log_tau.add_(0.1 * torch.randn(F, generator=g))
        if space == "log":
            r.log_theta.copy_(torch.empty(F).uniform_(np.log(0.01), np.log(6.0), generator=g))
            r.log_gamma.copy_(torch.empty(F).uniform_(1e-3, 0.999, generator=g).log())
        else:
            r.freq_param.copy_(2 * torch.randn(F, generator=g))
            r.gamma_param.copy_(2 * torch.randn(F, generator=g))
            if saturated:  # the reference's init when critical gamma exceeds max_gamma
                r.gamma_param[: F // 2] = torch.logit(torch.tensor(1 - 1e-6))
    return r


def _cases():
    for disc, space, mode, ptau, clamp in itertools.product(
            ("euler", "zoh", "foh"), ("log", "sigmoid"), ("tau", "gamma"),
            (None, "scalar", "vector"), (False, True)):
        yield disc, True, space, mode, ptau, clamp
    for space, clamp in itertools.product(("log", "sigmoid"), (False, True)):
        yield "foh", False, space, "tau", None, clamp


def _leaves(r):
    names = ["log_tau"] + (["log_theta", "log_gamma"] if r.param_space == "log"
                           else ["freq_param", "gamma_param"])
    return [getattr(r, n) for n in names]


def _run(fn, r, ptau, cots):
    for p in r.parameters():
        p.grad = None
    if ptau is not None and isinstance(ptau, torch.Tensor):
        ptau.grad = None
    outs = fn(ptau)
    loss = sum((g.conj() * o).real.sum() for g, o in zip(cots, outs))
    loss.backward()
    grads = [None if t.grad is None else t.grad.detach().clone() for t in _leaves(r)]
    if isinstance(ptau, torch.Tensor) and ptau.requires_grad:
        grads.append(ptau.grad.detach().clone())
    return [o.detach() for o in outs], grads


@pytest.mark.parametrize("disc,prospective,space,mode,ptau,clamp", list(_cases()))
def test_coefficients_match_reference_rqf(disc, prospective, space, mode, ptau, clamp):
    import prospective_rqf_b200 as rqf
    from prospective_rqf_b200 import ops

    rqf.uninstall()  # the fp32 comparison runs the reference's own expressions
    seed = zlib.crc32(repr((disc, prospective, space, mode, ptau, clamp)).encode()) % 1000
    r32 = _module(disc, space, clamp, seed).cuda()
    r64 = copy.deepcopy(r32).double()
    g = torch.Generator().manual_seed(seed + 1)
    cots = [torch.complex(torch.randn(F, generator=g), torch.randn(F, generator=g))
            for _ in range(3)]

    def tau_p(dtype):
        if ptau is None:
            return None
        if ptau == "scalar":
            return 0.0002
        v = torch.empty(F).uniform_(0.0, 0.0005, generator=torch.Generator().manual_seed(seed))
        return v.to("cuda", dtype).requires_grad_(True)

    ours, g_ours = _run(lambda p: ops.filter_two_tap_coefficients(r32, prospective, mode, p),
                        r32, tau_p(torch.float32), [c.cuda() for c in cots])
    ref64, g_ref = _run(lambda p: r64.compute_two_tap_coefficients(prospective, mode, p),
                        r64, tau_p(torch.float64), [c.cuda().to(torch.complex128) for c in cots])
    ref32 = [o.detach() for o in r32.compute_two_tap_coefficients(prospective, mode,
                                                                    tau_p(torch.float32))]

    for name, a, b, c in zip(("C1", "tap0", "tap1"), ours, ref64, ref32):
        assert a.dtype == c.dtype, f"{name}: dtype {a.dtype} vs the reference's {c.dtype}"
        a64 = a.cpu().numpy().astype(np.complex128)
        assert_close(a64, b.cpu().numpy(), 1e-6, f"{name} vs fp64 reference")
        assert_close(a64, c.cpu().numpy().astype(np.complex128),
                     5e-4 if disc == "foh" else FWD_TOL, f"{name} vs fp32 reference")
    assert len(g_ours) == len(g_ref)
    for i, (a, b) in enumerate(zip(g_ours, g_ref)):
        assert (a is None) == (b is None), f"gradient {i} presence differs"
        if a is not None:
            assert_close(a.cpu().numpy().astype(np.float64), b.cpu().numpy(), 1e-5,
                         f"leaf gradient {i}")


@pytest.mark.parametrize("disc", ["euler", "zoh", "foh"])
def test_saturated_sigmoid_leaves_match_fp64_reference(disc):
    """gamma_param at logit(1 - 1e-6), where the reference's init leaves it
    when critical damping exceeds max_gamma: the gradient through
    sig'(p) = s (1 - s) keeps its digits in double (this producer and the
    reference's fp64 run agree to 1e-5), while the reference's own fp32 run
    is several percent off there — reported, not asserted."""
    import prospective_rqf_b200 as rqf
    from prospective_rqf_b200 import ops

    rqf.uninstall()
    r32 = _module(disc, "sigmoid", False, 5, saturated=True).cuda()
    r64 = copy.deepcopy(r32).double()
    g = torch.Generator().manual_seed(6)
    cots = [torch.complex(torch.randn(F, generator=g), torch.randn(F, generator=g)).cuda()
            for _ in range(3)]
    _, g_ours = _run(lambda p: ops.filter_two_tap_coefficients(r32, True, "tau", p), r32, None,
                     cots)
    _, g_ref = _run(lambda p: r64.compute_two_tap_coefficients(True, "tau", p), r64, None,
                    [c.to(torch.complex128) for c in cots])
    _, g_ref32 = _run(lambda p: r32.compute_two_tap_coefficients(True, "tau", p), r32, None,
                      cots)
    for a, b, c in zip(g_ours, g_ref, g_ref32):
        if b is None:
            continue
        assert_close(a.cpu().numpy().astype(np.float64), b.cpu().numpy(), 1e-5, "leaf gradient")
        e32 = float((c.double() - b).abs().max() / b.abs().max())
        print(f"{disc}: the reference's fp32 leaf gradient vs its fp64 one: {e32:.2e}")


def test_install_routes_the_reference_module():
    import prospective_rqf_b200 as rqf
    from prospective_rqf_b200 import _timing

    r = _module("zoh", "log", False, 3).cuda()
    rqf.uninstall()
    want = [o.detach() for o in r.compute_two_tap_coefficients(True, "tau")]
    rqf.install()
    try:
        with _timing.KernelTimer() as timer:
            got = r.compute_two_tap_coefficients(True, "tau")
        assert "rqf_filter_two_tap_coefficients" in timer.summary()
        r64 = copy.deepcopy(r).double()  # float64 leaves keep the reference's own path
        assert r64.compute_two_tap_coefficients(True, "tau")[0].dtype == torch.complex128
    finally:
        rqf.uninstall()
    for a, b in zip(got, want):
        assert_close(a.detach().cpu().numpy(), b.cpu().numpy(), FWD_TOL, "installed")
