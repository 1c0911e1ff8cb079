"""Parity at the benchmark configurations' full sizes, against the fp64 oracle.

Each test runs one full-size launch pair (forward and backward) of the shape a
configuration times, then checks it against the oracle:

* (F,B,T) two-tap scans, config 2 (F=128, B=16, T=16000) and the config-5
  layer (F=256, B=32, T=16000): split-ReLU with recompute (fbt_recompute_scan,
  pure.py:234-238) and the raw last block (fbt_prospective_scan), and the
  config-5 TBPTT(1) layer.  Every row is checked: the oracle runs over all
  rows a few filters at a time (rows are independent), so the per-filter
  coefficient gradients, sums over all B*T samples of a filter, are checked
  whole.  Coefficients come from this backend's own coefficient producer on
  the paper recipe's leaves (log-uniform theta band, critical gamma), so the
  poles include the slowest ones the model trains with (|C1| = 1 - 4e-4).
* (B,T,F) scans of config 4: the S4-RQF two-tap shape (B=16, T=16384, F=64)
  and the P-S5 plain shape (B=16, T=16384, F=32), under both kernel families.
* the selective scan of config 3 (F=256, B=32, T=4096, 8 frequency-warp
  groups, sigmoid gamma and write, prospective): the full launch, checked on
  the filters of two whole groups (their group cotangent dD sums over exactly
  those filters), every batch row and time step.
* the rank-1 first block of configs 2 and 5, against the general first block
  on the same inputs (full BPTT and TBPTT(1)).

Bounds: forward normwise max relative error <= 1e-4, gradients <= 1e-3; the
element-wise relative error with a floor of 1e-3 x max|ref| is bounded beside
it (1e-2 forward, 5e-2 gradients).  Split-ReLU decisions: the oracle VJP is
evaluated with the kernel's own decisions, which must differ from fp64 only
where |state| < 1e-4 x max.
"""

import math

import numpy as np
import pytest
import torch

from _util import FWD_ELEM_TOL, FWD_TOL, GRAD_ELEM_TOL, GRAD_TOL, assert_close
from oracle import oracle

pytestmark = pytest.mark.gpu

MASK_EDGE = 1e-4
DT, TAU = 1.0 / 16000.0, 0.0003125


@pytest.fixture(scope="module", autouse=True)
def _device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import prospective_rqf_b200 as rqf

    rqf.read_device_error(clear=True)
    yield
    rqf.check_device_errors()


def _h(t):
    return t.detach().cpu().numpy().astype(np.complex128)


def _model_coefficients(F, seed):
    from prospective_rqf_b200.encoder import RQFCoefficients

    r = RQFCoefficients(F, DT, TAU, 1.0, generator=torch.Generator().manual_seed(seed)).cuda()
    with torch.no_grad():
        return [t.detach().contiguous() for t in r.two_tap()]


class _Acc:
    """Worst normwise and element-wise errors over chunks of rows."""

    def __init__(self):
        self.worst = {}

    def add(self, name, a, b, tol, elem_tol):
        e, ee = assert_close(a, b, tol, name, elem_tol=elem_tol)
        w = self.worst.get(name, (0.0, 0.0))
        self.worst[name] = (max(w[0], e), max(w[1], ee))


def _check_fbt_rows(c1, t0, t1, z, gy, y, gz, gc1, gt0, gt1, fuse, tbptt=False, gzw=None):
    """Oracle over all rows, CHUNK filters at a time; returns the worst errors."""
    F, B, T = z.shape
    chunk = max(1, (1 << 23) // (B * T))  # ~8 M samples per oracle call
    c1h, t0h, t1h = _h(c1), _h(t0), _h(t1)
    acc = _Acc()
    sums = np.zeros((3, F), np.complex128)
    for f0 in range(0, F, chunk):
        sl = slice(f0, min(F, f0 + chunk))
        zc, gyc, yc = _h(z[sl]), _h(gy[sl]), _h(y[sl])
        args = (c1h[sl], t0h[sl], t1h[sl], zc)
        y_ref = oracle.two_tap_forward(*args, "fbt", fuse_act=fuse)
        acc.add("y", yc, y_ref, FWD_TOL, FWD_ELEM_TOL)
        mask = None
        if fuse:
            mask = oracle.relu_mask_from_output(yc)
            raw_ref = oracle.two_tap_forward(*args, "fbt", fuse_act=False)
            edge = oracle.mask_disagreement(mask, raw_ref)
            assert edge < MASK_EDGE, f"split-ReLU decision differs at |state| = {edge:.2e} max"
            del raw_ref
        if tbptt:
            g_ref = gyc
            if fuse:
                g_ref = (np.where(mask[..., 0], gyc.real, 0.0)
                         + 1j * np.where(mask[..., 1], gyc.imag, 0.0))
            gz_ref, gzw_ref, a, b, c = oracle.tbptt_backward(*args, g_ref, "fbt", fuse_act=False)
            acc.add("gzw", _h(gzw[sl]), gzw_ref, GRAD_TOL, GRAD_ELEM_TOL)
        else:
            gz_ref, a, b, c = oracle.two_tap_backward(*args, gyc, "fbt", fuse_act=fuse,
                                                      mask=mask)
        acc.add("gz", _h(gz[sl]), gz_ref, GRAD_TOL, GRAD_ELEM_TOL)
        sums[0, sl], sums[1, sl], sums[2, sl] = a, b, c
    for name, got, ref in zip(("gc1", "gtap0", "gtap1"), (gc1, gt0, gt1), sums):
        acc.add(name, _h(got), ref, GRAD_TOL, GRAD_ELEM_TOL)
    print({k: f"{v[0]:.2e} / {v[1]:.2e}" for k, v in acc.worst.items()})
    return acc.worst


@pytest.mark.parametrize("F,B", [(128, 16), (256, 32)], ids=["config2", "config5-layer"])
@pytest.mark.parametrize("fuse", [True, False], ids=["split-relu", "raw"])
def test_fbt_full_size_all_rows_vs_oracle(F, B, fuse):
    import prospective_rqf_b200 as rqf

    T = 16000
    c1, t0, t1 = (t.requires_grad_(True) for t in _model_coefficients(F, seed=F + B))
    gen = torch.Generator(device="cuda").manual_seed(F * B)
    z = torch.randn(F, B, T, dtype=torch.complex64, device="cuda", generator=gen)
    gy = torch.randn(F, B, T, dtype=torch.complex64, device="cuda", generator=gen)
    z.requires_grad_(True)
    y = rqf.fbt_recompute_scan(c1, t0, t1, z) if fuse else rqf.fbt_prospective_scan(
        c1, t0, t1, z, False)
    gz, gc1, gt0, gt1 = torch.autograd.grad(y, (z, c1, t0, t1), gy)
    _check_fbt_rows(c1, t0, t1, z, gy, y, gz, gc1, gt0, gt1, fuse)


def test_fbt_tbptt1_config5_layer_all_rows_vs_oracle():
    import prospective_rqf_b200 as rqf

    F, B, T = 256, 32, 16000
    c1, t0, t1 = (t.requires_grad_(True) for t in _model_coefficients(F, seed=7))
    gen = torch.Generator(device="cuda").manual_seed(17)
    z = torch.randn(F, B, T, dtype=torch.complex64, device="cuda", generator=gen)
    gy = torch.randn(F, B, T, dtype=torch.complex64, device="cuda", generator=gen)
    lag = z.clone().requires_grad_(True)
    z.requires_grad_(True)
    y = rqf.tbptt1_two_tap_scan(z, c1, t0, t1, delayed_u=lag, layout="fbt", fuse_act=True)
    gz, gzw, gc1, gt0, gt1 = torch.autograd.grad(y, (z, lag, c1, t0, t1), gy)
    _check_fbt_rows(c1, t0, t1, z, gy, y, gz, gc1, gt0, gt1, True, tbptt=True, gzw=gzw)


@pytest.fixture(params=[1, 2], ids=["streaming", "resident"])
def btf_path(request):
    """Runs a (B,T,F) test under each kernel family (the per-call path
    argument): 1 = streaming (few chains), 2 = tile-resident (many chains)."""
    from prospective_rqf_b200 import ops

    with ops.btf_kernel_family(request.param):
        yield request.param


def _btf_coeffs(F, seed):
    rng = np.random.default_rng(seed)
    lam = rng.uniform(0.8, 0.9999, F) * np.exp(1j * rng.uniform(0, 2 * np.pi, F))
    t0 = 0.5 * (rng.standard_normal(F) + 1j * rng.standard_normal(F))
    t1 = 0.5 * (rng.standard_normal(F) + 1j * rng.standard_normal(F))
    return [torch.from_numpy(a.astype(np.complex64)).cuda().requires_grad_(True)
            for a in (lam, t0, t1)]


@pytest.mark.parametrize("kind,F", [("s4rqf-two-tap", 64), ("ps5-plain", 32)])
def test_btf_config4_full_size_vs_oracle(kind, F, btf_path):
    import prospective_rqf_b200 as rqf

    B, T = 16, 16384
    c1, t0, t1 = _btf_coeffs(F, seed=F)
    gen = torch.Generator(device="cuda").manual_seed(F + 1)
    x = torch.randn(B, T, F, dtype=torch.complex64, device="cuda", generator=gen)
    gy = torch.randn(B, T, F, dtype=torch.complex64, device="cuda", generator=gen)
    x.requires_grad_(True)
    if kind == "ps5-plain":
        y = rqf._triton_chunked_scan(c1, t0, x)
        gx, gc1, gc2 = torch.autograd.grad(y, (x, c1, t0), gy)
        y_ref = oracle.two_tap_forward(_h(c1), _h(t0), None, _h(x), "btf")
        gx_ref, gc1_ref, gc2_ref, _ = oracle.two_tap_backward(_h(c1), _h(t0), None, _h(x),
                                                             _h(gy), "btf")
        pairs = [("gx", gx, gx_ref), ("gc1", gc1, gc1_ref), ("gc2", gc2, gc2_ref)]
    else:
        y = rqf._triton_chunked_scan_prospective(c1, t0, t1, x)
        gc1, gt0, gt1, gx = torch.autograd.grad(y, (c1, t0, t1, x), gy)
        y_ref = oracle.two_tap_forward(_h(c1), _h(t0), _h(t1), _h(x), "btf")
        gx_ref, gc1_ref, gt0_ref, gt1_ref = oracle.two_tap_backward(
            _h(c1), _h(t0), _h(t1), _h(x), _h(gy), "btf")
        pairs = [("gx", gx, gx_ref), ("gc1", gc1, gc1_ref), ("gtap0", gt0, gt0_ref),
                 ("gtap1", gt1, gt1_ref)]
    assert_close(_h(y), y_ref, FWD_TOL, "y", elem_tol=FWD_ELEM_TOL)
    for name, got, ref in pairs:
        assert_close(_h(got), ref, GRAD_TOL, name, elem_tol=GRAD_ELEM_TOL)


def test_selective_config3_full_launch_vs_oracle_on_two_groups():
    from oracle import selective
    from test_gpu_selective import run_kernel

    F, B, T, G = 256, 32, 4096, 8
    opt = (True, True, True, False, 0.223, 0.223, True, False, True, 2.0, 0.0, True)
    rng = np.random.default_rng(33)
    c32 = lambda a: np.asarray(a, np.float32).astype(np.float64)  # noqa: E731
    theta = c32(rng.uniform(0.05, 2.5, F))
    groups = np.repeat(np.arange(G), F // G)
    rng.shuffle(groups)
    gen = torch.Generator(device="cuda").manual_seed(34)

    def randn(*shape, cplx=False):
        t = torch.randn(*shape, dtype=torch.complex64 if cplx else torch.float32,
                        device="cuda", generator=gen)
        return t.cpu().numpy().astype(np.complex128 if cplx else np.float64)

    d = dict(gl=randn(F, B, T), dl=randn(G, B, T), wl=randn(F, B, T),
             bias=c32(rng.standard_normal(F)), theta=theta, groups=groups,
             lo=c32(np.full(F, 1e-6)), span=c32(np.full(F, 1 - 2e-6)), step=c32(np.full(F, 0.2)),
             horizon=c32(np.full(F, 1.0)), th_lo=c32(theta * 0.4), th_hi=c32(theta * 1.6))
    z, gy, gx = (randn(F, B, T, cplx=True) for _ in range(3))
    raw, act, (dz, dzw, dG, dD, dW, dbias, dtheta) = run_kernel(z, d, opt, gy, gx, False)

    gsel = np.array([1, 6])
    fsel = np.flatnonzero(np.isin(groups, gsel))
    remap = np.full(G, -1)
    remap[gsel] = np.arange(len(gsel))
    ins = dict(gl=d["gl"][fsel], dl=d["dl"][gsel], wl=d["wl"][fsel], bias=d["bias"][fsel],
               theta=theta[fsel], groups=remap[groups[fsel]], lo=d["lo"][fsel],
               span=d["span"][fsel], step=d["step"][fsel], horizon=d["horizon"][fsel],
               th_lo=d["th_lo"][fsel], th_hi=d["th_hi"][fsel], opt=opt)
    zs = z[fsel]
    y_ref, co = selective.forward(zs, **ins)
    act_ref = np.maximum(y_ref.real, 0) + 1j * np.maximum(y_ref.imag, 0)
    assert_close(raw[fsel], y_ref, FWD_TOL, "raw", elem_tol=FWD_ELEM_TOL)
    assert_close(act[fsel], act_ref, FWD_TOL, "act", elem_tol=FWD_ELEM_TOL)
    mask = oracle.relu_mask_from_output(act[fsel])
    edge = oracle.mask_disagreement(mask, y_ref)
    assert edge < MASK_EDGE, f"split-ReLU decision differs at |state| = {edge:.2e} max"
    rdz, rdzw, rdG, rdD, rdW, rdbias, rdtheta = selective.backward(
        zs, y_ref, co, gy[fsel], gx[fsel], truncated=False, mask=mask, **ins)
    for name, got, ref in (("dz", dz[fsel], rdz), ("dzw", dzw[fsel], rdzw),
                           ("dG", dG[fsel], rdG), ("dW", dW[fsel], rdW),
                           ("dD", dD[gsel], rdD), ("dbias", dbias[fsel], rdbias),
                           ("dtheta", dtheta[fsel], rdtheta)):
        assert_close(got, ref, GRAD_TOL, name, elem_tol=GRAD_ELEM_TOL)
    assert math.isfinite(float(np.abs(dz).max()))


@pytest.mark.parametrize("F,B", [(128, 16), (256, 32)])
def test_rank1_first_block_full_size(F, B):
    """The first block over a one-channel input at configs 2 and 5 (T = 16000),
    on the rank-1 kernels against the general first block on the same inputs
    (rqf_lowrank_drive, the row forward with the fused skip, the row backward
    and rqf_rowdot; both already checked against the oracle): the forward bit
    for bit (the same operations), the backward's coefficient gradients and row
    sums, full BPTT and TBPTT(1), within fp32 summation-order noise."""
    from prospective_rqf_b200 import ops

    T = 16000
    c1, t0, t1 = _model_coefficients(F, 11 + F)
    g = torch.Generator(device="cuda").manual_seed(F + B)
    x = (0.5 * torch.randn(B, T, device="cuda", generator=g)).clamp(-1, 1)
    u = 0.2 * torch.randn(F, dtype=torch.complex64, device="cuda", generator=g)
    beta = 0.1 * torch.randn(F, dtype=torch.complex64, device="cuda", generator=g)
    w = torch.randn(F, device="cuda", generator=g)
    bb = 0.1 * torch.randn(F, device="cuda", generator=g)
    gy = torch.randn(F, B, T, dtype=torch.complex64, device="cuda", generator=g)
    xr = x.reshape(1, -1)

    out1, saved1 = ops.rank1_block_forward(u, beta, w, bb, x, c1, t0, t1, True)
    z, h0 = ops.lowrank_drive(u[:, None], xr, beta, w[:, None], bb)
    out2, saved2 = ops._fbt_forward(c1, t0, t1, z.view(F, B, T), True, h0.view(F, B, T))
    assert torch.equal(out1, out2), "rank-1 forward differs from the general first block"
    del out1, out2

    tol = 1e-4
    gc1, gt0, gt1, G, Gs = ops.rank1_block_backward(saved1, gy, True, True, True)
    rc1, rt0, rt1, gz = ops._fbt_backward(saved2, gy, True)
    for a, b, name in ((gc1, rc1, "gc1"), (gt0, rt0, "gtap0"), (gt1, rt1, "gtap1"),
                       (G, ops.rowdot(gz, xr, with_sum=True), "sum gz [x; 1]"),
                       (Gs, ops.rowdot(gy, xr, with_sum=True), "sum g [x; 1]")):
        assert_close(_h(a), _h(b), tol, "full BPTT " + name)
    del gz

    gc1, gt0, gt1, G, Gw, Gs = ops.rank1_tbptt_backward(saved1, gy, True, True, True)
    rc1, rt0, rt1, gz, gsum = ops._tbptt_backward_wsum(saved2, gy, True)
    for a, b, name in ((gc1, rc1, "gc1"), (gt0, rt0, "gtap0"), (gt1, rt1, "gtap1"),
                       (G, ops.rowdot(gz, xr, with_sum=True), "sum gz [x; 1]"),
                       (Gw, ops.rowdot(gsum, xr, with_sum=True), "sum (gz + gzw) [x; 1]"),
                       (Gs, ops.rowdot(gy, xr, with_sum=True), "sum g [x; 1]")):
        assert_close(_h(a), _h(b), tol, "TBPTT(1) " + name)
