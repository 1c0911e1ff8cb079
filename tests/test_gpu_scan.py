"""GPU parity of the sm_100a scan kernels (through the C ABI) against the
fp64 CPU oracle and the reference's golden vectors.

Tolerances (written here, from the benchmark's stated bounds): forward normwise max
relative error <= 1e-4, gradients <= 1e-3, fp32 kernels vs fp64 oracle.
"""

import numpy as np
import pytest
import torch

from _util import FWD_TOL, GRAD_TOL, assert_close, golden
from oracle import oracle

pytestmark = pytest.mark.gpu


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


@pytest.fixture(params=[1, 2], ids=["streaming", "resident"])
def btf_path(request):
    """Runs a (B,T,F) test under each kernel family (the per-call path
    argument): 1 = streaming (few chains), 2 = tile-resident (many chains)."""
    from prospective_rqf_b200 import ops

    with ops.btf_kernel_family(request.param):
        yield request.param


def dev(a, dtype=torch.complex64, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dtype)
    return t.requires_grad_(grad)


def host(t):
    return t.detach().cpu().numpy().astype(np.complex128)


def crandn(rng, shape, scale=1.0):
    return scale * (rng.standard_normal(shape) + 1j * rng.standard_normal(shape))


def coeffs(rng, F, rmin=0.8, rmax=0.999):
    mag = rng.uniform(rmin, rmax, F)
    lam = mag * np.exp(1j * rng.uniform(0, 2 * np.pi, F))
    return lam.astype(np.complex64).astype(np.complex128)


def c64(a):
    return np.asarray(a).astype(np.complex64).astype(np.complex128)


# split-ReLU decisions of the fp32 kernel may differ from fp64 only where the
# state is within rounding of zero (relu' is discontinuous there).
MASK_EDGE = 1e-4


def check_fbt(ins, y, gy, c1, t0, t1, z, fuse, layout="fbt"):
    """Forward vs the fp64 oracle; backward vs the oracle VJP evaluated with
    the kernel's own split-ReLU decisions (checked to differ from fp64 only
    at |state| < MASK_EDGE * max|state|)."""
    y_ref = oracle.two_tap_forward(c1, t0, t1, z, layout, fuse_act=fuse)
    assert_close(host(y), y_ref, FWD_TOL, "y")
    mask = None
    if fuse:
        mask = oracle.relu_mask_from_output(host(y))
        raw_ref = oracle.two_tap_forward(c1, t0, t1, z, layout, fuse_act=False)
        edge = oracle.mask_disagreement(mask, raw_ref)
        assert edge < MASK_EDGE, f"split-ReLU decision differs at |state| = {edge:.2e} max"
    y.backward(dev(gy))
    gz, gc1, gt0, gt1 = oracle.two_tap_backward(c1, t0, t1, z, gy, layout, fuse_act=fuse,
                                                mask=mask)
    for t, r, k in zip(ins, (gc1, gt0, gt1, gz), ("gc1", "gt0", "gt1", "gz")):
        assert_close(host(t.grad), r, GRAD_TOL, k)


# ----------------------------------------------------------- goldens
def test_golden_scan_complex(btf_path):
    g = golden("scan_complex")
    c1, c2, u = dev(g["c1"], grad=True), dev(g["c2"], grad=True), dev(g["u"], grad=True)
    y = rqf()._triton_chunked_scan(c1, c2, u)
    assert_close(host(y), g["y"], FWD_TOL, "y")
    y.backward(dev(g["gy"]))
    for t, k in ((c1, "gc1"), (c2, "gc2"), (u, "gu")):
        assert_close(host(t.grad), g[k], GRAD_TOL, k)


def test_golden_real_input_cfg1_style(btf_path):
    g = golden("scan_real_cfg1")
    c1, c2 = dev(g["c1"], grad=True), dev(g["c2"], grad=True)
    u = dev(g["u"], dtype=torch.float32, grad=True)
    y = rqf().sequential_scan(c1, c2, u)
    assert y.dtype == torch.complex64
    assert_close(host(y), g["y"], FWD_TOL, "y")
    (y.real ** 2 + y.imag ** 2).sum().backward()
    assert u.grad.dtype == torch.float32
    assert_close(host(c1.grad), g["gc1"], GRAD_TOL, "gc1")
    assert_close(host(c2.grad), g["gc2"], GRAD_TOL, "gc2")
    assert_close(u.grad.cpu().numpy(), g["gu"], GRAD_TOL, "gu")


def test_golden_prospective_btf(btf_path):
    g = golden("prospective_btf")
    ins = [dev(g[k], grad=True) for k in ("c1", "tap0", "tap1", "x")]
    y = rqf()._triton_chunked_scan_prospective(*ins)
    assert_close(host(y), g["y"], FWD_TOL, "y")
    y.backward(dev(g["gy"]))
    for t, k in zip(ins, ("gc1", "gt0", "gt1", "gx")):
        assert_close(host(t.grad), g[k], GRAD_TOL, k)


@pytest.mark.parametrize("name,fuse", [("fbt_split_relu", True), ("fbt_raw", False)])
def test_golden_fbt(name, fuse):
    g = golden(name)
    ins = [dev(g[k], grad=True) for k in ("c1", "tap0", "tap1", "z")]
    if fuse:
        y = rqf().fbt_recompute_scan(*ins)
    else:
        y = rqf().fbt_prospective_scan(*ins, False)
    assert_close(host(y), g["y"], FWD_TOL, "y")
    y.backward(dev(g["gy"]))
    for t, k in zip(ins, ("gc1", "gt0", "gt1", "gz")):
        assert_close(host(t.grad), g[k], GRAD_TOL, k)


def test_golden_tbptt():
    g = golden("tbptt")
    ins = [dev(g[k], grad=True) for k in ("c1", "tap0", "tap1", "u")]
    lag = dev(g["u"], grad=True)
    y = rqf().tbptt1_two_tap_scan(ins[3], ins[0], ins[1], ins[2], delayed_u=lag)
    assert_close(host(y), g["y"], FWD_TOL, "y")
    y.backward(dev(g["gy"]))
    for t, k in zip(ins + [lag], ("gc1", "gt0", "gt1", "gu", "gd")):
        assert_close(host(t.grad), g[k], GRAD_TOL, k)
    ins2 = [dev(g[k], grad=True) for k in ("c1", "tap0", "tap1", "u")]
    y2 = rqf().tbptt1_two_tap_scan(ins2[3], ins2[0], ins2[1], ins2[2])
    y2.backward(dev(g["gy"]))
    for t, k in zip(ins2, ("gc1_nolag", "gt0_nolag", "gt1_nolag", "gu_nolag")):
        assert_close(host(t.grad), g[k], GRAD_TOL, k)


# ------------------------------------------- (F,B,T) sweeps vs oracle
FBT_T = [1, 2, 3, 31, 2047, 2048, 2049, 4097, 5001, 6144]


@pytest.mark.parametrize("T", FBT_T)
@pytest.mark.parametrize("fuse", [True, False])
def test_fbt_lookback_tiles_vs_oracle(T, fuse):
    rng = np.random.default_rng(1000 + T + int(fuse))
    F, B = 3, 5
    c1 = coeffs(rng, F)
    t0, t1 = c64(crandn(rng, F, 0.5)), c64(crandn(rng, F, 0.5))
    z = c64(crandn(rng, (F, B, T)))
    gy = c64(crandn(rng, (F, B, T)))
    ins = [dev(a, grad=True) for a in (c1, t0, t1, z)]
    y = rqf().fbt_prospective_scan(*ins, fuse)
    check_fbt(ins, y, gy, c1, t0, t1, z, fuse)


# Row counts >= the resident CTAs of the persistent kernels (at most 3 per SM
# on 148 SMs = 444) take the persistent row-sequential path; the sweep above
# (15 rows) takes the look-back tile path.
@pytest.mark.parametrize("T", [2, 2048, 2050, 6000])
@pytest.mark.parametrize("fuse", [True, False])
def test_fbt_persistent_rows_vs_oracle(T, fuse):
    rng = np.random.default_rng(2000 + T + int(fuse))
    F, B = 37, 16  # 592 rows
    c1 = coeffs(rng, F)
    t0, t1 = c64(crandn(rng, F, 0.5)), c64(crandn(rng, F, 0.5))
    z = c64(crandn(rng, (F, B, T)))
    gy = c64(crandn(rng, (F, B, T)))
    ins = [dev(a, grad=True) for a in (c1, t0, t1, z)]
    y = rqf().fbt_prospective_scan(*ins, fuse)
    check_fbt(ins, y, gy, c1, t0, t1, z, fuse)


def test_fbt_long_sequence_undamped_poles_lookback():
    """Same hardest case through the look-back tile kernels (few rows)."""
    rng = np.random.default_rng(8)
    F, B, T = 8, 4, 16000
    mag = np.concatenate([np.full(4, np.exp(-2e-7)), rng.uniform(0.9, 0.9999, 4)])
    c1 = c64(mag * np.exp(1j * rng.uniform(0, np.pi, F)))
    t0, t1 = c64(crandn(rng, F, 0.05)), c64(crandn(rng, F, 0.05))
    z = c64(crandn(rng, (F, B, T)))
    gy = c64(crandn(rng, (F, B, T)))
    ins = [dev(a, grad=True) for a in (c1, t0, t1, z)]
    y = rqf().fbt_recompute_scan(*ins)
    check_fbt(ins, y, gy, c1, t0, t1, z, True)


def test_fbt_long_sequence_undamped_poles():
    """T = 16000 with |C1| up to 1 - 2e-7 (the paper recipe's gamma -> 1e-6
    edge) — the hardest case for cross-tile carry accuracy."""
    rng = np.random.default_rng(7)
    F, B, T = 8, 80, 16000  # 640 rows: persistent path
    mag = np.concatenate([np.full(4, np.exp(-2e-7)), rng.uniform(0.9, 0.9999, 4)])
    c1 = c64(mag * np.exp(1j * rng.uniform(0, np.pi, F)))
    t0, t1 = c64(crandn(rng, F, 0.05)), c64(crandn(rng, F, 0.05))
    z = c64(crandn(rng, (F, B, T)))
    gy = c64(crandn(rng, (F, B, T)))
    ins = [dev(a, grad=True) for a in (c1, t0, t1, z)]
    y = rqf().fbt_recompute_scan(*ins)
    check_fbt(ins, y, gy, c1, t0, t1, z, True)


def test_fbt_full_size_linearity_and_adjoint():
    """Config-2 shape (F=128, B=16, T=16000): size-independent properties of
    the raw (linear) scan — linearity in z and the adjoint identity
    Re<gy, J dz> == Re<J^H gy, dz> that the backward must satisfy."""
    torch.manual_seed(0)
    F, B, T = 128, 16, 16000
    c1 = (torch.rand(F, device="cuda") * 0.1 + 0.9) * torch.exp(
        1j * torch.rand(F, device="cuda") * 3.0)
    c1 = c1.to(torch.complex64)
    t0 = torch.randn(F, dtype=torch.complex64, device="cuda") * 0.1
    t1 = torch.randn(F, dtype=torch.complex64, device="cuda") * 0.1
    z1 = torch.randn(F, B, T, dtype=torch.complex64, device="cuda")
    z2 = torch.randn(F, B, T, dtype=torch.complex64, device="cuda")
    a, b = 0.7 - 0.2j, -1.3 + 0.4j
    scan = rqf().fbt_prospective_scan
    y12 = scan(c1, t0, t1, a * z1 + b * z2, False)
    y1, y2 = scan(c1, t0, t1, z1, False), scan(c1, t0, t1, z2, False)
    lin = (y12 - (a * y1 + b * y2)).abs().max() / y12.abs().max()
    assert lin.item() < FWD_TOL
    zz = z1.clone().requires_grad_(True)
    y = scan(c1, t0, t1, zz, False)
    gy = torch.randn_like(y)
    (gz,) = torch.autograd.grad(y, zz, gy)
    lhs = torch.sum(gy.conj() * y).real.double()  # <gy, J z1>
    rhs = torch.sum(gz.conj() * z1).real.double()  # <J^H gy, z1>
    assert abs(lhs - rhs).item() / abs(lhs).item() < GRAD_TOL


def test_fbt_matches_btf_layout():
    rng = np.random.default_rng(3)
    B, T, F = 4, 3000, 40
    c1 = coeffs(rng, F)
    t0, t1 = c64(crandn(rng, F, 0.3)), c64(crandn(rng, F, 0.3))
    x = dev(crandn(rng, (B, T, F)))
    args = [dev(c1), dev(t0), dev(t1)]
    y_btf = rqf()._triton_chunked_scan_prospective(*args, x)
    y_fbt = rqf().fbt_prospective_scan(*args, x.permute(2, 0, 1).contiguous(), False)
    err = (y_fbt.permute(1, 2, 0) - y_btf).abs().max() / y_btf.abs().max()
    assert err.item() < FWD_TOL


# ------------------------------------------- (B,T,F) sweeps vs oracle
# Every shape runs under both (B,T,F) kernel families.  Chains = B * ceil(F / 32).
# Streaming tiles: S x 128 steps, S = 8 below 20 chains, 4 below 40, 2 below 80,
# else 1.  Tile-resident tiles: 1..4 (forward) or 1..2 (backward) x 64 steps,
# the longest leaving a tile per SM, no longer than T needs.
BTF_SHAPES = [(1, 1, 1), (2, 63, 5), (2, 128, 32), (3, 129, 33), (2, 1023, 8), (1, 777, 16),
              (2, 4096, 96), (2, 16000, 32),    # resident: 125 / 250 tiles per chain
              (10, 2000, 96), (16, 3001, 33),   # 30 / 32 chains
              (45, 700, 32),                    # 45 chains
              (80, 300, 32), (40, 257, 70),     # 80 / 120 chains
              (160, 1100, 32)]                  # 160 chains: resident tiles of 4 x 64


@pytest.mark.parametrize("B,T,F", BTF_SHAPES)
def test_btf_plain_vs_oracle(B, T, F, btf_path):
    rng = np.random.default_rng(B * 100000 + T * 10 + F)
    c1 = coeffs(rng, F)
    c2 = c64(crandn(rng, F, 0.1))
    u = c64(crandn(rng, (B, T, F)))
    gy = c64(crandn(rng, (B, T, F)))
    ins = [dev(a, grad=True) for a in (c1, c2, u)]
    y = rqf()._triton_chunked_scan(*ins)
    assert_close(host(y), oracle.chunked_scan(c1, c2, u), FWD_TOL, "y")
    y.backward(dev(gy))
    gc1, gc2, gu = oracle.chunked_scan_backward(c1, c2, u, gy)
    for t, r, k in zip(ins, (gc1, gc2, gu), ("gc1", "gc2", "gu")):
        assert_close(host(t.grad), r, GRAD_TOL, k)


@pytest.mark.parametrize("B,T,F", BTF_SHAPES)
def test_btf_prospective_vs_oracle(B, T, F, btf_path):
    rng = np.random.default_rng(7 + B * 100000 + T * 10 + F)
    c1 = coeffs(rng, F)
    t0, t1 = c64(crandn(rng, F, 0.5)), c64(crandn(rng, F, 0.5))
    x = c64(crandn(rng, (B, T, F)))
    gy = c64(crandn(rng, (B, T, F)))
    ins = [dev(a, grad=True) for a in (c1, t0, t1, x)]
    y = rqf()._triton_chunked_scan_prospective(*ins)
    assert_close(host(y), oracle.two_tap_forward(c1, t0, t1, x, "btf"), FWD_TOL, "y")
    y.backward(dev(gy))
    gx, gc1, gt0, gt1 = oracle.two_tap_backward(c1, t0, t1, x, gy, "btf")
    for t, r, k in zip(ins, (gc1, gt0, gt1, gx), ("gc1", "gt0", "gt1", "gx")):
        assert_close(host(t.grad), r, GRAD_TOL, k)


def test_btf_real_input_matches_promoted(btf_path):
    rng = np.random.default_rng(5)
    B, T, F = 3, 500, 20
    c1, c2 = coeffs(rng, F), c64(crandn(rng, F))
    u = rng.standard_normal((B, T, F)).astype(np.float32)
    ur = dev(u, dtype=torch.float32, grad=True)
    uc = dev(u.astype(np.complex128), grad=True)
    yr = rqf()._triton_chunked_scan(dev(c1), dev(c2), ur)
    yc = rqf()._triton_chunked_scan(dev(c1), dev(c2), uc)
    torch.testing.assert_close(yr, yc, rtol=1e-5, atol=1e-5)
    gy = dev(crandn(rng, (B, T, F)))
    yr.backward(gy)
    yc.backward(gy)
    torch.testing.assert_close(ur.grad, uc.grad.real, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("B,T,F,real", [(1, 1, 1, False), (2, 1023, 8, False), (3, 500, 20, True),
                                         (80, 300, 32, False), (160, 1100, 32, True)])
def test_scan_abs_epilogue_vs_oracle(B, T, F, real, btf_path):
    """sequential_scan_abs without gradients: |y| written by the scan's epilogue
    (float32 output), against |oracle scan|."""
    rng = np.random.default_rng(11 + B * 1000 + T + F)
    c1, c2 = coeffs(rng, F), c64(crandn(rng, F, 0.5))
    if real:
        u = rng.standard_normal((B, T, F)).astype(np.float32).astype(np.float64)
        ud = dev(u, dtype=torch.float32)
    else:
        u = c64(crandn(rng, (B, T, F)))
        ud = dev(u)
    with torch.no_grad():
        y = rqf().sequential_scan_abs(dev(c1), dev(c2), ud)
    assert y.dtype == torch.float32 and tuple(y.shape) == (B, T, F)
    ref = np.abs(oracle.chunked_scan(c1, c2, u))
    assert_close(y.cpu().numpy().astype(np.float64), ref, FWD_TOL, "|y|")


def test_config1_exact_shapes(btf_path):
    """Benchmark config 1: u real [32,161,128] ~ N(0,1), lambda = r e^{i theta},
    r ~ U(0.90, 0.999), theta ~ U(0, pi), b ~ CN(0,1)/sqrt(2), y0 = 0; grads of
    sum |y|^2 w.r.t. u, lambda and b."""
    g = torch.Generator().manual_seed(0)
    B, T, H = 32, 161, 128
    u = torch.randn(B, T, H, generator=g)
    r = 0.90 + 0.099 * torch.rand(H, generator=g)
    th = torch.pi * torch.rand(H, generator=g)
    lam = torch.polar(r, th)
    b = torch.complex(torch.randn(H, generator=g), torch.randn(H, generator=g)) / np.sqrt(2.0)
    ins = [lam.cuda().requires_grad_(True), b.cuda().requires_grad_(True),
           u.cuda().requires_grad_(True)]
    y = rqf().sequential_scan(*ins)
    y_ref = oracle.chunked_scan(lam.numpy(), b.numpy(), u.numpy())
    assert_close(host(y), y_ref, FWD_TOL, "y")
    (y.real ** 2 + y.imag ** 2).sum().backward()
    gc1, gc2, gu = oracle.chunked_scan_backward(lam.numpy(), b.numpy(), u.numpy(), 2.0 * y_ref)
    assert_close(host(ins[0].grad), gc1, GRAD_TOL, "grad lambda")
    assert_close(host(ins[1].grad), gc2, GRAD_TOL, "grad b")
    assert_close(ins[2].grad.cpu().numpy(), gu.real, GRAD_TOL, "grad u")


# ------------------------------------------------------- TBPTT(1)
@pytest.mark.parametrize("layout", ["btf", "fbt"])
@pytest.mark.parametrize("T,B", [(1, 3), (5, 3), (2049, 3), (3000, 3), (1500, 30), (700, 90)])
def test_tbptt_vs_oracle(layout, T, B, btf_path):
    rng = np.random.default_rng(T + B + (0 if layout == "btf" else 1))
    F = 6
    shape = (B, T, F) if layout == "btf" else (F, B, T)
    c1 = coeffs(rng, F)
    t0, t1 = c64(crandn(rng, F, 0.5)), c64(crandn(rng, F, 0.5))
    z = c64(crandn(rng, shape))
    gy = c64(crandn(rng, shape))
    for fuse in ([False] if layout == "btf" else [False, True]):
        ins = [dev(a, grad=True) for a in (c1, t0, t1, z)]
        lag = dev(z, grad=True)
        y = rqf().tbptt1_two_tap_scan(ins[3], ins[0], ins[1], ins[2], delayed_u=lag,
                                      layout=layout, fuse_act=fuse)
        ref_y = oracle.two_tap_forward(c1, t0, t1, z, layout, fuse_act=fuse)
        assert_close(host(y), ref_y, FWD_TOL, "y")
        y.backward(dev(gy))
        gz, gzw, gc1, gt0, gt1 = oracle.tbptt_backward(c1, t0, t1, z, gy, layout, fuse_act=fuse)
        for t, r, k in zip(ins + [lag], (gc1, gt0, gt1, gz, gzw),
                           ("gc1", "gt0", "gt1", "gz", "gzw")):
            assert_close(host(t.grad), r, GRAD_TOL, f"{k} fuse={fuse}")


@pytest.mark.parametrize("T", [2, 2048, 2050, 5000])
@pytest.mark.parametrize("fuse", [False, True])
def test_tbptt_fbt_persistent_rows_vs_oracle(T, fuse):
    """640 rows: the persistent TBPTT(1) kernel.  g is pointwise here, so the
    oracle is evaluated on the cotangent pre-masked by the kernel's own
    split-ReLU decisions (checked to differ from fp64 only near 0)."""
    rng = np.random.default_rng(3000 + T + int(fuse))
    F, B = 40, 16
    c1 = coeffs(rng, F)
    t0, t1 = c64(crandn(rng, F, 0.5)), c64(crandn(rng, F, 0.5))
    z = c64(crandn(rng, (F, B, T)))
    gy = c64(crandn(rng, (F, B, T)))
    ins = [dev(a, grad=True) for a in (c1, t0, t1, z)]
    lag = dev(z, grad=True)
    y = rqf().tbptt1_two_tap_scan(ins[3], ins[0], ins[1], ins[2], delayed_u=lag, layout="fbt",
                                  fuse_act=fuse)
    ref_y = oracle.two_tap_forward(c1, t0, t1, z, "fbt", fuse_act=fuse)
    assert_close(host(y), ref_y, FWD_TOL, "y")
    g_ref = gy
    if fuse:
        mask = oracle.relu_mask_from_output(host(y))
        raw_ref = oracle.two_tap_forward(c1, t0, t1, z, "fbt", fuse_act=False)
        assert oracle.mask_disagreement(mask, raw_ref) < MASK_EDGE
        g_ref = np.where(mask[..., 0], gy.real, 0.0) + 1j * np.where(mask[..., 1], gy.imag, 0.0)
    y.backward(dev(gy))
    gz, gzw, gc1, gt0, gt1 = oracle.tbptt_backward(c1, t0, t1, z, g_ref, "fbt", fuse_act=False)
    for t, r, k in zip(ins + [lag], (gc1, gt0, gt1, gz, gzw), ("gc1", "gt0", "gt1", "gz", "gzw")):
        assert_close(host(t.grad), r, GRAD_TOL, k)


@pytest.mark.parametrize("F,B,T", [(40, 16, 5000), (40, 16, 4096), (3, 2, 5001), (3, 2, 2049)])
@pytest.mark.parametrize("fuse", [False, True])
def test_tbptt_fbt_wsum_matches_separate_outputs(F, B, T, fuse):
    """rqf_fbt_tbptt1_backward_wsum (grad_z and grad_z + grad_zw) against
    rqf_tbptt1_two_tap_backward on the same saved context: grad_z and the
    coefficient gradients equal, the sum equal to the two outputs added (at
    fp32 rounding), over the persistent row kernel (640 rows, whose tiles
    complete the sum across their boundary) and the per-tile kernel (6 rows),
    T cut inside a tile and T a multiple of it."""
    from prospective_rqf_b200 import ops

    rng = np.random.default_rng(4100 + F + T + int(fuse))
    c1 = coeffs(rng, F)
    t0, t1 = c64(crandn(rng, F, 0.5)), c64(crandn(rng, F, 0.5))
    z = dev(c64(crandn(rng, (F, B, T))))
    gy = dev(c64(crandn(rng, (F, B, T))))
    c1d, t0d, t1d = dev(c1), dev(t0), dev(t1)
    _, saved = ops._fbt_forward(c1d, t0d, t1d, z, fuse)
    a = ops._tbptt_backward(saved, "fbt", (F, B, T), gy, fuse)
    b = ops._tbptt_backward_wsum(saved, gy, fuse)
    for x, y_, name in zip(a[:4], b[:4], ("gc1", "gt0", "gt1", "gz")):
        assert torch.equal(x, y_), name
    assert_close(host(b[4]), host(a[3]) + host(a[4]), 1e-6, "gz + gzw")
    rqf().check_device_errors()


# ------------------------------------------------------- edge cases
def test_empty_shapes_give_zero_grads():
    for shape in [(0, 10, 4), (2, 0, 4)]:
        c1 = torch.full((4,), 0.9 + 0.1j, dtype=torch.complex64, device="cuda",
                        requires_grad=True)
        c2 = torch.ones(4, dtype=torch.complex64, device="cuda", requires_grad=True)
        u = torch.zeros(shape, dtype=torch.complex64, device="cuda", requires_grad=True)
        y = rqf()._triton_chunked_scan(c1, c2, u)
        assert y.shape == shape
        y.sum().abs().backward()
        assert torch.count_nonzero(c1.grad).item() == 0
        assert u.grad.shape == shape
    z = torch.zeros((4, 0, 7), dtype=torch.complex64, device="cuda", requires_grad=True)
    y = rqf().fbt_recompute_scan(c1, c1, c1, z)
    assert y.shape == (4, 0, 7)


def test_conj_and_noncontiguous_inputs():
    rng = np.random.default_rng(11)
    F, B, T = 4, 3, 300
    c1 = coeffs(rng, F)
    t0, t1 = c64(crandn(rng, F)), c64(crandn(rng, F))
    z = c64(crandn(rng, (B, T, F)))
    z_dev = dev(z).permute(2, 0, 1)  # non-contiguous (F,B,T) view
    y = rqf().fbt_prospective_scan(dev(c1).conj(), dev(t0), dev(t1), z_dev, True)
    ref = oracle.two_tap_forward(np.conj(c1), t0, t1, z.transpose(2, 0, 1), "fbt", fuse_act=True)
    assert_close(host(y), ref, FWD_TOL, "y")


def test_cpu_tensors_raise():
    with pytest.raises(RuntimeError, match="CUDA"):
        rqf().fbt_recompute_scan(torch.ones(2, dtype=torch.complex64),
                                 torch.ones(2, dtype=torch.complex64),
                                 torch.ones(2, dtype=torch.complex64),
                                 torch.ones(2, 1, 3, dtype=torch.complex64))


def test_repeated_calls_are_deterministic():
    torch.manual_seed(3)
    F, B, T = 16, 8, 7000
    c1 = (0.95 * torch.exp(1j * torch.rand(F) * 3)).to(torch.complex64).cuda()
    t0 = torch.randn(F, dtype=torch.complex64, device="cuda")
    t1 = torch.randn(F, dtype=torch.complex64, device="cuda")
    z = torch.randn(F, B, T, dtype=torch.complex64, device="cuda", requires_grad=True)
    gy = torch.randn(F, B, T, dtype=torch.complex64, device="cuda")
    outs = []
    for _ in range(3):
        c = c1.clone().requires_grad_(True)
        y = rqf().fbt_recompute_scan(c, t0, t1, z)
        gz, gc = torch.autograd.grad(y, (z, c), gy)
        outs.append((y, gz, gc))
    for y, gz, gc in outs[1:]:
        assert torch.equal(y, outs[0][0])
        assert torch.equal(gz, outs[0][1])
        assert torch.equal(gc, outs[0][2])


# ------------------------------------------- multi-oscillator scans
def _mosc_ref(c1, c2, u, cw, n):
    """fp64 torch restatement: the scan over the repeated input, then the
    C-weighted sum per filter (rqf_models/backbones/rqf/block.py:_c_weighted_sum)."""
    B, T, F = u.shape
    ur = u.repeat_interleave(n, dim=-1)
    x = torch.zeros(B, F * n, dtype=torch.complex128)
    outs = []
    for t in range(T):
        x = c1 * x + c2 * ur[:, t]
        outs.append((x.view(B, F, n) * cw.view(F, n)).sum(-1))
    return torch.stack(outs, 1)


@pytest.mark.parametrize("B,T,F,n,real", [(2, 300, 3, 4, False), (3, 700, 16, 2, True),
                                          (2, 1100, 10, 8, False), (40, 257, 4, 32, False),
                                          (2, 200, 5, 3, False), (1, 1, 2, 16, True)])
def test_multi_osc_vs_fp64(B, T, F, n, real):
    """The fused multi-oscillator scan (lanes = oscillators, C-weighted sum in
    the epilogue; n = 3 takes the composed path) against fp64, with the
    gradients of C1, C2, u and the real (F*n, 2) C-weights."""
    rng = np.random.default_rng(B * 7 + T + F * 11 + n)
    Fs = F * n
    c1, c2 = coeffs(rng, Fs), c64(crandn(rng, Fs, 0.5))
    cw = (0.5 * rng.standard_normal((Fs, 2))).astype(np.float32).astype(np.float64)
    u = (rng.standard_normal((B, T, F)).astype(np.float32).astype(np.float64) if real
         else c64(crandn(rng, (B, T, F))))
    gy = c64(crandn(rng, (B, T, F)))
    ins = [dev(c1, grad=True), dev(c2, grad=True),
           dev(u, dtype=torch.float32 if real else torch.complex64, grad=True),
           dev(cw, dtype=torch.float32, grad=True)]
    y = rqf().ops._triton_sequential_scan_multi_osc(*ins, n)
    refs = [torch.from_numpy(np.asarray(a)).requires_grad_(True) for a in (c1, c2, u, cw)]
    y_ref = _mosc_ref(refs[0], refs[1], refs[2], torch.view_as_complex(refs[3]), n)
    assert_close(host(y), y_ref.detach().numpy(), FWD_TOL, "y")
    y.backward(dev(gy))
    y_ref.backward(torch.from_numpy(gy))
    for t, r, k in zip(ins, refs, ("gc1", "gc2", "gu", "gcw")):
        assert_close(t.grad.detach().cpu().numpy().astype(np.complex128),
                     r.grad.numpy().astype(np.complex128), GRAD_TOL, k)


@pytest.mark.parametrize("n,real", [(4, False), (8, True), (3, False)])
def test_multi_osc_abs_epilogue(n, real):
    rng = np.random.default_rng(n + 100)
    B, T, F = 3, 500, 6
    Fs = F * n
    c1, c2 = coeffs(rng, Fs), c64(crandn(rng, Fs, 0.5))
    cw = (0.5 * rng.standard_normal((Fs, 2))).astype(np.float32).astype(np.float64)
    u = (rng.standard_normal((B, T, F)).astype(np.float32).astype(np.float64) if real
         else c64(crandn(rng, (B, T, F))))
    ops = rqf().ops
    ud = dev(u, dtype=torch.float32 if real else torch.complex64)
    with torch.no_grad():
        if real:
            y = ops._sequential_scan_multi_osc_real_forward_abs_raw(
                dev(c1), dev(c2), ud, dev(cw, dtype=torch.float32), n)
        else:
            cwd = dev(cw, dtype=torch.float32)
            y = ops._sequential_scan_multi_osc_forward_abs_raw(
                dev(c1), dev(c2), ud, cwd[:, 0].contiguous(), cwd[:, 1].contiguous(), n)
    assert y.dtype == torch.float32
    ref = _mosc_ref(torch.from_numpy(np.asarray(c1)), torch.from_numpy(np.asarray(c2)),
                    torch.from_numpy(np.asarray(u)), torch.view_as_complex(torch.from_numpy(cw)),
                    n).abs()
    assert_close(y.cpu().numpy().astype(np.float64), ref.numpy(), FWD_TOL, "|y|")
