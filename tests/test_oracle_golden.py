"""Pin the CPU oracle to the reference: every golden vector under
tests/golden/ was produced by the reference implementation itself
(tests/golden/make_golden.py).  CPU only."""

import numpy as np

from _util import assert_close, golden
from oracle import oracle

FP64 = 1e-9   # oracle (fp64) vs reference fp64 PyTorch paths
FP32 = 2e-5   # oracle (fp64) vs reference fp32 kernels / loops


def test_scan_complex_parallel_scan_fp64():
    g = golden("scan_complex")
    y = oracle.chunked_scan(g["c1"], g["c2"], g["u"])
    assert_close(y, g["y"], FP64, "y")
    gc1, gc2, gu = oracle.chunked_scan_backward(g["c1"], g["c2"], g["u"], g["gy"])
    assert_close(gc1, g["gc1"], FP64, "gc1")
    assert_close(gc2, g["gc2"], FP64, "gc2")
    assert_close(gu, g["gu"], FP64, "gu")


def test_scan_real_cfg1_sum_of_squares():
    g = golden("scan_real_cfg1")
    u = g["u"].astype(np.complex128)
    y = oracle.chunked_scan(g["c1"], g["c2"], u)
    assert_close(y, g["y"], FP64, "y fp64")
    assert_close(y, g["y32"], FP32, "y vs sequential_scan fp32")
    # loss = sum |y|^2  ->  dL/dy (PyTorch convention) = 2 y
    gc1, gc2, gu = oracle.chunked_scan_backward(g["c1"], g["c2"], u, 2.0 * y)
    assert_close(gc1, g["gc1"], FP64, "gc1")
    assert_close(gc2, g["gc2"], FP64, "gc2")
    # parallel_scan promotes real u to complex64 (scan.py:516-517), so the
    # reference's grad of a real u carries fp32 rounding.
    assert_close(gu.real, g["gu"], 1e-6, "gu (real input)")
    assert_close(gc1, g["gc1_32"], 1e-4, "gc1 vs fp32 reference")
    assert_close(gu.real, g["gu_32"], 1e-4, "gu vs fp32 reference")


def test_prospective_btf_fp64():
    g = golden("prospective_btf")
    y = oracle.two_tap_forward(g["c1"], g["tap0"], g["tap1"], g["x"], "btf")
    assert_close(y, g["y"], FP64, "y")
    gx, gc1, gt0, gt1 = oracle.two_tap_backward(g["c1"], g["tap0"], g["tap1"], g["x"], g["gy"],
                                                "btf")
    for a, k in ((gx, "gx"), (gc1, "gc1"), (gt0, "gt0"), (gt1, "gt1")):
        assert_close(a, g[k], FP64, k)


def _check_fbt(name, fuse_act):
    g = golden(name)
    y = oracle.two_tap_forward(g["c1"], g["tap0"], g["tap1"], g["z"], "fbt", fuse_act=fuse_act)
    assert_close(y, g["y"], FP64, "y fp64")
    assert_close(y, g["y32"], FP32, "y vs reference Triton kernel")
    gz, gc1, gt0, gt1 = oracle.two_tap_backward(g["c1"], g["tap0"], g["tap1"], g["z"], g["gy"],
                                                "fbt", fuse_act=fuse_act)
    for a, k in ((gz, "gz"), (gc1, "gc1"), (gt0, "gt0"), (gt1, "gt1")):
        assert_close(a, g[k], FP64, k)
        assert_close(a, g[k + "_32"], 1e-4, k + " vs reference Triton kernel")


def test_fbt_split_relu_vs_reference_kernel():
    _check_fbt("fbt_split_relu", True)


def test_fbt_raw_vs_reference_kernel():
    _check_fbt("fbt_raw", False)


def test_btf_vs_reference_triton_kernels():
    g = golden("triton_btf")
    y = oracle.chunked_scan(g["c1"], g["c2"], g["u"])
    assert_close(y, g["y"], FP32, "chunked y")
    gc1, gc2, gu = oracle.chunked_scan_backward(g["c1"], g["c2"], g["u"], g["gy"])
    assert_close(gc1, g["gc1"], 1e-4, "chunked gc1")
    assert_close(gc2, g["gc2"], 1e-4, "chunked gc2")
    assert_close(gu, g["gu"], 1e-4, "chunked gu")
    yp = oracle.two_tap_forward(g["c1"], g["tap0"], g["tap1"], g["u"], "btf")
    assert_close(yp, g["yp"], FP32, "prospective y")
    gx, pgc1, pgt0, pgt1 = oracle.two_tap_backward(g["c1"], g["tap0"], g["tap1"], g["u"], g["gy"],
                                                   "btf")
    for a, k in ((gx, "pgx"), (pgc1, "pgc1"), (pgt0, "pgt0"), (pgt1, "pgt1")):
        assert_close(a, g[k], 1e-4, k)


def test_tbptt_surrogate_fp64():
    g = golden("tbptt")
    y = oracle.two_tap_forward(g["c1"], g["tap0"], g["tap1"], g["u"], "btf")
    assert_close(y, g["y"], FP64, "y")
    assert_close(y, g["y_nolag"], FP64, "y (no lag source)")
    gz, gzw, gc1, gt0, gt1 = oracle.tbptt_backward(g["c1"], g["tap0"], g["tap1"], g["u"],
                                                   g["gy"], "btf")
    assert_close(gz, g["gu"], FP64, "grad u (lag source separate)")
    assert_close(gzw, g["gd"], FP64, "grad delayed_u")
    assert_close(gz + gzw, g["gu_nolag"], FP64, "grad u (own lag source)")
    for a, k in ((gc1, "gc1"), (gt0, "gt0"), (gt1, "gt1")):
        assert_close(a, g[k], FP64, k)
        assert_close(a, g[k + "_nolag"], FP64, k + " nolag")


def test_layouts_agree():
    """BTF and FBT restatements are the same recurrence on permuted data."""
    rng = np.random.default_rng(0)
    B, T, F = 3, 50, 4
    x = rng.standard_normal((B, T, F)) + 1j * rng.standard_normal((B, T, F))
    c1 = 0.95 * np.exp(1j * rng.uniform(0, np.pi, F))
    t0 = rng.standard_normal(F) + 1j * rng.standard_normal(F)
    t1 = rng.standard_normal(F) + 1j * rng.standard_normal(F)
    y_btf = oracle.two_tap_forward(c1, t0, t1, x, "btf", fuse_act=True)
    y_fbt = oracle.two_tap_forward(c1, t0, t1, x.transpose(2, 0, 1), "fbt", fuse_act=True)
    np.testing.assert_allclose(y_fbt.transpose(1, 2, 0), y_btf, rtol=1e-13, atol=1e-13)
