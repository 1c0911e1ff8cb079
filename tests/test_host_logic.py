"""Host-side logic that needs no GPU: loud failure on CPU tensors (no
fallback), argument checks, and the install() rebinding of the reference's
dispatch names."""

import os
import sys
import types
from pathlib import Path

import pytest
import torch

import prospective_rqf_b200 as rqf
from prospective_rqf_b200 import integration, ops

# The reference's modules: its offline install under baseline/_ref (or RQF_REFERENCE).
REFERENCE = Path(os.environ.get("RQF_REFERENCE",
                                Path(__file__).resolve().parent.parent / "baseline" / "_ref"))


def c(*shape):
    return torch.ones(*shape, dtype=torch.complex64)


@pytest.mark.parametrize("fn,args", [
    (rqf._triton_chunked_scan, (c(3), c(3), c(2, 5, 3))),
    (rqf._triton_chunked_scan_prospective, (c(3), c(3), c(3), c(2, 5, 3))),
    (rqf.fbt_prospective_scan, (c(3), c(3), c(3), c(3, 2, 5), True)),
    (rqf.fbt_recompute_scan, (c(3), c(3), c(3), c(3, 2, 5))),
    (rqf.sequential_scan, (c(3), c(3), torch.ones(2, 5, 3))),
])
def test_cpu_tensors_raise_no_fallback(fn, args):
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        fn(*args)


def test_per_step_cross_entropy_checks_its_arguments():
    """The per-step loss refuses logits that do not match (classes,
    batch*time) float32 or labels that are not (batch,) before any launch,
    and CPU tensors with the no-fallback error."""
    from prospective_rqf_b200 import ops

    y = torch.zeros(2, dtype=torch.int64)
    with pytest.raises(ValueError):
        ops.per_step_cross_entropy(torch.zeros(5, 7), y, 2, 4)            # 7 != 2 * 4
    with pytest.raises(ValueError):
        ops.per_step_cross_entropy(torch.zeros(5, 8, dtype=torch.float64), y, 2, 4)
    with pytest.raises(ValueError):
        ops.per_step_cross_entropy(torch.zeros(5, 8), torch.zeros(3, dtype=torch.int64), 2, 4)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.per_step_cross_entropy(torch.zeros(5, 8), y, 2, 4)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.readout_bias_relu(torch.zeros(2, 2, 8), None)


def test_tbptt_rejects_bad_arguments():
    with pytest.raises(ValueError):
        rqf.tbptt1_two_tap_scan(c(2, 5, 3), c(3), c(3), c(3), layout="tbf")
    with pytest.raises(ValueError):
        rqf.tbptt1_two_tap_scan(c(2, 5, 3), c(3), c(3), c(3), layout="btf", fuse_act=True)
    with pytest.raises(ValueError):
        rqf.tbptt1_two_tap_scan(c(2, 5, 3), c(3), c(3), c(3), delayed_u=c(2, 4, 3))


def _fake_reference(monkeypatch):
    """Minimal stand-ins for the reference modules install() rebinds."""
    names = {
        "rqf_models": {},
        "rqf_models.ops": {},
        "rqf_models.ops.chunked_scan_kernel": {"_triton_chunked_scan": "orig",
                                               "_triton_chunked_scan_prospective": "orig"},
        "rqf_models.ops.scan": {"_triton_chunked_scan": "orig"},
        "rqf_models.ops.fbt_scan_kernel": {"fbt_prospective_scan": "orig",
                                           "fbt_recompute_scan": "orig"},
        "rqf_models.ops.selective_scan_kernel": {"selective_forward": "orig",
                                                 "selective_backward": "orig"},
        "rqf_models.ops.selective_scan": {"_SelectiveLayerScan": "orig"},
        "rqf_models.backbones": {},
        "rqf_models.backbones.rqf": {},
        "rqf_models.backbones.rqf.block": {"_triton_chunked_scan_prospective": "orig"},
        "rqf_models.backbones.rqf.pure": {"fbt_prospective_scan": "orig",
                                          "fbt_recompute_scan": "orig"},
    }
    for name, attrs in names.items():
        mod = types.ModuleType(name)
        for k, v in attrs.items():
            setattr(mod, k, v)
        monkeypatch.setitem(sys.modules, name, mod)

    class BaseRQFBlock:
        def __init__(self, tbptt):
            self.tbptt = tbptt

        def _use_tbptt1_scan_grad(self):
            return self.tbptt

        def _scan_two_tap_with_grad_mode(self, u, C1, tap0, tap1, *, delayed_u=None):
            return "reference-two-tap"

        def _scan_with_grad_mode(self, u, C1, C2):
            return "reference-single-tap"

    sys.modules["rqf_models.backbones.rqf.block"].BaseRQFBlock = BaseRQFBlock

    class RQF:
        param_space = "log"

        def __init__(self):
            self.log_tau = torch.zeros(3)
            self.log_theta = torch.zeros(3)
            self.log_gamma = torch.zeros(3)

        def compute_two_tap_coefficients(self, prospective=True, mode="tau",
                                         prospective_tau=None):
            return "reference-coefficients"

    filt = types.ModuleType("rqf_models.backbones.rqf.filter")
    filt.RQF = RQF
    monkeypatch.setitem(sys.modules, "rqf_models.backbones.rqf.filter", filt)
    return BaseRQFBlock


def test_install_rebinds_and_uninstall_restores(monkeypatch):
    Block = _fake_reference(monkeypatch)
    integration.uninstall()
    try:
        patched = rqf.install()
        assert "rqf_models.ops.scan._triton_chunked_scan" in patched
        assert sys.modules["rqf_models.ops.scan"]._triton_chunked_scan is ops._triton_chunked_scan
        assert sys.modules["rqf_models.backbones.rqf.pure"].fbt_recompute_scan is \
            ops.fbt_recompute_scan
        assert sys.modules["rqf_models.backbones.rqf.block"]._triton_chunked_scan_prospective \
            is ops._triton_chunked_scan_prospective
        # TBPTT wrapper: CPU tensors keep the reference's own path.
        blk = Block(tbptt=True)
        assert blk._scan_two_tap_with_grad_mode(c(1, 2, 3), c(3), c(3), c(3)) == \
            "reference-two-tap"
        assert blk._scan_with_grad_mode(c(1, 2, 3), c(3), c(3)) == "reference-single-tap"
        # Coefficient producer: CPU leaves keep the reference's own torch path.
        filt = sys.modules["rqf_models.backbones.rqf.filter"]
        assert "rqf_models.backbones.rqf.filter.RQF.compute_two_tap_coefficients" in patched
        assert filt.RQF().compute_two_tap_coefficients() == "reference-coefficients"
        assert filt.RQF.compute_two_tap_coefficients.__wrapped__ is not None
    finally:
        integration.uninstall()
    assert sys.modules["rqf_models.ops.scan"]._triton_chunked_scan == "orig"
    assert Block(tbptt=True)._scan_with_grad_mode(None, None, None) == "reference-single-tap"


@pytest.mark.skipif(not (REFERENCE / "rqf_models").exists(), reason="reference tree absent")
def test_install_against_the_reference_tree(monkeypatch):
    monkeypatch.syspath_prepend(str(REFERENCE))
    for name in list(sys.modules):
        if name.startswith("rqf_models"):
            monkeypatch.delitem(sys.modules, name)
    integration.uninstall()
    try:
        patched = rqf.install()
        import rqf_models.backbones.rqf.pure as pure
        import rqf_models.ops.scan as scan

        assert scan._triton_chunked_scan is ops._triton_chunked_scan
        assert pure.fbt_recompute_scan is ops.fbt_recompute_scan
        assert pure.fbt_prospective_scan is ops.fbt_prospective_scan
        import rqf_models.ops.selective_scan_kernel as sk

        assert sk.selective_forward is ops.selective_forward
        assert scan._sequential_scan_forward_abs_raw_block_f is \
            ops._sequential_scan_forward_abs_raw_block_f
        import rqf_models.ops.selective_scan as ss

        assert ss._SelectiveLayerScan is ops._SelectiveLayerScan
        assert "rqf_models.backbones.rqf.selective._SplitProjection" in patched
        assert len(patched) == 25
    finally:
        integration.uninstall()


def test_synthetic_waveforms_shape_range_and_fresh_batches():
    """Config 2/5 synthetic batches: (B, T, 1) in [-1, 1], labels in range, a
    new draw per step, and the same seed gives the same stream."""
    import torch

    from prospective_rqf_b200.train import StepConfig, synthetic_batches

    cfg = StepConfig(batch=3, time=800, num_classes=35)
    a = synthetic_batches(cfg, "cpu", seed=7)
    x0, y0 = next(a)
    x1, _ = next(a)
    assert x0.shape == (3, 800, 1) and x0.dtype == torch.float32
    assert y0.shape == (3,) and int(y0.min()) >= 0 and int(y0.max()) < 35
    assert float(x0.abs().max()) <= 1.0 and float(x0.std()) > 0.05
    assert not torch.equal(x0, x1)
    assert torch.equal(next(synthetic_batches(cfg, "cpu", seed=7))[0], x0)


def test_clip_grad_norm_matches_torch():
    """train.clip_grad_norm_ (foreach over real views) equals
    torch.nn.utils.clip_grad_norm_ on mixed real/complex gradients, clipping
    and not clipping."""
    import torch

    from prospective_rqf_b200.train import clip_grad_norm_

    g = torch.Generator().manual_seed(0)
    for max_norm in (0.5, 1e6):
        a = [torch.nn.Parameter(torch.randn(5, 4, dtype=torch.complex64, generator=g)),
             torch.nn.Parameter(torch.randn(7, generator=g)),
             torch.nn.Parameter(torch.randn(3, 3, dtype=torch.complex64, generator=g))]
        b = [torch.nn.Parameter(p.detach().clone()) for p in a]
        for p, q in zip(a, b):
            p.grad = torch.randn(p.shape, dtype=p.dtype, generator=g)
            q.grad = p.grad.clone()
        ta = clip_grad_norm_(a, max_norm)
        tb = torch.nn.utils.clip_grad_norm_(b, max_norm)
        assert torch.allclose(ta, tb, rtol=1e-6)
        for p, q in zip(a, b):
            assert torch.allclose(p.grad, q.grad, rtol=1e-6, atol=1e-7)


def test_bench_gemm_roofline_arithmetic():
    """bench.gemm_roofline: fp32-work FLOPs over the GEMM launch times against
    the split-TF32 ceiling (bf16 / 2 / 3); non-GEMM launches are ignored."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import bench

    flops = 10 * 8 * 256 * 256 * 512000
    r = bench.gemm_roofline({
        "rqf_projection": {"launches": 10, "total_ms": 10.0, "mean_ms": 1.0, "flops": flops},
        "rqf_fbt_block_forward": {"launches": 5, "total_ms": 2.5, "mean_ms": 0.5, "flops": 0}})
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert abs(r["achieved"] - flops / 10e-3 / 1e12) < 0.1
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-3
    assert list(r["per_kernel"]) == ["rqf_projection"]
    assert bench.gemm_roofline({"x": {"launches": 1, "total_ms": 1.0, "mean_ms": 1.0, "flops": 0}}) is None
