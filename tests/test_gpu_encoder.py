"""Encoder-level parity: the B200 Pure RQF stack (prospective_rqf_b200.encoder —
fused skip blocks, ZOH two-tap coefficients, TBPTT(1) layers, readout)
against an fp64 CPU restatement of the same model whose scans run through the
fp64 oracle, on identical parameters and inputs.  Mirrors the reference's
FBT-vs-standard encoder check (tests/test_scan_backends_parity.py:109-162).
Tolerances: outputs 1e-4, parameter and input gradients 1e-3."""

import math

import numpy as np
import pytest
import torch

from _util import FWD_TOL, GRAD_TOL, assert_close, rel_err
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import prospective_rqf_b200 as rqf

    rqf.read_device_error(clear=True)
    yield
    rqf.check_device_errors()


def _np(t):
    return t.detach().resolve_conj().numpy()


class _OracleScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, c1, t0, t1, z, act):
        y = oracle.two_tap_forward(_np(c1), _np(t0), _np(t1), _np(z), "fbt", fuse_act=act)
        ctx.save_for_backward(c1, t0, t1, z)
        ctx.act = act
        return torch.from_numpy(y)

    @staticmethod
    def backward(ctx, g):
        c1, t0, t1, z = ctx.saved_tensors
        gz, gc1, gt0, gt1 = oracle.two_tap_backward(_np(c1), _np(t0), _np(t1), _np(z), _np(g),
                                                    "fbt", fuse_act=ctx.act)
        f = torch.from_numpy
        return f(gc1), f(gt0), f(gt1), f(gz), None


class _OracleTBPTT(torch.autograd.Function):
    """TBPTT(1): exact forward; surrogate grads, lag cotangent to W only."""

    @staticmethod
    def forward(ctx, h, W, c1, t0, t1, act):
        F_in, B, T = h.shape
        z = (W.detach() @ h.detach().reshape(F_in, B * T)).reshape(-1, B, T)
        y = oracle.two_tap_forward(_np(c1), _np(t0), _np(t1), _np(z), "fbt", fuse_act=act)
        ctx.save_for_backward(h, W, c1, t0, t1, z)
        ctx.act = act
        return torch.from_numpy(y)

    @staticmethod
    def backward(ctx, g):
        h, W, c1, t0, t1, z = ctx.saved_tensors
        gz, gzw, gc1, gt0, gt1 = oracle.tbptt_backward(_np(c1), _np(t0), _np(t1), _np(z),
                                                       _np(g), "fbt", fuse_act=ctx.act)
        gz, gzw = torch.from_numpy(gz), torch.from_numpy(gzw)
        F_in, B, T = h.shape
        gh = (W.mH @ gz.reshape(-1, B * T)).reshape(F_in, B, T)
        gW = (gz + gzw).reshape(-1, B * T) @ h.reshape(F_in, B * T).mH
        f = torch.from_numpy
        return gh, gW, f(gc1), f(gt0), f(gt1), None


def _two_tap(log_theta, log_gamma, dt, tau):
    gamma, theta = log_gamma.exp(), log_theta.exp()
    a = torch.complex(-gamma / tau, (theta / tau) * (1.0 - gamma)) * dt
    c1 = torch.exp(a)
    phi = torch.where(a.abs() < 1e-4, 1 + a / 2 + a ** 2 / 6 + a ** 3 / 24 + a ** 4 / 120,
                      (torch.exp(a) - 1) / torch.where(a.abs() < 1e-4, torch.ones_like(a), a))
    extra = gamma * c1
    return c1, gamma * (dt / tau) * phi + extra, -extra


def reference_forward(model, x, params):
    enc = model.encoder
    B, T, I = x.shape
    h = params["input_proj.weight"] @ x.permute(2, 0, 1).reshape(I, B * T)
    if "input_proj.bias" in params:
        h = h + params["input_proj.bias"][:, None]
    h = h.reshape(-1, B, T).to(torch.complex128)
    n = len(enc.W)
    for i in range(n):
        r = enc.rqf[i]
        c1, t0, t1 = _two_tap(params[f"rqf.{i}.log_theta"], params[f"rqf.{i}.log_gamma"], r.dt,
                              r.tau)
        W = params[f"W.{i}"]
        act = enc.final_activation or i + 1 < n
        skip = enc.skip and W.shape[0] == W.shape[1]
        if enc.scan_grad_mode == "tbptt1":
            out = _OracleTBPTT.apply(h, W, c1, t0, t1, act)
        else:
            z = (W @ h.reshape(W.shape[1], B * T)).reshape(W.shape[0], B, T)
            out = _OracleScan.apply(c1, t0, t1, z, act)
        h = out + h if skip else out
    F = h.shape[0]
    feats = torch.cat([h.real, h.imag], dim=0).reshape(2 * F, B * T)
    hid = torch.relu(params["fc1.weight"] @ feats + params["fc1.bias"][:, None])
    logits = (params["fc2.weight"] @ hid + params["fc2.bias"][:, None]).reshape(-1, B, T)
    return logits.mean(dim=2).t()


@pytest.mark.parametrize("mode,T", [("full", 3000), ("full", 1000), ("tbptt1", 2500)])
def test_encoder_matches_fp64_restatement(mode, T):
    from prospective_rqf_b200.train import StepConfig, build_model

    torch.manual_seed(0)
    cfg = StepConfig(batch=4, time=T, hidden=16, depth=3, num_classes=5, readout_hidden=32,
                     scan_grad_mode=mode)
    model = build_model(cfg, "cuda", seed=3)
    # gamma spread over the recipe band so some poles are nearly undamped
    with torch.no_grad():
        for r in model.encoder.rqf:
            r.log_gamma.copy_(torch.linspace(math.log(1e-3), math.log(0.9), 16))
    g = torch.Generator().manual_seed(5)
    x = (0.5 * torch.randn(cfg.batch, T, 1, generator=g)).clamp(-1, 1)
    y = torch.randint(0, cfg.num_classes, (cfg.batch,), generator=g)

    xg = x.cuda().requires_grad_(True)
    loss = torch.nn.functional.cross_entropy(model(xg), y.cuda())
    loss.backward()

    names = {}
    for name, p in model.named_parameters():
        key = name.replace("encoder.", "").replace("readout.", "")
        names[key] = p
    params = {k: (p.detach().cpu().to(torch.complex128 if p.is_complex() else torch.float64)
                  .requires_grad_(True)) for k, p in names.items()}
    xr = x.double().requires_grad_(True)
    logits_ref = reference_forward(model, xr, params)
    loss_ref = torch.nn.functional.cross_entropy(logits_ref, y)
    loss_ref.backward()

    assert_close(model(x.cuda()).detach().cpu().double().numpy(), logits_ref.detach().numpy(),
                 FWD_TOL, "logits")
    assert abs(loss.item() - loss_ref.item()) <= FWD_TOL * max(1.0, abs(loss_ref.item()))
    assert_close(xg.grad.cpu().double().numpy(), xr.grad.numpy(), GRAD_TOL, "grad x")
    for k, p in names.items():
        ref = params[k].grad
        assert ref is not None, k
        assert_close(p.grad.cpu().numpy().astype(np.complex128 if p.is_complex() else np.float64),
                     ref.numpy(), GRAD_TOL, f"grad {k}")


def _lowrank_case(I, bias, skip, T, lowrank, mode="full"):
    """Logits and every parameter gradient of a small encoder + readout, and
    the fp64 restatement's, with the first block on the low-rank path or on
    the general F x F GEMM path."""
    from prospective_rqf_b200 import encoder as E

    E.LOWRANK_MAX_INPUTS = 4 if lowrank else 0
    torch.manual_seed(0)
    enc = E.PureRQFEncoderB200(input_dims=I, hidden_dims=16, num_layers=3, skip_connection=skip,
                               input_proj_bias=bias, scan_grad_mode=mode, seed=4)
    model = E.RQFClassifier(enc, 5, 32).cuda()
    with torch.no_grad():
        for r in model.encoder.rqf:
            r.log_gamma.copy_(torch.linspace(math.log(1e-3), math.log(0.9), 16))
    g = torch.Generator().manual_seed(6)
    B = 4
    x = (0.5 * torch.randn(B, T, I, generator=g)).clamp(-1, 1)
    y = torch.randint(0, 5, (B,), generator=g)
    logits = model(x.cuda())
    torch.nn.functional.cross_entropy(logits, y.cuda()).backward()
    names = {n.replace("encoder.", "").replace("readout.", ""): p
             for n, p in model.named_parameters()}
    params = {k: (p.detach().cpu().to(torch.complex128 if p.is_complex() else torch.float64)
                  .requires_grad_(True)) for k, p in names.items()}
    logits_ref = reference_forward(model, x.double(), params)
    torch.nn.functional.cross_entropy(logits_ref, y).backward()
    got = {"logits": logits.detach().cpu().double().numpy()}
    ref = {"logits": logits_ref.detach().numpy()}
    for k, p in names.items():
        got[k] = p.grad.cpu().numpy().astype(np.complex128 if p.is_complex() else np.float64)
        ref[k] = params[k].grad.numpy()
    return got, ref


@pytest.mark.parametrize("I,bias,skip,T,mode", [
    (1, False, True, 3000, "full"), (1, True, True, 1000, "full"), (3, True, False, 1000, "full"),
    (2, False, True, 2001, "full"), (1, False, True, 2500, "tbptt1"), (2, True, True, 1000, "tbptt1"),
    (1, True, False, 1000, "tbptt1")])
def test_encoder_lowrank_first_block_matches_fp64(I, bias, skip, T, mode, monkeypatch):
    """The first block over the low-rank input projection (_InputBlock, and
    _InputTBPTT for TBPTT(1): rqf_lowrank_drive forward, rqf_rowdot
    cotangents) against the fp64
    restatement, which runs the F x F projection on h0 = w_in x + b_in.
    Each quantity is within tolerance of fp64 or no worse than the general
    path (F x F GEMMs) on the same inputs: some of these small configurations
    put a late layer's log_theta gradient near 1e-3 from fp64 in fp32 on
    either path."""
    from prospective_rqf_b200 import encoder as E
    from prospective_rqf_b200 import ops

    calls = []
    real_drive = ops.lowrank_drive
    monkeypatch.setattr(ops, "lowrank_drive", lambda *a, **k: calls.append(1) or real_drive(*a, **k))
    monkeypatch.setattr(E, "LOWRANK_MAX_INPUTS", E.LOWRANK_MAX_INPUTS)
    gen, ref = _lowrank_case(I, bias, skip, T, lowrank=False, mode=mode)
    assert not calls
    low, ref2 = _lowrank_case(I, bias, skip, T, lowrank=True, mode=mode)
    assert calls, "the low-rank first block did not run"
    for k in ref:
        e_low, e_gen = rel_err(low[k], ref2[k]), rel_err(gen[k], ref[k])
        tol = FWD_TOL if k == "logits" else GRAD_TOL
        assert e_low <= max(tol, 1.05 * e_gen), f"{k}: {e_low:.3e} vs fp64 (general path {e_gen:.3e})"


@pytest.mark.parametrize("H,B,T", [(7, 3, 1000), (5, 2, 33), (4, 3, 1), (16, 4, 4096)])
def test_readout_relu_pool_vs_torch(H, B, T):
    """rqf_readout_relu_pool / _backward against torch fp64 on the same z:
    the pooled ReLU means, the mask bits, the cotangent and the counts."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(H * 100 + T)
    z = torch.randn(H, B, T, generator=g)
    bias = 0.3 * torch.randn(H, generator=g)
    pooled, mask = ops.readout_relu_pool(z.cuda(), bias.cuda())
    pre = z.double() + bias.double()[:, None, None]
    ref = torch.relu(pre).mean(dim=2)
    assert_close(pooled.cpu().double().numpy(), ref.numpy(), 1e-6, "pooled")
    on = pre > 0
    words = (T + 31) // 32
    bits = torch.zeros(H, B, words * 32, dtype=torch.bool)
    bits[:, :, :T] = on
    want = (bits.reshape(H, B, words, 32).long() << torch.arange(32)).sum(-1)
    got = mask.cpu().long() & 0xFFFFFFFF
    assert torch.equal(got, want), "mask bits"
    scale = torch.randn(H, B, generator=g)
    gc, counts = ops.readout_relu_pool_backward(mask, scale.cuda(), T)
    assert torch.equal(gc.cpu(), on.float() * scale[:, :, None])
    assert torch.equal(counts.cpu(), on.sum(dim=2).float())


def test_synthetic_waveforms_drawn_on_the_gpu():
    from prospective_rqf_b200.train import StepConfig, synthetic_batches

    cfg = StepConfig(batch=4, time=16000, num_classes=35)
    x, y = next(synthetic_batches(cfg, "cuda", seed=1))
    assert x.is_cuda and y.is_cuda and x.shape == (4, 16000, 1)
    assert float(x.abs().max()) <= 1.0 and 0.05 < float(x.std()) < 1.0
    assert int(y.min()) >= 0 and int(y.max()) < 35


def test_two_tap_coefficient_kernels_vs_fp64_autograd():
    """ops.TwoTapCoefficients (rqf_two_tap_coefficients[_backward]) against
    the same expressions in torch fp64 with autograd: values and the leaves'
    gradients, over the recipe band and leaves small enough that |a| takes
    the 4th-order Taylor branch of (e^a - 1)/a."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(8)
    dt, tau = 1 / 16000, 5 / 16000
    lt = torch.cat([torch.rand(200, generator=g) * 7 - 8, torch.full((8,), -12.0)])
    lg = torch.cat([torch.rand(200, generator=g) * 13.5 - 13.8, torch.full((8,), -13.0)])
    lt64 = lt.double().requires_grad_(True)
    lg64 = lg.double().requires_grad_(True)
    gam, th = lg64.exp(), lt64.exp()
    a = torch.complex(-gam / tau, (th / tau) * (1.0 - gam)) * dt
    small = a.abs() < 1e-4
    safe = torch.where(small, torch.ones_like(a), a)
    phi = torch.where(small, 1 + a / 2 + a ** 2 / 6 + a ** 3 / 24 + a ** 4 / 120,
                      (torch.exp(a) - 1) / safe)
    c1 = torch.exp(a)
    ref = (c1, gam * (dt / tau) * phi + gam * c1, -gam * c1)
    assert bool(small.any()) and bool((~small).any())
    cot = [torch.randn(208, dtype=torch.complex128, generator=g) for _ in range(3)]
    loss = sum((torch.conj(w) * y).real.sum() for w, y in zip(cot, ref))
    glt_ref, glg_ref = torch.autograd.grad(loss, (lt64, lg64))
    ltc, lgc = lt.cuda().requires_grad_(True), lg.cuda().requires_grad_(True)
    out = ops.TwoTapCoefficients.apply(ltc, lgc, dt, tau)
    for o, r in zip(out, ref):
        assert_close(o.detach().cpu().numpy().astype(np.complex128), r.detach().numpy(), 1e-6,
                     "two-tap coefficients")
    l2 = sum((torch.conj(w.to(torch.complex64).cuda()) * y).real.sum() for w, y in zip(cot, out))
    glt, glg = torch.autograd.grad(l2, (ltc, lgc))
    assert_close(glt.cpu().double().numpy(), glt_ref.numpy(), 1e-5, "grad log_theta")
    assert_close(glg.cpu().double().numpy(), glg_ref.numpy(), 1e-5, "grad log_gamma")


def test_rowdot_and_lowrank_drive_vs_fp64():
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(2)
    F, N, I = 37, 2 * 20011, 3
    a = _crandn(g, F, N)
    x = torch.randn(I, N, generator=g)
    out = ops.rowdot(a.cuda(), x.cuda(), with_sum=True).cpu().numpy()
    a64, x64 = a.numpy().astype(np.complex128), x.numpy().astype(np.float64)
    ref = np.concatenate([a64 @ x64.T, a64.sum(1, keepdims=True)], axis=1)
    assert_close(out.astype(np.complex128), ref, 1e-5, "rowdot")
    assert torch.equal(ops.rowdot(a.cuda(), x.cuda(), True).cpu(), torch.from_numpy(out))
    u, beta = _crandn(g, F, I), _crandn(g, F)
    w, b = torch.randn(F, I, generator=g), torch.randn(F, generator=g)
    z, h = ops.lowrank_drive(u.cuda(), x.cuda(), beta.cuda(), w.cuda(), b.cuda())
    zr = u.numpy().astype(np.complex128) @ x64 + beta.numpy()[:, None]
    hr = w.numpy().astype(np.float64) @ x64 + b.numpy()[:, None]
    assert_close(z.cpu().numpy().astype(np.complex128), zr, 1e-6, "drive z")
    assert_close(h.cpu().numpy().astype(np.complex128), hr.astype(np.complex128), 1e-6, "drive h")
    z2, h2 = ops.lowrank_drive(u.cuda(), x.cuda())
    assert h2 is None
    assert_close(z2.cpu().numpy().astype(np.complex128), u.numpy().astype(np.complex128) @ x64,
                 1e-6, "drive z, no bias")


# ------------------------------------------- fused skip (rqf_fbt_block_forward)
def _crandn(g, *shape):
    return torch.randn(*shape, dtype=torch.complex64, generator=g)


def _coef(g, F):
    mag = 0.8 + 0.199 * torch.rand(F, generator=g)
    lam = torch.polar(mag, 6.283 * torch.rand(F, generator=g)).to(torch.complex64)
    return lam, 0.5 * _crandn(g, F), 0.5 * _crandn(g, F)


# 15 rows take the look-back tile kernels; 640 rows (>= the resident CTAs of
# every persistent forward kernel: 4 per SM x 148 without skip, 3 with) take
# the row-sequential kernels.  Between those counts the plain and the skip
# forward take different kernels, whose fp32 sums associate differently.
@pytest.mark.parametrize("F,B,T", [(3, 5, 5001), (40, 16, 2050), (40, 16, 1)])
@pytest.mark.parametrize("fuse", [True, False])
def test_block_forward_fused_skip(F, B, T, fuse):
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(F * 1000 + T + int(fuse))
    c1, t0, t1 = (t.cuda() for t in _coef(g, F))
    z, h = _crandn(g, F, B, T).cuda(), _crandn(g, F, B, T).cuda()
    fused, saved = ops._fbt_forward(c1, t0, t1, z, fuse, h)
    plain, _ = ops._fbt_forward(c1, t0, t1, z, fuse)
    # same scan arithmetic, one fp32 add at the store: bit-identical
    assert torch.equal(fused, plain + h)
    ref = oracle.two_tap_forward(_np(c1.cpu()), _np(t0.cpu()), _np(t1.cpu()), _np(z.cpu()), "fbt",
                                 fuse_act=fuse) + _np(h.cpu())
    assert_close(_np(fused.cpu()), ref, FWD_TOL, "act(y) + skip")
    assert saved[3].data_ptr() == z.data_ptr()  # the backward recomputes from z, not from out


@pytest.mark.parametrize("F,B,T", [(4, 3, 3000), (40, 16, 2100)])
@pytest.mark.parametrize("fuse,skip", [(True, True), (False, True), (True, False)])
def test_pure_block_matches_unfused_composition(F, B, T, fuse, skip, monkeypatch):
    """_PureBlock (GEMM + fused scan/skip + one accumulating GEMM backward)
    against W @ h -> fbt_prospective_scan -> + h composed by autograd, both
    with torch's projection GEMM so the scan sees bit-identical z."""
    import prospective_rqf_b200 as rqf
    from prospective_rqf_b200 import encoder
    from prospective_rqf_b200.encoder import _PureBlock

    monkeypatch.setattr(encoder, "PROJECTION", "torch")

    g = torch.Generator().manual_seed(F + B + T)
    c1, t0, t1 = (t.cuda() for t in _coef(g, F))
    W = (_crandn(g, F, F) / math.sqrt(2 * F)).cuda()
    h = _crandn(g, F, B, T).cuda()
    gy = _crandn(g, F, B, T).cuda()

    leaves_a = [t.clone().requires_grad_(True) for t in (h, W, c1, t0, t1)]
    out_a = _PureBlock.apply(*leaves_a, fuse, skip)
    out_a.backward(gy)

    leaves_b = [t.clone().requires_grad_(True) for t in (h, W, c1, t0, t1)]
    hb, Wb, c1b, t0b, t1b = leaves_b
    z = (Wb @ hb.reshape(F, B * T)).reshape(F, B, T)
    out_b = rqf.fbt_prospective_scan(c1b, t0b, t1b, z, fuse)
    if skip:
        out_b = out_b + hb
    out_b.backward(gy)

    assert torch.equal(out_a, out_b)
    for a, b, k in zip(leaves_a, leaves_b, ("h", "W", "c1", "tap0", "tap1")):
        assert_close(_np(a.grad.cpu()), _np(b.grad.cpu()), 1e-5, f"grad {k}")


@pytest.mark.parametrize("F,B,T", [(32, 4, 3000), (40, 16, 2100)])
@pytest.mark.parametrize("fuse", [False, True])
def test_pure_block_tc_projection_matches_torch(F, B, T, fuse, monkeypatch):
    """The block with its projections on the split-TF32 tcgen05 GEMM against
    the same block on torch's fp32 GEMM.  With the split-ReLU on, an fp32
    rounding difference may flip relu' at a state within rounding of 0, so
    only the forward is compared there."""
    from prospective_rqf_b200 import encoder
    from prospective_rqf_b200.encoder import _PureBlock

    g = torch.Generator().manual_seed(F * 3 + T)
    c1, t0, t1 = (t.cuda() for t in _coef(g, F))
    W = (_crandn(g, F, F) / math.sqrt(2 * F)).cuda()
    h = _crandn(g, F, B, T).cuda()
    gy = _crandn(g, F, B, T).cuda()
    res = {}
    for mode in ("tc", "torch"):
        monkeypatch.setattr(encoder, "PROJECTION", mode)
        leaves = [t.clone().requires_grad_(True) for t in (h, W, c1, t0, t1)]
        out = _PureBlock.apply(*leaves, fuse, True)
        out.backward(gy)
        res[mode] = (out.detach(), [l.grad for l in leaves])
    assert_close(_np(res["tc"][0].cpu()), _np(res["torch"][0].cpu()), 1e-5, "out")
    if not fuse:
        for a, b, k in zip(res["tc"][1], res["torch"][1], ("h", "W", "c1", "tap0", "tap1")):
            assert_close(_np(a.cpu()), _np(b.cpu()), 1e-4, f"grad {k}")


# -------------------------------- readout on the tensor-core projections
@pytest.mark.parametrize("per_step", [False, True])
def test_readout_tc_matches_torch(per_step, monkeypatch):
    """ComplexReadout with its hidden layer as Re(V h) on the split-TF32
    projections (and, when mean-pooled, the output layer after pooling)
    against the plain torch composition on [Re h; Im h]."""
    from prospective_rqf_b200 import encoder

    g = torch.Generator().manual_seed(13)
    F, H, C, B, T = 64, 96, 7, 3, 2048
    ro = encoder.ComplexReadout(F, C, H, seed=2).cuda()
    with torch.no_grad():  # an output layer large enough to matter in the gradients
        ro.fc2.weight.normal_(0.0, 0.1, generator=torch.Generator("cuda").manual_seed(3))
    h = _crandn(g, F, B, T).cuda()
    gout = torch.randn((B, T, C) if per_step else (B, C), generator=g).cuda()
    res = {}
    for mode in ("tc", "torch"):
        monkeypatch.setattr(encoder, "PROJECTION", mode)
        ro.zero_grad(set_to_none=True)
        hh = h.clone().requires_grad_(True)
        out = ro(hh, per_step=per_step)
        out.backward(gout)
        res[mode] = (out.detach(), hh.grad, {n: p.grad for n, p in ro.named_parameters()})
    assert_close(_np(res["tc"][0].cpu()), _np(res["torch"][0].cpu()), FWD_TOL, "logits")
    assert_close(_np(res["tc"][1].cpu()), _np(res["torch"][1].cpu()), GRAD_TOL, "grad h")
    for n in res["torch"][2]:
        assert_close(_np(res["tc"][2][n].cpu()), _np(res["torch"][2][n].cpu()), GRAD_TOL,
                     f"grad {n}")


@pytest.mark.parametrize("bias,skip,T", [(False, True, 4000), (True, True, 2000),
                                         (False, False, 4096), (True, False, 1004)])
def test_rank1_first_block_matches_general_path(bias, skip, T, monkeypatch):
    """The first block over a one-channel input on the rank-1 kernels
    (rqf_fbt_rank1_forward / _backward: drive and skip made from x inside
    the scan, no grad_z, the row sums reduced in the backward) against the
    same block on rqf_lowrank_drive + the (F,B,T) row kernels + rqf_rowdot:
    the features bit-identical (the same operations), logits and every
    parameter gradient within fp32 summation-order noise.  1024 rows, so the
    persistent row kernels apply; T a multiple of 4 with the last tile cut."""
    from prospective_rqf_b200 import _timing, ops
    from prospective_rqf_b200 import encoder as E

    def run(rank1):
        if not rank1:
            monkeypatch.setattr(ops, "rank1_supported", lambda *a: False)
        torch.manual_seed(0)
        enc = E.PureRQFEncoderB200(input_dims=1, hidden_dims=128, num_layers=2,
                                   skip_connection=skip, input_proj_bias=bias, seed=4)
        model = E.RQFClassifier(enc, 5, 32).cuda()
        g = torch.Generator().manual_seed(6)
        x = (0.5 * torch.randn(8, T, 1, generator=g)).clamp(-1, 1).cuda()
        y = torch.randint(0, 5, (8,), generator=g).cuda()
        with _timing.KernelTimer() as tm:
            feats = model.encoder(x)
            logits = model.readout(feats)
            torch.nn.functional.cross_entropy(logits, y).backward()
        grads = {n: p.grad.detach().clone() for n, p in model.named_parameters()}
        return feats.detach().clone(), logits.detach().clone(), grads, set(tm.summary())

    f1, l1, g1, k1 = run(True)
    assert {"rqf_fbt_rank1_forward", "rqf_fbt_rank1_backward"} <= k1
    f2, l2, g2, k2 = run(False)
    assert "rqf_fbt_rank1_forward" not in k2
    assert torch.equal(f1, f2), "features differ from the general first block"
    assert rel_err(l1.cpu().numpy(), l2.cpu().numpy()) <= 1e-6
    for n in g1:
        e = rel_err(g1[n].cpu().numpy(), g2[n].cpu().numpy())
        assert e <= 1e-4, f"{n}: {e:.2e}"


@pytest.mark.parametrize("bias,skip,T", [(False, True, 4000), (True, False, 1004)])
def test_rank1_first_block_tbptt_matches_general_path(bias, skip, T, monkeypatch):
    """The TBPTT(1) encoder's first layer over a one-channel input on the
    rank-1 kernels (rqf_fbt_rank1_forward, rqf_fbt_rank1_tbptt_backward: no
    grad_z, the row sums reduced in the backward) against rqf_lowrank_drive +
    the row forward + the torch skip add, the (F,B,T) TBPTT(1) kernel and
    rqf_rowdot: the features bit-identical, every parameter gradient within
    fp32 summation-order noise."""
    from prospective_rqf_b200 import _timing, ops
    from prospective_rqf_b200 import encoder as E

    def run(rank1):
        if not rank1:
            monkeypatch.setattr(ops, "rank1_supported", lambda *a: False)
        torch.manual_seed(0)
        enc = E.PureRQFEncoderB200(input_dims=1, hidden_dims=128, num_layers=2,
                                   skip_connection=skip, input_proj_bias=bias, seed=4,
                                   scan_grad_mode="tbptt1")
        model = E.RQFClassifier(enc, 5, 32).cuda()
        g = torch.Generator().manual_seed(6)
        x = (0.5 * torch.randn(8, T, 1, generator=g)).clamp(-1, 1).cuda()
        y = torch.randint(0, 5, (8,), generator=g).cuda()
        with _timing.KernelTimer() as tm:
            feats = model.encoder(x)
            logits = model.readout(feats)
            torch.nn.functional.cross_entropy(logits, y).backward()
        grads = {n: p.grad.detach().clone() for n, p in model.named_parameters()}
        return feats.detach().clone(), grads, set(tm.summary())

    f1, g1, k1 = run(True)
    assert {"rqf_fbt_rank1_forward", "rqf_fbt_rank1_tbptt_backward"} <= k1
    f2, g2, k2 = run(False)
    assert "rqf_fbt_rank1_forward" not in k2
    assert torch.equal(f1, f2), "features differ from the general first layer"
    for n in g1:
        e = rel_err(g1[n].cpu().numpy(), g2[n].cpu().numpy())
        assert e <= 1e-4, f"{n}: {e:.2e}"


@pytest.mark.parametrize("C,B,T,eps", [(35, 4, 1000, 0.1), (35, 3, 257, 0.0), (5, 2, 64, 0.3),
                                       (1, 2, 7, 0.1)])
def test_per_step_cross_entropy_matches_torch(C, B, T, eps):
    """rqf_per_step_cross_entropy and its backward against
    torch.nn.functional.cross_entropy on the (batch*time, classes) view of the
    same logits (train.py:per_step_cross_entropy :663-674): loss and logit
    gradient in fp64, for an upstream gradient other than one."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(C * 7 + B + T)
    logits = (3.0 * torch.randn(C, B * T, generator=g)).cuda().requires_grad_(True)
    y = torch.randint(0, C, (B,), generator=g).cuda()
    loss = ops.per_step_cross_entropy(logits, y, B, T, eps)
    (2.5 * loss).backward()
    ref_l = logits.detach().double().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(
        ref_l.t().reshape(B, T, C).reshape(B * T, C), y[:, None].expand(B, T).reshape(-1),
        label_smoothing=eps)
    (2.5 * ref).backward()
    lv, rv = float(loss.detach()), float(ref.detach())
    assert abs(lv - rv) <= 1e-6 * max(1.0, abs(rv))
    assert_close(logits.grad.cpu().numpy().astype(np.float64), ref_l.grad.cpu().numpy(), 1e-5,
                 "grad logits")


def test_tbptt_step_loss_matches_torch_cross_entropy():
    """The TBPTT(1) training step's loss through RQFClassifier.per_step_loss
    against torch's cross entropy of forward(x, per_step=True), and the same
    parameter gradients."""
    from prospective_rqf_b200 import encoder as E

    def run(fused):
        torch.manual_seed(0)
        enc = E.PureRQFEncoderB200(input_dims=1, hidden_dims=64, num_layers=2, seed=2,
                                   scan_grad_mode="tbptt1")
        model = E.RQFClassifier(enc, 7, 32).cuda()
        g = torch.Generator().manual_seed(3)
        x = (0.5 * torch.randn(4, 2048, 1, generator=g)).clamp(-1, 1).cuda()
        y = torch.randint(0, 7, (4,), generator=g).cuda()
        if fused:
            loss = model.per_step_loss(x, y, 0.1)
        else:
            logits = model(x, per_step=True)
            loss = torch.nn.functional.cross_entropy(
                logits.reshape(4 * 2048, 7), y[:, None].expand(4, 2048).reshape(-1),
                label_smoothing=0.1)
        loss.backward()
        return float(loss), {n: p.grad.detach().clone() for n, p in model.named_parameters()}

    l1, g1 = run(True)
    l2, g2 = run(False)
    assert abs(l1 - l2) <= 1e-6 * max(1.0, abs(l2))
    for n in g1:
        assert rel_err(g1[n].cpu().numpy(), g2[n].cpu().numpy()) <= 1e-4, n


@pytest.mark.parametrize("H,B,T", [(16, 3, 1000), (8, 2, 32), (5, 1, 70)])
def test_readout_bias_relu_matches_torch(H, B, T):
    """rqf_readout_bias_relu (in place) and its backward against
    relu(z + b) and the masked cotangent with its sum over (b, t): exact."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(H + B + T)
    z = torch.randn(H, B, T, generator=g).cuda()
    b = torch.randn(H, generator=g).cuda()
    gy = torch.randn(H, B, T, generator=g).cuda()
    ref = torch.relu(z + b[:, None, None])
    hid, mask = ops.readout_bias_relu(z.clone(), b)
    assert torch.equal(hid, ref)
    gr, rowsum = ops.readout_bias_relu_backward(gy, mask)
    want = gy * (z + b[:, None, None] > 0)
    assert torch.equal(gr, want)
    assert torch.allclose(rowsum.double(), want.double().sum(dim=2), rtol=1e-6, atol=1e-5)
