"""The benched model against the reference's own modules.

bench.py trains prospective_rqf_b200.encoder.RQFClassifier: PureRQFEncoderB200
(the (F,B,T) stack of rqf_models/backbones/rqf/pure.py:510-536 on this
backend's kernels, with its first block over the low-rank input) and
ComplexReadout (train.py:ComplexReadoutClassifier :74-136, mean-pooled or
per-step).  Here the reference's own parameters are loaded into it and the
results compared:

* with the reference's ComplexReadoutClassifier(PureRQFEncoder) run on the
  reference's CPU path (fixtures written by tests/golden/make_model_golden.py:
  width 64, depth 6, T = 4000 full BPTT with pooled logits, T = 2000 TBPTT(1)
  with per-step logits): logits, loss and every parameter gradient, with the
  first block on the low-rank path and on the general GEMM path;
* with the reference's PureRQFEncoder on its stock GPU path (its Triton
  kernels, from the offline install in baseline/_ref): the complex features
  and every parameter gradient of mean |h|^2, width 64, depth 6, B = 4,
  T = 4000, full BPTT and TBPTT(1).

Forward: normwise max relative error <= 1e-4; gradients <= 1e-3 (two fp32
implementations); the element-wise error (floor 1e-3 of the tensor's maximum)
is reported and bounded beside it.  Parameter gradients are sums over every
sample and step, so the split-ReLU derivative's few decisions that can differ
between two fp32 implementations (a state within rounding of zero) stay far
below these bounds.
"""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as tnf

from _util import (FWD_ELEM_TOL, FWD_TOL, GRAD_ELEM_TOL, GRAD_TOL, assert_close, golden)

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
TAU, FS = 0.0003125, 16000.0


def _ours(hidden, depth, classes, readout_hidden, mode):
    from prospective_rqf_b200.encoder import PureRQFEncoderB200, RQFClassifier

    enc = PureRQFEncoderB200(input_dims=1, hidden_dims=hidden, num_layers=depth,
                             samp_frequency=FS, tau=TAU, seq_duration=1.0,
                             skip_connection=True, final_activation=False,
                             input_proj_bias=False, scan_grad_mode=mode)
    return RQFClassifier(enc, classes, readout_hidden).cuda()


def _name_map(depth):
    """Reference parameter name -> (our module path, attribute)."""
    m = {"encoder.input_proj.weight": "encoder.input_proj.weight",
         "head.0.weight": "readout.fc1.weight", "head.0.bias": "readout.fc1.bias",
         "head.3.weight": "readout.fc2.weight", "head.3.bias": "readout.fc2.bias"}
    for i in range(depth):
        m[f"encoder.blocks.{i}.W"] = f"encoder.W.{i}"
        m[f"encoder.blocks.{i}.rqf_fwd.log_theta"] = f"encoder.rqf.{i}.log_theta"
        m[f"encoder.blocks.{i}.rqf_fwd.log_gamma"] = f"encoder.rqf.{i}.log_gamma"
    return m


def _load(model, params, depth):
    ours = dict(model.named_parameters())
    with torch.no_grad():
        for ref_name, our_name in _name_map(depth).items():
            ours[our_name].copy_(torch.from_numpy(np.asarray(params[ref_name])))


@pytest.mark.parametrize("first_block", ["lowrank", "gemm"])
@pytest.mark.parametrize("case", ["model_full", "model_tbptt1"])
def test_classifier_matches_reference_fixture(case, first_block):
    g = golden(case)
    hidden, depth, batch, time, rh, classes, per_step = (int(v) for v in g["config"])
    for i in range(depth):  # the reference's fixed tau and dt are ours
        assert np.allclose(g[f"buffer/encoder.blocks.{i}.rqf_fwd._min_gamma"], 1e-6)
        np.testing.assert_allclose(g[f"param/encoder.blocks.{i}.rqf_fwd.log_tau"],
                                   np.log(np.float32(TAU)), rtol=1e-6)
    mode = "tbptt1" if per_step else "full"
    model = _ours(hidden, depth, classes, rh, mode)
    params = {k[len("param/"):]: g[k] for k in g.files if k.startswith("param/")}
    _load(model, params, depth)
    model.train()

    x = torch.from_numpy(g["x"]).cuda()
    if first_block == "gemm":  # an input that needs a gradient takes the general first block
        x.requires_grad_(True)
    y = torch.from_numpy(g["y"]).cuda()
    logits = model(x, per_step=bool(per_step))
    if per_step:
        b, t, c = logits.shape
        loss = tnf.cross_entropy(logits.reshape(b * t, c), y[:, None].expand(b, t).reshape(-1))
    else:
        loss = tnf.cross_entropy(logits, y)
    loss.backward()

    assert_close(logits.detach().cpu().numpy(), g["logits"], FWD_TOL, "logits",
                 elem_tol=FWD_ELEM_TOL)
    assert abs(loss.item() - float(g["loss"])) <= FWD_TOL * abs(float(g["loss"]))
    ours = dict(model.named_parameters())
    names = [k[len("grad/"):] for k in g.files if k.startswith("grad/")]
    assert set(names) == set(_name_map(depth)), sorted(set(names) ^ set(_name_map(depth)))
    for ref_name in names:
        got = ours[_name_map(depth)[ref_name]].grad
        assert got is not None, f"no gradient for {ref_name}"
        assert_close(got.cpu().numpy(), g["grad/" + ref_name], GRAD_TOL, ref_name,
                     elem_tol=GRAD_ELEM_TOL)


def _reference_encoder(hidden, depth, mode):
    if not (REF / "rqf_models").exists():
        pytest.skip("reference install (baseline/_ref) absent")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from rqf_models.backbones.rqf.pure import PureRQFEncoder

    torch.manual_seed(0)
    return PureRQFEncoder(
        input_dims=1, output_dims=8, hidden_dims=hidden, num_layers=depth,
        samp_frequency=FS, min_freq=1.0, max_freq=8000.0, tau=TAU, discretization="zoh",
        activation="split_relu", complex_weights=True, param_space="log", seq_duration=1.0,
        w_init="forward", final_activation=False, input_proj_bias=False,
        complex_output=True, prospective_input=True, prospective_mode="tau",
        skip_connection=True, scan_grad_mode=mode).cuda()


@pytest.mark.parametrize("first_block", ["lowrank", "gemm"])
@pytest.mark.parametrize("mode", ["full", "tbptt1"])
def test_encoder_matches_reference_stock_gpu_path(mode, first_block):
    import prospective_rqf_b200 as rqf

    rqf.uninstall()  # the reference on its own Triton kernels
    hidden, depth, batch, time = 64, 6, 4, 4000
    ref = _reference_encoder(hidden, depth, mode)
    ours = _ours(hidden, depth, 8, 16, mode).encoder
    params = {"encoder." + n: p.detach().cpu().numpy() for n, p in ref.named_parameters()}
    _load_encoder = {k: v for k, v in _name_map(depth).items() if k.startswith("encoder.")}
    with torch.no_grad():
        mine = dict(ours.named_parameters())
        for ref_name, our_name in _load_encoder.items():
            mine[our_name[len("encoder."):]].copy_(torch.from_numpy(params[ref_name]))

    gen = torch.Generator(device="cuda").manual_seed(5)
    x = 0.5 * torch.randn(batch, time, 1, device="cuda", generator=gen)

    # The loss of the other drop-in comparisons, mean |h|^2: its cotangent
    # follows the features, as a trained model's does.  (A random cotangent
    # makes every leaf gradient a sum of B*T terms of random sign that cancel
    # to ~1/sqrt(B*T) of their size, which both fp32 implementations round
    # at the 1e-3 level.)
    feats_ref = ref(x)  # (B, T, F) complex
    (feats_ref.abs() ** 2).mean().backward()
    xo = x.clone().requires_grad_(first_block == "gemm")
    feats = ours(xo)    # (F, B, T) complex
    (feats.abs() ** 2).mean().backward()

    errs = {"features": assert_close(feats.detach().permute(1, 2, 0).cpu().numpy(),
                                     feats_ref.detach().cpu().numpy(), FWD_TOL, "features",
                                     elem_tol=FWD_ELEM_TOL)}
    mine = dict(ours.named_parameters())
    refp = dict(ref.named_parameters())
    bad = []
    for ref_name, our_name in _load_encoder.items():
        a = mine[our_name[len("encoder."):]].grad
        b = refp[ref_name[len("encoder."):]].grad
        assert a is not None and b is not None, ref_name
        try:
            errs[ref_name] = assert_close(a.cpu().numpy(), b.cpu().numpy(), GRAD_TOL, ref_name,
                                          elem_tol=GRAD_ELEM_TOL)
        except AssertionError as exc:
            bad.append(str(exc))
    print({k: f"{v[0]:.2e} / {v[1]:.2e}" for k, v in errs.items()})
    assert not bad, bad
