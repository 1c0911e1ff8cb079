"""Generate the golden vectors that pin the oracle to the reference.

Run in a container that has the reference tree (read-only) available:

    python tests/golden/make_golden.py --reference /path/to/prospective-rqf

Every fixture is produced by calling the REFERENCE implementation
(rqf_models from the reference tree) on seeded inputs:

* fp64 PyTorch paths (CPU): rqf_models/ops/scan.py:parallel_scan (:435,
  Blelloch, honours complex128), BaseRQFBlock._apply_prospective_taps
  (block.py:644) and BaseRQFBlock._scan_two_tap_with_grad_mode (block.py:904)
  for TBPTT(1); gradients by torch autograd through those paths.
* the reference's own Triton kernels run by the Triton CPU interpreter
  (TRITON_INTERPRET=1, fp32): chunked_scan_kernel._triton_chunked_scan,
  _triton_chunked_scan_prospective, fbt_scan_kernel.fbt_recompute_scan and
  fbt_prospective_scan.
* scan.py:sequential_scan on CPU (fp32), the config-1 benchmark entry point.

Outputs: tests/golden/*.npz (small; committed).  Nothing at test time reads
the reference tree.
"""

from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _np(t):
    return t.detach().cpu().numpy()


def _coeffs(num_filters, seed, dtype):
    """Coefficient draw of the reference parity suite
    (tests/test_scan_backends_parity.py:_coeffs, :25-31)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    mag = 0.8 + 0.19 * torch.rand(num_filters, generator=g, dtype=torch.float64)
    phase = 2 * torch.pi * torch.rand(num_filters, generator=g, dtype=torch.float64)
    c1 = (mag * torch.exp(1j * phase)).to(dtype)
    c2 = 0.1 * torch.randn(num_filters, 2, generator=g, dtype=torch.float64)
    return c1, torch.complex(c2[:, 0], c2[:, 1]).to(dtype)


def _taps(num_filters, seed, dtype):
    import torch

    g = torch.Generator().manual_seed(seed)
    t0 = torch.complex(0.5 * torch.randn(num_filters, generator=g, dtype=torch.float64),
                       0.5 * torch.randn(num_filters, generator=g, dtype=torch.float64))
    t1 = torch.complex(0.5 * torch.randn(num_filters, generator=g, dtype=torch.float64),
                       0.5 * torch.randn(num_filters, generator=g, dtype=torch.float64))
    return t0.to(dtype), t1.to(dtype)


def _crandn(shape, seed, dtype):
    """complex normal with float32-representable parts (exact in fp32 and fp64)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    re = torch.randn(*shape, generator=g).double()
    im = torch.randn(*shape, generator=g).double()
    return torch.complex(re, im).to(dtype)


def _grads(fn, inputs, cot):
    import torch

    args = [a.clone().requires_grad_(True) for a in inputs]
    y = fn(*args)
    y.backward(cot)
    return y, [a.grad for a in args]


def case_scan_complex(out):
    """Single-tap scan, complex u, (B,T,F): fp64 parallel_scan (Blelloch)."""
    import torch
    from rqf_models.ops.scan import parallel_scan

    B, T, F = 2, 37, 5
    c1, c2 = _coeffs(F, 0, torch.complex128)
    u = _crandn((B, T, F), 1, torch.complex128)
    gy = _crandn((B, T, F), 2, torch.complex128)
    y, (gc1, gc2, gu) = _grads(lambda a, b, c: parallel_scan(a, b, c), [c1, c2, u], gy)
    np.savez(out / "scan_complex.npz", c1=_np(c1), c2=_np(c2), u=_np(u), gy=_np(gy), y=_np(y),
             gc1=_np(gc1), gc2=_np(gc2), gu=_np(gu))


def case_scan_real_cfg1(out):
    """Config 1 generator at reduced size: real u ~ N(0,1),
    lambda = r e^{i theta}, r ~ U(0.90, 0.999), theta ~ U(0, pi),
    b ~ CN(0,1)/sqrt(2), loss = sum |y|^2.  Reference: scan.py:sequential_scan
    on CPU (fp32) and parallel_scan with complex128 coefficients (fp64)."""
    import torch
    from rqf_models.ops.scan import parallel_scan, sequential_scan

    B, T, F = 3, 161, 8
    g = torch.Generator().manual_seed(11)
    r = 0.90 + 0.099 * torch.rand(F, generator=g, dtype=torch.float64)
    th = torch.pi * torch.rand(F, generator=g, dtype=torch.float64)
    lam = (r * torch.exp(1j * th)).to(torch.complex64).to(torch.complex128)
    b = torch.complex(torch.randn(F, generator=g), torch.randn(F, generator=g)) / np.sqrt(2.0)
    b = b.to(torch.complex64).to(torch.complex128)
    u = torch.randn(B, T, F, generator=g).double()

    def loss64(lam_, b_, u_):
        y = parallel_scan(lam_, b_, u_)
        return (y.real ** 2 + y.imag ** 2).sum(), y

    args = [a.clone().requires_grad_(True) for a in (lam, b, u)]
    loss, y = loss64(*args)
    loss.backward()
    args32 = [lam.to(torch.complex64).requires_grad_(True), b.to(torch.complex64).requires_grad_(True),
              u.float().requires_grad_(True)]
    y32 = sequential_scan(*args32)
    (y32.real ** 2 + y32.imag ** 2).sum().backward()
    np.savez(out / "scan_real_cfg1.npz", c1=_np(lam), c2=_np(b), u=_np(u), y=_np(y),
             gc1=_np(args[0].grad), gc2=_np(args[1].grad), gu=_np(args[2].grad),
             y32=_np(y32), gc1_32=_np(args32[0].grad), gc2_32=_np(args32[1].grad),
             gu_32=_np(args32[2].grad))


def case_prospective_btf(out):
    """Two-tap scan in (B,T,F): drive materialised by block.py
    _apply_prospective_taps then parallel_scan with unit gain (fp64)."""
    import torch
    from rqf_models.backbones.rqf.block import BaseRQFBlock
    from rqf_models.ops.scan import parallel_scan

    B, T, F = 2, 300, 6
    c1, _ = _coeffs(F, 3, torch.complex128)
    t0, t1 = _taps(F, 3, torch.complex128)
    x = _crandn((B, T, F), 4, torch.complex128)
    gy = _crandn((B, T, F), 5, torch.complex128)

    def fn(c1_, t0_, t1_, x_):
        drive = BaseRQFBlock._apply_prospective_taps(x_, t0_, t1_)
        return parallel_scan(c1_, torch.ones_like(c1_), drive)

    y, (gc1, gt0, gt1, gx) = _grads(fn, [c1, t0, t1, x], gy)
    np.savez(out / "prospective_btf.npz", c1=_np(c1), tap0=_np(t0), tap1=_np(t1), x=_np(x),
             gy=_np(gy), y=_np(y), gc1=_np(gc1), gt0=_np(gt0), gt1=_np(gt1), gx=_np(gx))


def case_fbt(out, fuse_act):
    """Two-tap scan in (F,B,T) with/without split-ReLU: fp64 PyTorch path and
    the reference Triton kernel (fbt_recompute_scan / fbt_prospective_scan)
    under the Triton CPU interpreter (fp32)."""
    import torch
    from rqf_models.backbones.rqf.block import BaseRQFBlock
    from rqf_models.ops.fbt_scan_kernel import fbt_prospective_scan, fbt_recompute_scan
    from rqf_models.ops.scan import parallel_scan

    F, B, T = 2, 2, 2100
    c1, _ = _coeffs(F, 6, torch.complex128)
    t0, t1 = _taps(F, 6, torch.complex128)
    z = _crandn((F, B, T), 7, torch.complex128)
    gy = _crandn((F, B, T), 8, torch.complex128)

    def fn64(c1_, t0_, t1_, z_):
        x = z_.permute(1, 2, 0)
        drive = BaseRQFBlock._apply_prospective_taps(x, t0_, t1_)
        y = parallel_scan(c1_, torch.ones_like(c1_), drive).permute(2, 0, 1)
        return torch.complex(y.real.relu(), y.imag.relu()) if fuse_act else y

    y, (gc1, gt0, gt1, gz) = _grads(fn64, [c1, t0, t1, z], gy)
    if fuse_act:
        tri = lambda a, b, c, d: fbt_recompute_scan(a, b, c, d)  # noqa: E731
    else:
        tri = lambda a, b, c, d: fbt_prospective_scan(a, b, c, d, False)  # noqa: E731
    y32, (gc1_32, gt0_32, gt1_32, gz_32) = _grads(
        tri, [c1.to(torch.complex64), t0.to(torch.complex64), t1.to(torch.complex64),
              z.to(torch.complex64)], gy.to(torch.complex64))
    name = "fbt_split_relu" if fuse_act else "fbt_raw"
    np.savez(out / f"{name}.npz", c1=_np(c1), tap0=_np(t0), tap1=_np(t1), z=_np(z), gy=_np(gy),
             y=_np(y), gc1=_np(gc1), gt0=_np(gt0), gt1=_np(gt1), gz=_np(gz), y32=_np(y32),
             gc1_32=_np(gc1_32), gt0_32=_np(gt0_32), gt1_32=_np(gt1_32), gz_32=_np(gz_32))


def case_triton_btf(out):
    """Reference Triton kernels (interpreter, fp32) in (B,T,F): plain and
    prospective, at a length that spans several reference chunks."""
    import torch
    from rqf_models.ops.chunked_scan_kernel import (
        _triton_chunked_scan,
        _triton_chunked_scan_prospective,
    )

    B, T, F = 2, 1023, 8
    c1, c2 = _coeffs(F, 9, torch.complex64)
    t0, t1 = _taps(F, 9, torch.complex64)
    u = _crandn((B, T, F), 10, torch.complex64)
    gy = _crandn((B, T, F), 12, torch.complex64)
    y, (gc1, gc2, gu) = _grads(_triton_chunked_scan, [c1, c2, u], gy)
    yp, (pgc1, pgt0, pgt1, pgx) = _grads(_triton_chunked_scan_prospective, [c1, t0, t1, u], gy)
    np.savez(out / "triton_btf.npz", c1=_np(c1), c2=_np(c2), tap0=_np(t0), tap1=_np(t1),
             u=_np(u), gy=_np(gy), y=_np(y), gc1=_np(gc1), gc2=_np(gc2), gu=_np(gu), yp=_np(yp),
             pgc1=_np(pgc1), pgt0=_np(pgt0), pgt1=_np(pgt1), pgx=_np(pgx))


def case_tbptt(out):
    """TBPTT(1) two-tap surrogate: the reference's own
    BaseRQFBlock._scan_two_tap_with_grad_mode (block.py:904-954), fp64, with
    and without a separate lag source delayed_u."""
    import torch
    from rqf_models.backbones.rqf.block import BaseRQFBlock
    from rqf_models.ops.scan import parallel_scan

    fake = types.SimpleNamespace()
    fake._use_tbptt1_scan_grad = lambda: True
    fake._scan = lambda u, c1, c2: parallel_scan(c1, c2, u)
    fake._apply_prospective_taps = BaseRQFBlock._apply_prospective_taps
    fake._shift_states = BaseRQFBlock._shift_states

    B, T, F = 2, 200, 5
    c1, _ = _coeffs(F, 13, torch.complex128)
    t0, t1 = _taps(F, 13, torch.complex128)
    u = _crandn((B, T, F), 14, torch.complex128)
    gy = _crandn((B, T, F), 15, torch.complex128)

    def with_lag(c1_, t0_, t1_, u_, d_):
        return BaseRQFBlock._scan_two_tap_with_grad_mode(fake, u_, c1_, t0_, t1_, delayed_u=d_)

    y, (gc1, gt0, gt1, gu, gd) = _grads(with_lag, [c1, t0, t1, u, u.clone()], gy)

    def no_lag(c1_, t0_, t1_, u_):
        return BaseRQFBlock._scan_two_tap_with_grad_mode(fake, u_, c1_, t0_, t1_)

    y2, (gc1b, gt0b, gt1b, gub) = _grads(no_lag, [c1, t0, t1, u], gy)
    np.savez(out / "tbptt.npz", c1=_np(c1), tap0=_np(t0), tap1=_np(t1), u=_np(u), gy=_np(gy),
             y=_np(y), gc1=_np(gc1), gt0=_np(gt0), gt1=_np(gt1), gu=_np(gu), gd=_np(gd),
             y_nolag=_np(y2), gc1_nolag=_np(gc1b), gt0_nolag=_np(gt0b), gt1_nolag=_np(gt1b),
             gu_nolag=_np(gub))


SELECTIVE_CASES = [
    # (controller config, prospective, truncated, horizon mode)
    ({}, True, False, "tau"),
    ({"gamma_link": "log_shift"}, True, False, "tau"),
    ({"gamma_control": False, "write_control": True}, True, False, "tau"),
    ({"gamma_control": False, "write_control": True, "write_link": "affine"}, False, False, "tau"),
    ({"gamma_control": False, "frequency_warp": "global"}, True, False, "tau"),
    ({"frequency_warp": "grouped", "num_groups": 3, "write_control": True}, True, False, "tau"),
    ({"frequency_warp": "grouped", "num_groups": 3, "write_control": True}, True, True, "tau"),
    ({"frequency_warp": "global", "write_control": True, "gamma_link": "log_shift"}, True, False,
     "gamma"),
    ({"frequency_warp": "grouped", "num_groups": 3, "warp_bound": "none"}, False, True, "tau"),
    ({"write_control": True}, True, True, "gamma"),
]


def case_selective(out, reference):
    """Selective scan: the reference's reference_layer_scan (selective_scan.py
    :71-104) in fp64 with autograd, on SelectiveScanInputs built by the
    reference's own SelectiveController (the model/test helpers of
    tests/test_selective_rqf.py).  Weight = identity so z = x; in truncated
    mode the lag cotangent reaches only the weight gradient."""
    import torch

    sys.path.insert(0, os.path.join(reference, "tests"))
    from rqf_models.ops.selective_scan import reference_layer_scan
    from test_selective_rqf import inputs_for, make_model

    fields = ("gamma_logits", "warp_logits", "write_logits", "bias", "theta")
    for ci, (cfg, prospective, truncated, mode) in enumerate(SELECTIVE_CASES):
        blk = make_model(cfg, active=True, num_layers=1, prospective_input=prospective,
                         prospective_mode=mode, samp_frequency=100.0).blocks[0].double()
        F = blk.W.shape[0]
        B, T = 2, 37
        g = torch.Generator().manual_seed(100 + ci)

        def cplx(*shape):
            return torch.complex(torch.randn(*shape, generator=g, dtype=torch.float64),
                                 torch.randn(*shape, generator=g, dtype=torch.float64))

        x = cplx(blk.W.shape[1], B, T)
        with torch.no_grad():
            inputs = inputs_for(blk, x)
        leaves = {k: getattr(inputs, k).detach().clone().requires_grad_(True) for k in fields}
        inp = inputs._replace(**leaves)
        z = cplx(F, B, T).requires_grad_(True)
        weight = torch.eye(F, dtype=torch.complex128).requires_grad_(True)
        raw, act = reference_layer_scan(z, weight, inp, truncated=truncated, activate=True,
                                        write_raw=True)
        gy, gx = cplx(F, B, T), cplx(F, B, T)
        loss = (gy.conj() * raw).real.sum() + (gx.conj() * act).real.sum()
        loss.backward()

        def arr(t):
            return np.zeros(0) if t is None or t.numel() == 0 else _np(t)

        opt = np.array([float(v) for v in inputs.options])
        np.savez(out / f"selective_{ci}.npz", z=_np(z), gy=_np(gy), gx=_np(gx), raw=_np(raw),
                 act=_np(act), dz=_np(z.grad), dweight=_np(weight.grad),
                 gamma_logits=arr(inputs.gamma_logits), warp_logits=arr(inputs.warp_logits),
                 write_logits=arr(inputs.write_logits), bias=_np(inputs.bias),
                 theta=_np(inputs.theta),
                 groups=np.zeros(0, np.int64) if inputs.groups is None else _np(inputs.groups),
                 minimum=_np(inputs.minimum), span=_np(inputs.span), step=_np(inputs.step),
                 horizon=_np(inputs.horizon), theta_minimum=_np(inputs.theta_minimum),
                 theta_maximum=_np(inputs.theta_maximum), options=opt,
                 truncated=np.array(truncated),
                 dG=arr(leaves["gamma_logits"].grad), dD=arr(leaves["warp_logits"].grad),
                 dW=arr(leaves["write_logits"].grad), dbias=_np(leaves["bias"].grad),
                 dtheta=_np(leaves["theta"].grad))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RQF_REFERENCE", ""))
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    if not args.reference:
        sys.exit("pass --reference <path to the reference project>")
    # The reference's Triton kernels run on CPU tensors under the interpreter.
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, args.reference)
    import torch

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = Path(args.out)
    case_scan_complex(out)
    case_scan_real_cfg1(out)
    case_prospective_btf(out)
    case_fbt(out, fuse_act=True)
    case_fbt(out, fuse_act=False)
    case_triton_btf(out)
    case_tbptt(out)
    case_selective(out, args.reference)
    print("golden vectors written to", out)


if __name__ == "__main__":
    main()
