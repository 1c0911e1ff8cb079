"""Informational timing of the reference's own paths beside this backend on the
same machine:
- its GPU path (its Triton kernels and its Pure RQF encoder) on the same B200,
  same shapes, same CUDA-event method;
- its CPU PyTorch path on the box's host cores (config 1: sequential_scan
  forward + backward on the exact benchmark tensors; config-2 scale:
  parallel_scan on one batch row), beside this backend's GPU op.

The reference comes from its offline install:

    python -m pip install --no-index --no-build-isolation --no-deps \\
        --find-links /opt/wheelhouse --target baseline/_ref <copy of the reference tree>

Run from the repository root on a GPU box:

    python benchmarks/reference_paths.py

Prints one JSON object: milliseconds per forward+backward (or per pass) for
each workload, "reference_triton" beside "b200", and the largest relative
difference of the selective scan's output between the two.  Op-level detail
for every configuration; bench.py carries the headline comparison (the full
training step and the workload's layer scan) in the line the driver records.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
sys.path.insert(0, str(ROOT))
os.environ.setdefault("TRITON_CACHE_DIR", "/tmp/triton_cache")

import torch  # noqa: E402

DEV = "cuda"


def timed(fn, warmup=3, iters=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return round(e0.elapsed_time(e1) / iters, 4)


def coeffs(F, g):
    mag = 0.9 + 0.0999 * torch.rand(F, generator=g)
    lam = torch.polar(mag, 6.283 * torch.rand(F, generator=g)).to(torch.complex64)
    t0 = 0.3 * torch.randn(F, dtype=torch.complex64, generator=g)
    t1 = 0.3 * torch.randn(F, dtype=torch.complex64, generator=g)
    return lam.to(DEV), t0.to(DEV), t1.to(DEV)


def fwd_bwd(op, args, z):
    zz = z.detach().requires_grad_(True)
    gy = torch.randn_like(z)

    def run():
        y = op(*args, zz)
        torch.autograd.grad(y, (zz,), gy)
    return run


def scans(out):
    import prospective_rqf_b200 as ours
    from rqf_models.ops.chunked_scan_kernel import (
        _triton_chunked_scan as ref_chunk,
        _triton_chunked_scan_prospective as ref_pro,
    )
    from rqf_models.ops.fbt_scan_kernel import fbt_recompute_scan as ref_fbt

    g = torch.Generator().manual_seed(0)
    c1, t0, t1 = coeffs(256, g)
    z = torch.randn(256, 32, 16000, dtype=torch.complex64, device=DEV)
    out["fbt_recompute_scan F256 B32 T16000 fwd+bwd"] = {
        "reference_triton": timed(fwd_bwd(ref_fbt, (c1, t0, t1), z)),
        "b200": timed(fwd_bwd(ours.fbt_recompute_scan, (c1, t0, t1), z))}
    del z
    c1, t0, _ = coeffs(32, g)
    u = torch.randn(16, 16384, 32, dtype=torch.complex64, device=DEV)
    out["_triton_chunked_scan B16 T16384 F32 fwd+bwd"] = {
        "reference_triton": timed(fwd_bwd(ref_chunk, (c1, t0), u)),
        "b200": timed(fwd_bwd(ours._triton_chunked_scan, (c1, t0), u))}
    c1, t0, t1 = coeffs(64, g)
    u = torch.randn(16, 16384, 64, dtype=torch.complex64, device=DEV)
    out["_triton_chunked_scan_prospective B16 T16384 F64 fwd+bwd"] = {
        "reference_triton": timed(fwd_bwd(ref_pro, (c1, t0, t1), u)),
        "b200": timed(fwd_bwd(ours._triton_chunked_scan_prospective, (c1, t0, t1), u))}


def selective(out):
    import prospective_rqf_b200 as ours
    from rqf_models.ops import selective_scan_kernel as sk
    from rqf_models.ops.selective_scan import SelectiveScanInputs

    F, B, T, G = 256, 32, 4096, 8
    g = torch.Generator().manual_seed(0)
    theta = (0.05 + 2 * torch.rand(F, generator=g)).to(DEV)
    tensors = (torch.randn(F, B, T, generator=g).to(DEV), torch.randn(G, B, T, generator=g).to(DEV),
               torch.randn(F, B, T, generator=g).to(DEV), torch.randn(F, generator=g).to(DEV),
               theta, torch.randint(0, G, (F,), generator=g).to(DEV),
               torch.full((F,), 1e-6, device=DEV), torch.full((F,), 1 - 2e-6, device=DEV),
               torch.full((F,), 0.2, device=DEV), torch.ones(F, device=DEV), theta * 0.4,
               theta * 1.6)
    options = (True, True, True, False, 0.223, 0.223, True, False, True, 2.0, 0.0, True)
    ref_in = SelectiveScanInputs(*tensors, options)
    our_in = tensors + (options,)
    z = torch.randn(F, B, T, dtype=torch.complex64, device=DEV)
    gy, gx = torch.randn_like(z), torch.randn_like(z)
    chunk = 256  # the reference's default for T >= 256 (selective_scan.py:213-214)
    raw_r, _, ent_r = sk.selective_forward(z, ref_in, True, True, chunk)
    raw_o, _, ent_o = ours.selective_forward(z, our_in, True, True, None)
    key = "selective F256 B32 T4096 G8 (all controllers, prospective)"
    out[key + " forward"] = {
        "reference_triton": timed(lambda: sk.selective_forward(z, ref_in, True, True, chunk), 3, 10),
        "b200": timed(lambda: ours.selective_forward(z, our_in, True, True, None), 3, 10)}
    out[key + " backward"] = {
        "reference_triton": timed(
            lambda: sk.selective_backward(z, ref_in, ent_r, gy, gx, True, False, chunk), 3, 10),
        "b200": timed(
            lambda: ours.selective_backward(z, our_in, ent_o, gy, gx, True, False, None), 3, 10)}
    out[key + " max relative difference of raw"] = float(
        ((raw_o - raw_r).abs().max() / raw_r.abs().max()).item())


def encoder(out):
    from rqf_models.backbones.rqf.pure import PureRQFEncoder

    from prospective_rqf_b200.encoder import PureRQFEncoderB200

    B, T, H = 32, 16000, 256
    # configs/model/pure_rqf_paper.yaml with benchmark config 5's width, depth and skip
    ref = PureRQFEncoder(input_dims=1, output_dims=32, hidden_dims=H, num_layers=6,
                         samp_frequency=16000.0, min_freq=1.0, max_freq=8000.0, tau=0.0003125,
                         discretization="zoh", activation="split_relu", complex_weights=True,
                         param_space="log", seq_duration=1.0, w_init="forward",
                         final_activation=False, input_proj_bias=False, complex_output=True,
                         prospective_input=True, prospective_mode="tau",
                         skip_connection=True).to(DEV)
    mine = PureRQFEncoderB200(input_dims=1, hidden_dims=H, num_layers=6, samp_frequency=16000.0,
                              tau=0.0003125, skip_connection=True, final_activation=False,
                              input_proj_bias=False).to(DEV)
    x = torch.randn(B, T, 1, device=DEV)

    def step(model):
        def run():
            model(x).abs().mean().backward()
        return run
    out["Pure RQF encoder B32 T16000 H256 depth6 fwd+bwd"] = {
        "reference_triton": timed(step(ref), 2, 3), "b200": timed(step(mine), 2, 3)}


def cpu_reference(out):
    """The reference's CPU PyTorch scans, timed on this host (all cores)."""
    import time

    import prospective_rqf_b200 as ours
    from rqf_models.ops.scan import parallel_scan, sequential_scan

    torch.set_num_threads(os.cpu_count() or 1)
    out["host_threads"] = torch.get_num_threads()

    def wall(fn, reps):
        fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return round((time.perf_counter() - t0) / reps * 1e3, 3)

    # config 1: u real N(0,1) [32,161,128]; lambda = r e^{i theta}, r ~ U(0.90, 0.999),
    # theta ~ U(0, pi); b ~ CN(0,1); loss sum |y|^2
    g = torch.Generator().manual_seed(0)
    B, T, H = 32, 161, 128
    u = torch.randn(B, T, H, generator=g)
    r = 0.90 + 0.099 * torch.rand(H, generator=g)
    lam = torch.polar(r, torch.pi * torch.rand(H, generator=g)).to(torch.complex64)
    b = (torch.randn(H, generator=g) + 1j * torch.randn(H, generator=g)).to(torch.complex64) / 2 ** 0.5

    def step(op, c1, c2, x):
        def run():
            xx = x.detach().requires_grad_(True)
            c1g, c2g = c1.detach().requires_grad_(True), c2.detach().requires_grad_(True)
            y = op(c1g, c2g, xx)
            (y.abs() ** 2).sum().backward()
        return run
    cpu_ms = wall(step(sequential_scan, lam, b, u), 3)
    gpu_ms = timed(step(ours.sequential_scan, lam.to(DEV), b.to(DEV), u.to(DEV)), 3, 10)
    out["config 1 sequential_scan B32 T161 H128 real u, fwd+bwd"] = {
        "reference_cpu": cpu_ms, "b200": gpu_ms}
    # config-2 scale, one batch row: complex u [1,16000,128], parallel_scan (Blelloch)
    u2 = (torch.randn(1, 16000, 128, generator=g) + 1j * torch.randn(1, 16000, 128, generator=g)).to(torch.complex64)
    lam2 = torch.polar(0.9 + 0.099 * torch.rand(128, generator=g), torch.pi * torch.rand(128, generator=g)).to(torch.complex64)
    cpu_ms = wall(step(parallel_scan, lam2, b, u2), 1)
    gpu_ms = timed(step(ours.parallel_scan, lam2.to(DEV), b.to(DEV), u2.to(DEV)), 3, 10)
    out["parallel_scan B1 T16000 H128 complex u, fwd+bwd"] = {"reference_cpu": cpu_ms, "b200": gpu_ms}


def main():
    out = {"unit": "ms", "device": torch.cuda.get_device_name()}
    scans(out)
    selective(out)
    encoder(out)
    cpu_reference(out)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
