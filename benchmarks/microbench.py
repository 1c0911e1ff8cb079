"""Op-level timing of the scan kernels: one forward and one backward of a
public op per iteration on seeded synthetic inputs, each C-ABI call timed with
CUDA events on its launching stream, reported as milliseconds per launch and
achieved algorithmic bandwidth against the measured HBM copy peak.

    python benchmarks/microbench.py --op fbt --F 256 --B 32 --T 16000

Ops:
  fbt        fbt_recompute_scan (split-ReLU fused), (F,B,T)
  fbt_raw    fbt_prospective_scan without activation, (F,B,T)
  fbt_skip   the Pure RQF block scan: split-ReLU output plus the fused skip
             input (rqf_fbt_block_forward) and its backward
  tbptt_fbt  tbptt1_two_tap_scan, (F,B,T), split-ReLU fused
  tbptt_btf  tbptt1_two_tap_scan, (B,T,F)
  btf        _triton_chunked_scan, complex input, (B,T,F)
  btf_real   _triton_chunked_scan, real input, (B,T,F)
  btf_pro    _triton_chunked_scan_prospective, (B,T,F)
  selective  selective_forward + selective_backward with every controller on
  selective_bf16  the same in the bf16 storage mode (bf16 logits, raw / act and
             logit cotangents)
             (--groups warp groups, --truncated for the TBPTT(1) variant)
  projection the block projection z = W h, its input cotangent W^H gz + g and
             its weight cotangent gz h^H (split-TF32 tcgen05 GEMMs, W of F x F
             complex); reports TFLOP/s (8 F^2 B T real flops per GEMM)
  projection_torch  the same two GEMMs through torch.matmul (cuBLAS fp32)
  block_scan the Pure RQF block forward fused into its projection
             (rqf_projection_block_scan, skip = h, split-ReLU), beside the
             unfused pair it replaces: rqf_projection, then rqf_fbt_block_forward
  block_scan_bwd  the backward of two stacked blocks in one launch
             (rqf_projection_block_scan_backward: W^H gz + acc with the lower
             block's scan VJP in the epilogue), beside the unfused pair:
             rqf_projection, then rqf_fbt_prospective_backward
  rank1      the first Pure RQF block over a one-channel input (drive and skip
             made from x inside the row scan; rqf_fbt_rank1_forward / _backward)
  mosc       the fused multi-oscillator scan (B,T,F) -> (B,T,F), --groups
             oscillators per filter

--btf-path forces one (B,T,F) kernel family (1 streaming, 2 tile-resident).

Every tensor is at least --T x --B x --F complex64; the shapes used for the
committed figures exceed the 126 MB L2, so the timings read HBM.
"""

from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from bench import hbm_peak, measured_peaks  # noqa: E402


def _coeffs(F, dev, g):
    mag = 0.9 + 0.0999 * torch.rand(F, generator=g)
    lam = torch.polar(mag, 2 * math.pi * torch.rand(F, generator=g)).to(torch.complex64)
    t0 = (0.3 * torch.randn(F, dtype=torch.complex64, generator=g))
    t1 = (0.3 * torch.randn(F, dtype=torch.complex64, generator=g))
    return lam.to(dev), t0.to(dev), t1.to(dev)


def make_case(op: str, F: int, B: int, T: int, groups: int = 8, truncated: bool = False):
    """Returns run() performing one forward + backward of `op`."""
    import prospective_rqf_b200 as rqf
    from prospective_rqf_b200 import ops

    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(0)
    c1, t0, t1 = _coeffs(F, dev, g)

    def crandn(*shape):
        return torch.randn(*shape, dtype=torch.complex64, generator=g).to(dev)

    if op in ("selective", "selective_bf16"):
        G = groups
        theta = (0.05 + 2 * torch.rand(F, generator=g)).to(dev)
        inputs = (torch.randn(F, B, T, generator=g).to(dev), torch.randn(G, B, T, generator=g).to(dev),
                  torch.randn(F, B, T, generator=g).to(dev), torch.randn(F, generator=g).to(dev),
                  theta, torch.randint(0, G, (F,), generator=g).to(dev),
                  torch.full((F,), 1e-6, device=dev), torch.full((F,), 1 - 2e-6, device=dev),
                  torch.full((F,), 0.2, device=dev), torch.ones(F, device=dev), theta * 0.4,
                  theta * 1.6,
                  (True, True, True, False, 0.223, 0.223, True, False, True, 2.0, 0.0, True))
        z = crandn(F, B, T)
        gy, gx = crandn(F, B, T), crandn(F, B, T)

        if op == "selective_bf16":
            inputs = tuple(t.to(torch.bfloat16) if i in (0, 1, 2) else t
                           for i, t in enumerate(inputs[:12])) + (inputs[12],)

            def run():
                _, _, ent = ops.selective_forward_bf16(z, inputs, True, True)
                ops.selective_backward_bf16(z, inputs, ent, gy, gx, True, truncated)
            return run

        def run():
            _, _, ent = rqf.selective_forward(z, inputs, True, True, None)
            rqf.selective_backward(z, inputs, ent, gy, gx, True, truncated, None)
        return run

    if op == "projection_real":  # the readout's real-cotangent GEMMs, beside the complex forms
        W = (crandn(F, F) / math.sqrt(2 * F))
        h = crandn(F, B, T)
        g_real = torch.randn(F, B, T, generator=g).to(dev)
        g_c = g_real.to(torch.complex64)

        def run():
            ops.projection_real(W, g_real, True)
            ops.projection_weight_grad_real(g_real, h)
            ops.projection(W, g_c, True)
            ops.projection_weight_grad(g_c, h)
        return run

    if op in ("projection", "projection_torch"):
        W = (crandn(F, F) / math.sqrt(2 * F))
        h, gz, gh = crandn(F, B, T), crandn(F, B, T), crandn(F, B, T)

        if op == "projection":
            def run():
                ops.projection(W, h)
                ops.projection(W, gz, True, gh)
                ops.projection_weight_grad(gz, h)
        else:
            from prospective_rqf_b200 import _timing

            def run():
                with _timing.launch("torch_matmul", F * B * T, 16 * F * B * T):
                    W @ h.reshape(F, B * T)
                with _timing.launch("torch_matmul_h", F * B * T, 24 * F * B * T):
                    torch.addmm(gh.reshape(F, B * T), W.mH, gz.reshape(F, B * T))
                with _timing.launch("torch_matmul_w", F * B * T, 16 * F * B * T):
                    gz.reshape(F, B * T) @ h.reshape(F, B * T).mH
        return run

    if op == "block_scan":  # the fused block forward beside its two unfused launches
        W = (crandn(F, F) / math.sqrt(2 * F))
        h = crandn(F, B, T)

        def run():
            ops.projection_block_scan(W, h, c1, t0, t1, True, h)
            z = ops.projection(W, h)
            ops._fbt_forward(c1, t0, t1, z, True, h)
        return run

    if op == "block_scan_bwd":  # the fused backward pair beside its two unfused launches
        W0 = (crandn(F, F) / math.sqrt(2 * F))
        h = crandn(F, B, T)
        _, saved = ops.projection_block_scan(W0, h, c1, t0, t1, True, h)
        W = (crandn(F, F) / math.sqrt(2 * F))
        gz_above, acc = crandn(F, B, T), crandn(F, B, T)

        def run():
            ops.projection_block_scan_backward(W, gz_above, acc, saved, True)
            g = ops.projection(W, gz_above, conj_transpose=True, acc=acc)
            ops._fbt_backward(saved, g, True)
        return run

    if op == "fbt_skip":
        z, h, gy = crandn(F, B, T), crandn(F, B, T), crandn(F, B, T)

        def run():
            out, saved = ops._fbt_forward(c1, t0, t1, z, True, h)
            ops._fbt_backward(saved, gy, True)
        return run

    if op == "rank1":  # the first block over a one-channel input, made inside the scan
        x = torch.randn(B, T, generator=g).to(dev)
        u, be = crandn(F), crandn(F)
        w, bb = torch.randn(F, generator=g).to(dev), torch.randn(F, generator=g).to(dev)
        gy = crandn(F, B, T)

        def run():
            out, saved = ops.rank1_block_forward(u, be, w, bb, x, c1, t0, t1, True)
            ops.rank1_block_backward(saved, gy, True, True, True)
        return run

    if op == "mosc":  # groups = oscillators per filter; F filters in and out
        n = groups
        c1m, c2m, _ = _coeffs(F * n, dev, g)
        cw = torch.randn(F * n, 2, generator=g).to(dev)
        u = crandn(B, T, F).requires_grad_(True)
        gy = crandn(B, T, F)

        def run():
            y = ops._triton_sequential_scan_multi_osc(c1m, c2m, u, cw, n)
            torch.autograd.grad(y, (u,), gy)
        return run

    fbt = op in ("fbt", "fbt_raw", "tbptt_fbt")
    shape = (F, B, T) if fbt else (B, T, F)
    if op == "btf_real":
        u = torch.randn(*shape, generator=g).to(dev)
    else:
        u = crandn(*shape)
    u.requires_grad_(True)
    gy = crandn(*shape)
    fwd = {
        "fbt": lambda: rqf.fbt_recompute_scan(c1, t0, t1, u),
        "fbt_raw": lambda: rqf.fbt_prospective_scan(c1, t0, t1, u, False),
        "tbptt_fbt": lambda: rqf.tbptt1_two_tap_scan(u, c1, t0, t1, layout="fbt", fuse_act=True),
        "tbptt_btf": lambda: rqf.tbptt1_two_tap_scan(u, c1, t0, t1, layout="btf"),
        "btf": lambda: rqf._triton_chunked_scan(c1, t0, u),
        "btf_real": lambda: rqf._triton_chunked_scan(c1, t0, u),
        "btf_pro": lambda: rqf._triton_chunked_scan_prospective(c1, t0, t1, u),
    }[op]

    def run():
        y = fwd()
        torch.autograd.grad(y, (u,), gy)
    return run


OPS = ("fbt", "fbt_raw", "fbt_skip", "tbptt_fbt", "tbptt_btf", "btf", "btf_real", "btf_pro",
       "selective", "selective_bf16", "projection", "projection_torch", "projection_real", "mosc",
       "block_scan", "block_scan_bwd", "rank1")


def measure(op, F, B, T, iters=10, warmup=3, groups=8, truncated=False) -> dict:
    import prospective_rqf_b200 as rqf
    from prospective_rqf_b200 import _timing

    run = make_case(op, F, B, T, groups, truncated)
    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    with _timing.KernelTimer() as tm:
        for _ in range(iters):
            run()
    s = tm.summary()
    rqf.check_device_errors()
    peak, kind = hbm_peak()
    kernels = {}
    for name, v in s.items():
        per = v["alg_bytes"] / max(v["launches"], 1)
        gbs = per / (v["mean_ms"] * 1e-3) / 1e9 if v["mean_ms"] else 0.0
        kernels[name] = {"launches": v["launches"], "mean_ms": round(v["mean_ms"], 4),
                         "alg_bytes_per_launch": int(per), "gbs": round(gbs, 1),
                         "frac": round(gbs / peak, 4)}
        if (op.startswith("projection") or op.startswith("block_scan")) and v["mean_ms"] \
                and name not in ("rqf_fbt_block_forward", "rqf_fbt_prospective_backward"):
            flops = 8.0 * F * F * B * T
            kernels[name]["tflops"] = round(flops / (v["mean_ms"] * 1e-3) / 1e12, 1)
    return {"op": op, "F": F, "B": B, "T": T, "iters": iters, "warmup": warmup,
            "peak_gbs": peak, "peak_kind": kind, "kernels": kernels}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--op", choices=OPS, default="fbt")
    ap.add_argument("--F", type=int, default=256)
    ap.add_argument("--B", type=int, default=32)
    ap.add_argument("--T", type=int, default=16000)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--groups", type=int, default=8)
    ap.add_argument("--truncated", action="store_true")
    ap.add_argument("--btf-path", type=int, choices=(0, 1, 2), default=0,
                    help="(B,T,F) kernel family: 0 automatic, 1 streaming, 2 tile-resident")
    a = ap.parse_args(argv)
    from prospective_rqf_b200 import ops

    with ops.btf_kernel_family(a.btf_path):
        out = measure(a.op, a.F, a.B, a.T, a.iters, a.warmup, a.groups, a.truncated)
    out["btf_path"] = a.btf_path
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
