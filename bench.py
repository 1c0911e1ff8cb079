#!/usr/bin/env python
"""Benchmark: RQF train samples/s and scan fwd+bwd HBM GB/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg5-full]
    python bench.py --impl reference ...     # CPU reference arm (oracle port)

One step = one full training step of the Pure RQF encoder (depth 6,
prospective two-tap input, skip connections) on one synthetic batch:
forward, loss, backward, gradient all-reduce across ranks (N > 1), clip,
AdamW, clamp of the filter leaves.  Default workload: benchmark config 5 per
GPU (H=256, 32 samples/GPU, T=16000, full BPTT), weak scaling over N ranks.

`value`  = global samples / s with inputs resident in HBM (max over ranks).
`e2e`    = the same with each step's inputs copied from pinned host memory and
           the loss read back to the host inside the timed region.
`roofline` = the scan kernels (fwd + bwd, the backend's own kernels) timed
           with CUDA events on their launching stream in a separate pass of
           steps after the timed ones (the events are not in `value`'s
           region); algorithmic bytes 24 B/element forward (z, skip, out) +
           24 B/element backward (g, z, gz).
`triton_reference` = the reference's own model on its stock GPU path (Triton),
           same B200, same batch shape (N = 1 only), for information;
`triton_reference_scan` = the workload's layer scan alone, the reference's
           Triton kernel beside this backend's (N = 1 only), for information;
`reference_cpu_path` = its own CPU PyTorch path at reduced T, for information.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

KERNELS_PER_CALL = {  # kernels each C-ABI call launches (the backward adds the reduction,
    "rqf_fbt_prospective_forward": 1,  # the projection its weight split)
    "rqf_projection": 2,
    "rqf_projection_weight_grad": 2,
    "rqf_fbt_block_forward": 1,
    "rqf_projection_block_scan": 2,
    "rqf_projection_block_scan_backward": 3,
    "rqf_fbt_prospective_backward": 2,
    "rqf_fbt_rank1_forward": 1,
    "rqf_fbt_rank1_backward": 3,
    "rqf_fbt_rank1_tbptt_backward": 3,
    "rqf_per_step_cross_entropy": 2,
    "rqf_tbptt1_two_tap_backward": 2,
}
SCAN_CALLS = ("rqf_fbt_prospective_forward", "rqf_fbt_block_forward",
              "rqf_fbt_prospective_backward", "rqf_tbptt1_two_tap_backward",
              "rqf_fbt_rank1_forward", "rqf_fbt_rank1_backward", "rqf_fbt_rank1_tbptt_backward")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default="cfg5-full", choices=["cfg2", "cfg5-full", "cfg5-tbptt"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-info", action="store_true",
                    help="skip the reference's own GPU (Triton) and CPU paths, for information")
    return ap.parse_args()


FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def measured_peaks() -> dict | None:
    """MEASURED_PEAKS.json beside this file (this pool's measured copy
    bandwidth and bf16 GEMM rates), or None."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return None
    return None


def hbm_peak() -> tuple[float, str]:
    """(GB/s, "measured" | "fallback"): the STREAM-style copy bandwidth."""
    pk = measured_peaks()
    if pk and pk.get("hbm_gbs"):
        return float(pk["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        self.ident = None
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            self.ident = None

    def __enter__(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
               "-lms", "200"]
        if self.ident:
            cmd += ["-i", self.ident]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self):
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ dist utils
def setup_dist(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()


# ---------------------------------------------------------- CPU reference
class _OracleScan(torch.autograd.Function):
    """(F,B,T) two-tap scan on CPU via the fp64 C oracle (reference arm only)."""

    @staticmethod
    def forward(ctx, c1, t0, t1, z, fuse):
        from oracle import oracle

        y = oracle.two_tap_forward(c1.detach().numpy(), t0.detach().numpy(),
                                   t1.detach().numpy(), z.detach().numpy(), "fbt", fuse_act=fuse)
        ctx.save_for_backward(c1, t0, t1, z)
        ctx.fuse = fuse
        return torch.from_numpy(y).to(torch.complex64)

    @staticmethod
    def backward(ctx, gy):
        from oracle import oracle

        c1, t0, t1, z = ctx.saved_tensors
        gz, gc1, gt0, gt1 = oracle.two_tap_backward(
            c1.numpy(), t0.numpy(), t1.numpy(), z.numpy(), gy.resolve_conj().numpy(), "fbt",
            fuse_act=ctx.fuse)
        f = lambda a: torch.from_numpy(a).to(torch.complex64)  # noqa: E731
        return f(gc1), f(gt0), f(gt1), f(gz), None


def cpu_reference_steps(cfg, steps: int, warmup: int, batch: int):
    """Time the CPU restatement of the training step (oracle scan + torch CPU
    GEMMs) on `batch` samples per step; returns (samples/s, threads, detail)."""
    from prospective_rqf_b200.encoder import ComplexReadout, RQFCoefficients, rqf_forward_std
    from prospective_rqf_b200.train import build_optimizer, waveform_batch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    os.environ["RQF_ORACLE_THREADS"] = str(threads)
    g = torch.Generator().manual_seed(0)
    H, depth = cfg.hidden, cfg.depth

    class CpuModel(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.inp = torch.nn.Linear(1, H, bias=False)
            self.rqf = torch.nn.ModuleList(RQFCoefficients(H, 1 / cfg.samp_frequency, cfg.tau, 1.0,
                                                           generator=g) for _ in range(depth))
            self.W = torch.nn.ParameterList(
                torch.nn.Parameter(torch.complex(torch.randn(H, H, generator=g),
                                                 torch.randn(H, H, generator=g))
                                   * rqf_forward_std(H, 0.5)) for _ in range(depth))
            self.readout = ComplexReadout(H, cfg.num_classes, cfg.readout_hidden)

        def forward(self, x):
            B, T, _ = x.shape
            h = (self.inp.weight @ x.permute(2, 0, 1).reshape(1, B * T)).reshape(H, B, T)
            h = h.to(torch.complex64)
            for i in range(depth):
                c1, t0, t1 = self.rqf[i].two_tap()
                z = (self.W[i] @ h.reshape(H, B * T)).reshape(H, B, T)
                h = _OracleScan.apply(c1, t0, t1, z, i + 1 < depth) + h
            return self.readout(h)

    model = CpuModel()
    opt = build_optimizer(model, cfg)
    x, y = waveform_batch(batch, cfg.time, cfg.samp_frequency, cfg.num_classes, g)

    def step():
        loss = torch.nn.functional.cross_entropy(model(x), y, label_smoothing=cfg.label_smoothing)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), cfg.clip)
        opt.step()
        for r in model.rqf:
            r.clamp_parameters()
        return float(loss.detach())

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = time.perf_counter() - t0
    return steps * batch / dt, threads, dt


# ------------------------------------------------------------------- main
def scan_roofline(timer_summary, peak_gbs, peak_kind, traffic):
    tot_bytes = 0.0
    tot_ms = 0.0
    per = {}
    for name, s in timer_summary.items():
        if name not in SCAN_CALLS:
            continue
        b = s["alg_bytes"]
        per[name] = {"launches": s["launches"], "mean_ms": round(s["mean_ms"], 4),
                     "gbs": round(b / (s["total_ms"] * 1e-3) / 1e9, 1) if s["total_ms"] else None,
                     "alg_bytes_per_launch": int(b / max(s["launches"], 1))}
        tot_bytes += b
        tot_ms += s["total_ms"]
    achieved = tot_bytes / (tot_ms * 1e-3) / 1e9 if tot_ms else 0.0
    return {
        "bound": "hbm", "kernel": "scan fwd+bwd (" + ", ".join(sorted(per)) + ")",
        "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
        "frac": round(achieved / peak_gbs, 4), "peak_kind": peak_kind,
        "traffic": traffic, "traffic_unit": "bytes per fwd+bwd launch pair (ncu)",
        "alg_bytes_per_pair": int(sum(v["alg_bytes_per_launch"] for v in per.values())),
        "per_kernel": per,
    }


def gemm_roofline(timer_summary):
    """The projection GEMMs, which take most of the step: fp32-work FLOPs
    (8 M K N for a complex product, 4 M K N for the real-operand forms) over
    their summed launch times.  One ceiling: the split-TF32 rate derived from
    the measured SUSTAINED bf16 rate (these GEMMs are timed inside a long
    step): three TF32 passes per fp32 product, TF32 at half the bf16 rate."""
    flops = ms = 0.0
    per = {}
    for name, s in timer_summary.items():
        if not s.get("flops"):
            continue
        flops += s["flops"]
        ms += s["total_ms"]
        per[name] = {"launches": s["launches"], "mean_ms": round(s["mean_ms"], 4),
                     "tflops": round(s["flops"] / (s["total_ms"] * 1e-3) / 1e12, 1)
                     if s["total_ms"] else None}
    if not ms:
        return None
    pk = measured_peaks() or {}
    bf16 = pk.get("bf16_tflops_sustained")
    kind = "measured sustained" if bf16 else "fallback burst"
    bf16 = bf16 or FALLBACK_BF16_TFLOPS
    ceiling = bf16 / 2 / 3
    achieved = flops / (ms * 1e-3) / 1e12
    return {"bound": "tensor", "kernel": "projection GEMMs (" + ", ".join(sorted(per)) + ")",
            "achieved": round(achieved, 1), "peak": round(ceiling, 1), "unit": "TFLOP/s",
            "frac": round(achieved / ceiling, 4),
            "peak_kind": f"{kind} bf16 {bf16:.0f} TFLOP/s / 2 (TF32) / 3 (split-TF32 passes)",
            "flops_unit": "fp32-work FLOPs", "per_kernel": per}


def load_traffic(workload):
    """DRAM bytes (read + write) of one scan forward+backward launch pair from
    the committed ncu capture (profiles/traffic.json), or None."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        entry = json.loads(p.read_text()).get(workload)
        return None if entry is None else int(entry["bytes_per_launch_pair"])
    except Exception:
        return None


def run_reference_arm(args, world, rank):
    """The reference arm: the CPU restatement of the step (oracle port), on
    all host cores, rank 0 only; each step a bounded sample of 1 sample of
    the workload whose config it reports (the same as this backend's arm)."""
    from prospective_rqf_b200.train import WORKLOADS

    if rank != 0:
        return
    cfg = WORKLOADS[args.workload]
    sps, threads, dt = cpu_reference_steps(cfg, args.steps, args.warmup, batch=1)
    line = {
        "metric": metric_name(cfg), "value": round(sps, 4), "unit": "samples/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64 scan / f32 GEMM", "data": "synthetic",
        "impl": "reference",
        "config": config_dict(cfg, cfg.batch, world),
        "cpu_baseline": {"value": round(sps, 4), "unit": "samples/s", "cores": threads,
                         "kind": "port",
                         "sample": f"1 sample/step of {cfg.name} (T={cfg.time}, H={cfg.hidden}), "
                                   "oracle fp64 scan + torch CPU fp32 GEMMs"},
        "e2e": {"value": round(sps, 4), "unit": "samples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------- the reference's own paths, for information
REF_INSTALL = ROOT / "baseline" / "_ref"


def _reference_modules():
    """The reference's PureRQFEncoder from its offline install, or None."""
    if not (REF_INSTALL / "rqf_models").exists():
        return None
    if str(REF_INSTALL) not in sys.path:
        sys.path.insert(0, str(REF_INSTALL))
    os.environ.setdefault("TRITON_CACHE_DIR", "/tmp/rqf_triton_cache")
    from rqf_models.backbones.rqf.pure import PureRQFEncoder

    return PureRQFEncoder


def _reference_classifier(PureRQFEncoder, cfg, device):
    """The reference's model for this workload: PureRQFEncoder (the paper
    recipe, configs/model/pure_rqf_paper.yaml, at the workload's width, depth
    and gradient mode) under the head that train.py:ComplexReadoutClassifier
    (:74-136) builds: per-timestep Linear(2F, R) -> ReLU -> Dropout(0) ->
    Linear(R, C) on [Re h; Im h], logits mean-pooled over time (or per step)."""
    torch.manual_seed(0)
    enc = PureRQFEncoder(
        input_dims=1, output_dims=8, hidden_dims=cfg.hidden, num_layers=cfg.depth,
        samp_frequency=cfg.samp_frequency, min_freq=1.0, max_freq=8000.0, tau=cfg.tau,
        discretization="zoh", activation="split_relu", complex_weights=True,
        param_space="log", seq_duration=1.0, w_init="forward", final_activation=False,
        input_proj_bias=False, complex_output=True, prospective_input=True,
        prospective_mode="tau", skip_connection=True, scan_grad_mode=cfg.scan_grad_mode)
    head = torch.nn.Sequential(torch.nn.Linear(2 * cfg.hidden, cfg.readout_hidden),
                               torch.nn.ReLU(), torch.nn.Dropout(0.0),
                               torch.nn.Linear(cfg.readout_hidden, cfg.num_classes))
    return torch.nn.ModuleDict({"encoder": enc, "head": head}).to(device)


def reference_gpu_step(cfg, steps: int, warmup: int, device):
    """The reference's own model on its stock GPU path (its Triton kernels),
    one training step as train.py:run_epoch (:792-843) takes it: forward,
    cross-entropy, backward, clip_grad_norm_, AdamW, clamp_parameters, on
    the same synthetic batch shape as this backend's arm.  CUDA events."""
    PureRQFEncoder = _reference_modules()
    if PureRQFEncoder is None:
        return {"unavailable": "reference install (baseline/_ref) absent"}
    from prospective_rqf_b200.train import waveform_batch

    model = _reference_classifier(PureRQFEncoder, cfg, device)
    model.train()
    leaves = [p for n, p in model.named_parameters() if "rqf_fwd" in n and p.requires_grad]
    rest = [p for n, p in model.named_parameters() if "rqf_fwd" not in n and p.requires_grad]
    opt = torch.optim.AdamW([{"params": rest, "lr": cfg.lr, "weight_decay": cfg.weight_decay},
                             {"params": leaves, "lr": cfg.lr * cfg.rqf_lr_factor,
                              "weight_decay": 0.0}], eps=1e-8)
    g = torch.Generator().manual_seed(1000)
    x, y = waveform_batch(cfg.batch, cfg.time, cfg.samp_frequency, cfg.num_classes, g)
    x, y = x.to(device), y.to(device)
    per_step = cfg.scan_grad_mode == "tbptt1"

    def step():
        feats = model["encoder"](x)  # (B, T, F) complex
        B, T, F = feats.shape
        logits = model["head"](torch.cat([feats.real, feats.imag], dim=-1).reshape(B * T, 2 * F))
        logits = logits.reshape(B, T, -1)
        if per_step:
            loss = torch.nn.functional.cross_entropy(
                logits.reshape(B * T, -1), y[:, None].expand(B, T).reshape(-1),
                label_smoothing=cfg.label_smoothing)
        else:
            loss = torch.nn.functional.cross_entropy(logits.mean(dim=1), y,
                                                     label_smoothing=cfg.label_smoothing)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), cfg.clip)
        opt.step()
        model["encoder"].clamp_parameters()
        return loss.detach()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        loss = step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    del model, opt
    return {"value": round(steps * cfg.batch / (ms * 1e-3), 3), "unit": "samples/s",
            "ms_per_step": round(ms / steps, 3), "steps": steps, "warmup": warmup,
            "loss": round(float(loss), 5), "same_config": True,
            "what": "the reference's PureRQFEncoder (paper recipe) + the train.py "
                    "ComplexReadoutClassifier head, full training step on its stock Triton "
                    "path, same B200, same batch shape, from baseline/_ref"}


def reference_gpu_scan(cfg, device):
    """The workload's dominant scan alone, the reference's Triton kernel
    beside this backend's: fbt_recompute_scan (fbt_scan_kernel.py:667) at the
    layer shape (F = hidden, B, T), forward + backward, CUDA events, warm."""
    if _reference_modules() is None:
        return {"unavailable": "reference install (baseline/_ref) absent"}
    import prospective_rqf_b200 as rqf
    from rqf_models.ops.fbt_scan_kernel import fbt_recompute_scan as ref_scan

    F, B, T = cfg.hidden, cfg.batch, cfg.time
    g = torch.Generator(device=device).manual_seed(3)
    mag = 0.9 + 0.0999 * torch.rand(F, device=device, generator=g)
    c1 = torch.polar(mag, 6.283 * torch.rand(F, device=device, generator=g))
    t0 = 0.3 * torch.randn(F, dtype=torch.complex64, device=device, generator=g)
    t1 = 0.3 * torch.randn(F, dtype=torch.complex64, device=device, generator=g)
    z = torch.randn(F, B, T, dtype=torch.complex64, device=device, generator=g)
    gy = torch.randn_like(z)
    zz = z.requires_grad_(True)

    def timed(op):
        def run():
            y = op(c1, t0, t1, zz)
            torch.autograd.grad(y, (zz,), gy)
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            run()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 5

    ref_ms, ours_ms = timed(ref_scan), timed(rqf.fbt_recompute_scan)
    return {"op": f"fbt_recompute_scan F={F} B={B} T={T} fwd+bwd", "reference_ms": round(ref_ms, 4),
            "b200_ms": round(ours_ms, 4), "speedup": round(ref_ms / ours_ms, 3)}


def reference_cpu_paths(cfg, threads: int):
    """The reference's own CPU PyTorch path, timed on the host cores:
    PureRQFEncoder forward+backward (per sample, at reduced T: its CPU
    backward does not finish a T=16000 sample in minutes) and config 1's
    sequential_scan op (the exact benchmark shape)."""
    PureRQFEncoder = _reference_modules()
    if PureRQFEncoder is None:
        return {"unavailable": "reference install (baseline/_ref) absent"}
    from rqf_models.ops.scan import sequential_scan

    torch.set_num_threads(threads)
    out = {"cores": threads}
    T = 2000
    enc = PureRQFEncoder(
        input_dims=1, output_dims=8, hidden_dims=cfg.hidden, num_layers=cfg.depth,
        samp_frequency=cfg.samp_frequency, min_freq=1.0, max_freq=8000.0, tau=cfg.tau,
        discretization="zoh", activation="split_relu", complex_weights=True,
        param_space="log", seq_duration=1.0, w_init="forward", final_activation=False,
        input_proj_bias=False, complex_output=True, prospective_input=True,
        prospective_mode="tau", skip_connection=True, scan_grad_mode=cfg.scan_grad_mode)
    x = torch.randn(1, T, 1, generator=torch.Generator().manual_seed(0))
    enc(x).abs().mean().backward()
    t0 = time.perf_counter()
    enc(x).abs().mean().backward()
    dt = time.perf_counter() - t0
    out["encoder"] = {"value": round(1.0 / dt, 4), "unit": "samples/s",
                      "shape": f"B=1, T={T}, H={cfg.hidden}, depth {cfg.depth}, "
                               f"{cfg.scan_grad_mode} BPTT; encoder fwd+bwd only"}
    g = torch.Generator().manual_seed(0)
    u = torch.randn(32, 161, 128, generator=g)
    lam = torch.polar(0.90 + 0.099 * torch.rand(128, generator=g),
                      torch.pi * torch.rand(128, generator=g)).to(torch.complex64)
    b = (torch.randn(128, generator=g) + 1j * torch.randn(128, generator=g)).to(
        torch.complex64) / 2 ** 0.5

    def op():
        lg, bg, ug = (t.detach().requires_grad_(True) for t in (lam, b, u))
        (sequential_scan(lg, bg, ug).abs() ** 2).sum().backward()
    op()
    t0 = time.perf_counter()
    for _ in range(3):
        op()
    out["config1_sequential_scan"] = {
        "ms": round((time.perf_counter() - t0) / 3 * 1e3, 3),
        "shape": "B=32, T=161, H=128, real u, fwd+bwd of sum |y|^2"}
    return out


def safe_info(fn, *a):
    """An informational key never stops the line."""
    try:
        return fn(*a)
    except Exception as exc:  # noqa: BLE001
        return {"error": f"{type(exc).__name__}: {exc}"[:300]}


def metric_name(cfg):
    return (f"RQF train samples/s (Pure RQF depth {cfg.depth}, H={cfg.hidden}, T={cfg.time}, "
            f"{'TBPTT(1)' if cfg.scan_grad_mode == 'tbptt1' else 'full BPTT'}); "
            "scan fwd+bwd HBM GB/s vs peak")


def config_dict(cfg, batch, world):
    return {"workload": f"{cfg.name}: Pure RQF encoder depth {cfg.depth}, H={cfg.hidden}, "
                        f"prospective two-tap (tau=5dt), skip, {cfg.scan_grad_mode} BPTT, "
                        "per-timestep [Re;Im] MLP readout, AdamW",
            "per_gpu_batch": batch, "global_batch": batch * world, "seq_len": cfg.time,
            "hidden": cfg.hidden, "depth": cfg.depth, "parallelism": f"dp{world}",
            "l2": "inputs larger than L2 (every scan tensor is >= 0.26 GB)"}


def main():
    args = parse()
    world, rank, local = setup_dist(args.gpus)
    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        if world > 1:
            dist.destroy_process_group()
        return

    import prospective_rqf_b200 as rqf
    from prospective_rqf_b200 import _timing
    from prospective_rqf_b200.train import WORKLOADS, TrainStep, waveform_batch

    assert args.warmup >= 3, "at least 3 warm-up steps"
    cfg = WORKLOADS[args.workload]
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    step = TrainStep(cfg, device, seed=0)  # identical params on every rank
    g = torch.Generator().manual_seed(1000 + rank)  # rank-offset data
    x_host, y_host = waveform_batch(cfg.batch, cfg.time, cfg.samp_frequency, cfg.num_classes, g)
    x_host, y_host = x_host.pin_memory(), y_host.pin_memory()
    x_dev, y_dev = x_host.to(device), y_host.to(device)

    rqf.read_device_error(device, clear=True)
    for _ in range(args.warmup):
        step(x_dev, y_dev)
    torch.cuda.synchronize()

    # ---- value: inputs resident in HBM; nothing but the steps in the timed region
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(device.index) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            loss = step(x_dev, y_dev)
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world)

    # ---- e2e: host buffers, H2D of inputs and D2H of the loss every step
    barrier(world)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        xd = x_host.to(device, non_blocking=True)
        yd = y_host.to(device, non_blocking=True)
        loss_val = float(step(xd, yd).cpu())
    f1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(f0.elapsed_time(f1), world)

    # ---- kernel pass (not part of `value`): each C-ABI call bracketed by CUDA
    # events on its launching stream, for the roofline keys and the launch count
    kpass = max(1, min(args.steps, 5))
    barrier(world)
    with _timing.KernelTimer() as timer:
        for _ in range(kpass):
            step(x_dev, y_dev)
        torch.cuda.synchronize()
    barrier(world)
    kt = timer.summary()
    rqf.check_device_errors(device)
    if not (loss_val == loss_val):
        raise FloatingPointError("non-finite loss")

    hbm, peak_kind = hbm_peak()
    roof = scan_roofline(kt, hbm, peak_kind, load_traffic(cfg.name))
    launches_per_step = sum(s["launches"] * KERNELS_PER_CALL.get(n, 1)
                            for n, s in kt.items()) / kpass
    samples = args.steps * cfg.batch * world
    line = {
        "metric": metric_name(cfg),
        "value": round(samples / (ms * 1e-3), 3), "unit": "samples/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (split-TF32 GEMMs)", "data": "synthetic",
        "config": config_dict(cfg, cfg.batch, world),
        "roofline": roof,
        "roofline_gemm": safe_info(gemm_roofline, kt),
        "kernel_pass_steps": kpass,
        "e2e": {"value": round(samples / (ms_e2e * 1e-3), 3), "unit": "samples/s",
                "h2d_bytes_per_step": int(x_host.numel() * x_host.element_size()
                                          + y_host.numel() * y_host.element_size()),
                "d2h_bytes_per_step": 4},
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "clocks": clocks.summary(),
        "loss": round(loss_val, 5),
    }
    if rank == 0 and world == 1:
        del step
        torch.cuda.empty_cache()
        if not args.no_reference_info:
            line["triton_reference"] = safe_info(reference_gpu_step, cfg, 3, 3, device)
            tr = line["triton_reference"]
            if isinstance(tr, dict) and tr.get("value"):
                tr["value_over_reference"] = round(line["value"] / tr["value"], 3)
            if cfg.scan_grad_mode == "full":
                line["triton_reference_scan"] = safe_info(reference_gpu_scan, cfg, device)
        threads = os.cpu_count() or 1
        if not args.no_cpu_baseline:
            sps, threads, dt = cpu_reference_steps(cfg, steps=2, warmup=1, batch=1)
            line["cpu_baseline"] = {"value": round(sps, 4), "unit": "samples/s",
                                    "cores": threads, "kind": "port",
                                    "sample": f"1 sample/step x 2 steps of {cfg.name} "
                                              f"(T={cfg.time}), oracle fp64 scan + torch CPU "
                                              "fp32 GEMMs"}
        if not args.no_reference_info:
            line["reference_cpu_path"] = safe_info(reference_cpu_paths, cfg, threads)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
