#!/usr/bin/env python
"""Benchmark: RQF train samples/s and scan fwd+bwd HBM GB/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg5-full]
    python bench.py --impl reference ...     # CPU reference arm (oracle port)

One step = one full training step of the Pure RQF encoder (depth 6,
prospective two-tap input, skip connections) on one synthetic batch:
forward, loss, backward, gradient all-reduce across ranks (N > 1), clip,
AdamW, clamp of the filter leaves.  Default workload: BASELINE config 5 per
GPU (H=256, 32 samples/GPU, T=16000, full BPTT), weak scaling over N ranks.

`value`  = global samples / s with inputs resident in HBM (max over ranks).
`e2e`    = the same with each step's inputs copied from pinned host memory and
           the loss read back to the host inside the timed region.
`roofline` = the scan kernels (fwd + bwd, the backend's own kernels) timed
           with CUDA events on their launching stream during the timed steps;
           algorithmic bytes 16 B/element forward + 24 B/element backward.
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
    "rqf_fbt_prospective_backward": 2,
    "rqf_tbptt1_two_tap_backward": 2,
}
SCAN_CALLS = ("rqf_fbt_prospective_forward", "rqf_fbt_block_forward",
              "rqf_fbt_prospective_backward", "rqf_tbptt1_two_tap_backward")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default="cfg5-full", choices=["cfg2", "cfg5-full", "cfg5-tbptt"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def peaks():
    from prospective_rqf_b200.microbench import hbm_peak

    return hbm_peak()


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
def scan_roofline(timer_summary, hbm_peak, peak_kind, traffic):
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
        "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
        "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
        "traffic": traffic, "traffic_unit": "bytes per fwd+bwd launch pair (ncu)",
        "alg_bytes_per_pair": int(sum(v["alg_bytes_per_launch"] for v in per.values())),
        "per_kernel": per,
    }


def gemm_roofline(timer_summary):
    """The projection GEMMs, which take most of the step: fp32-work FLOPs
    (8 M K N for a complex product, 4 M K N for the real-operand forms) over
    their summed launch times, against the split-TF32 ceiling: three TF32
    passes per fp32 product, TF32 at half the measured bf16 rate."""
    from prospective_rqf_b200.microbench import measured_peaks

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
    pk = measured_peaks()
    bf16 = pk.get("bf16_tflops") if pk else None
    kind = "measured" if bf16 else "fallback"
    bf16 = bf16 or 1590.0
    ceiling = bf16 / 2 / 3
    achieved = flops / (ms * 1e-3) / 1e12
    out = {"bound": "tensor", "kernel": "projection GEMMs (" + ", ".join(sorted(per)) + ")",
           "achieved": round(achieved, 1), "peak": round(ceiling, 1), "unit": "TFLOP/s",
           "frac": round(achieved / ceiling, 4),
           "peak_kind": f"{kind} bf16 burst {bf16:.0f} TFLOP/s / 2 (TF32) / 3 (split passes)",
           "flops_unit": "fp32-work FLOPs", "per_kernel": per}
    if pk and pk.get("bf16_tflops_sustained"):
        out["frac_vs_sustained"] = round(achieved / (pk["bf16_tflops_sustained"] / 6), 4)
    return out


def safe_gemm_roofline(timer_summary):
    """gemm_roofline, or {"error": ...}: an informational key never stops the line."""
    try:
        return gemm_roofline(timer_summary)
    except Exception as exc:  # noqa: BLE001
        return {"error": f"{type(exc).__name__}: {exc}"}


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
        "config": config_dict(cfg, 1, world),
        "cpu_baseline": {"value": round(sps, 4), "unit": "samples/s", "cores": threads,
                         "kind": "port",
                         "sample": f"1 sample/step of {cfg.name} (T={cfg.time}, H={cfg.hidden}), "
                                   "oracle fp64 scan + torch CPU fp32 GEMMs"},
        "e2e": {"value": round(sps, 4), "unit": "samples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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

    # ---- value: inputs resident in HBM
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(device.index) as clocks, _timing.KernelTimer() as timer:
        e0.record(stream)
        for _ in range(args.steps):
            loss = step(x_dev, y_dev)
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    kt = timer.summary()

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
    rqf.check_device_errors(device)
    if not (loss_val == loss_val):
        raise FloatingPointError("non-finite loss")

    hbm, peak_kind = peaks()
    roof = scan_roofline(kt, hbm, peak_kind, load_traffic(cfg.name))
    launches = sum(s["launches"] * KERNELS_PER_CALL.get(n, 1) for n, s in kt.items())
    samples = args.steps * cfg.batch * world
    line = {
        "metric": metric_name(cfg),
        "value": round(samples / (ms * 1e-3), 3), "unit": "samples/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(cfg, cfg.batch, world),
        "roofline": roof,
        "roofline_gemm": safe_gemm_roofline(kt),
        "e2e": {"value": round(samples / (ms_e2e * 1e-3), 3), "unit": "samples/s",
                "h2d_bytes_per_step": int(x_host.numel() * x_host.element_size()
                                          + y_host.numel() * y_host.element_size()),
                "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
        "loss": round(loss_val, 5),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sps, threads, dt = cpu_reference_steps(cfg, steps=2, warmup=1, batch=1)
        line["cpu_baseline"] = {"value": round(sps, 4), "unit": "samples/s", "cores": threads,
                                "kind": "port",
                                "sample": f"1 sample/step x 2 steps of {cfg.name} (T={cfg.time}), "
                                          "oracle fp64 scan + torch CPU fp32 GEMMs"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
