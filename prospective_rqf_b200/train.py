"""Batch-sharded training step for the Pure RQF encoder on the B200 kernels.

Restates the reference's step (train.py:run_epoch :792-843 with
build_optimizer :630-660, per_step_cross_entropy :663-674,
clip_model_grad_norm_ :777-789) around PureRQFEncoderB200: forward, loss,
backward, one NCCL all-reduce of the flat parameter gradients across ranks
(the only collective; every (b, f) scan row is independent so the batch
shards with no exchange inside the scan), gradient clipping, AdamW, and the
post-step clamp of the log-space filter leaves.

Synthetic inputs follow the benchmarked waveform workloads: each waveform is a sum of 3
sinusoids (freq ~ U(50, 4000) Hz at fs = 16 kHz, amplitude ~ U(0.1, 0.5)) plus
N(0, 0.05) noise, clipped to [-1, 1]; labels uniform over 35 classes.  The
Speech Commands audio the reference trains on is not available here.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .encoder import PureRQFEncoderB200, RQFClassifier


@dataclass
class StepConfig:
    name: str = "cfg5-full"
    batch: int = 32            # per rank
    time: int = 16000
    hidden: int = 256
    depth: int = 6
    num_classes: int = 35
    readout_hidden: int = 256
    scan_grad_mode: str = "full"   # or "tbptt1" (per-step local loss)
    samp_frequency: float = 16000.0
    tau: float = 5.0 / 16000.0
    lr: float = 1e-3
    weight_decay: float = 1e-4
    rqf_lr_factor: float = 0.1
    label_smoothing: float = 0.1
    clip: float = 1.0


WORKLOADS = {
    # config 2: Pure RQF depth 6, H=128, [B=16, T=16000, 1], full BPTT
    "cfg2": StepConfig(name="cfg2", batch=16, hidden=128),
    # config 5 per-rank shard: H=256, 32 samples per GPU, full BPTT / TBPTT(1)
    "cfg5-full": StepConfig(name="cfg5-full", batch=32, hidden=256),
    "cfg5-tbptt": StepConfig(name="cfg5-tbptt", batch=32, hidden=256, scan_grad_mode="tbptt1"),
}


def waveform_batch(batch: int, time: int, fs: float, num_classes: int,
                   generator: torch.Generator, device="cpu"):
    """(x (B,T,1) float32 in [-1, 1], y (B,) int64) — the config 2/5 waveform generator.

    Drawn on the generator's device: a CUDA generator makes the whole batch on
    the GPU (no host work or copy per step); a CPU generator draws on the host
    and the batch is then moved to `device`."""
    g = generator
    gd = g.device
    freq = 50.0 + (4000.0 - 50.0) * torch.rand(batch, 3, 1, generator=g, device=gd)
    amp = 0.1 + 0.4 * torch.rand(batch, 3, 1, generator=g, device=gd)
    phase = 2 * math.pi * torch.rand(batch, 3, 1, generator=g, device=gd)
    t = torch.arange(time, dtype=torch.float64, device=gd) / fs
    x = (amp.double() * torch.sin(2 * math.pi * freq.double() * t + phase.double())).sum(1)
    x = x + 0.05 * torch.randn(batch, time, generator=g, dtype=torch.float64, device=gd)
    x = x.clamp(-1.0, 1.0).float().unsqueeze(-1)
    y = torch.randint(0, num_classes, (batch,), generator=g, device=gd)
    return x.to(device), y.to(device)


def synthetic_batches(cfg: "StepConfig", device, seed: int = 0):
    """Endless fresh batches of the workload's synthetic waveforms, drawn on
    `device` (a CUDA device keeps data generation on the GPU)."""
    g = torch.Generator(device=device).manual_seed(seed)
    while True:
        yield waveform_batch(cfg.batch, cfg.time, cfg.samp_frequency, cfg.num_classes, g, device)


def build_model(cfg: StepConfig, device, seed: int = 0) -> RQFClassifier:
    enc = PureRQFEncoderB200(input_dims=1, hidden_dims=cfg.hidden, num_layers=cfg.depth,
                             samp_frequency=cfg.samp_frequency, tau=cfg.tau,
                             skip_connection=True, final_activation=False,
                             input_proj_bias=False, scan_grad_mode=cfg.scan_grad_mode, seed=seed)
    return RQFClassifier(enc, cfg.num_classes, cfg.readout_hidden).to(device)


def build_optimizer(model: torch.nn.Module, cfg: StepConfig) -> torch.optim.Optimizer:
    """Two groups as train.py:build_optimizer: filter leaves at lr*rqf_lr_factor
    without weight decay, everything else at lr with weight decay."""
    rqf, base = [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        (rqf if ".rqf." in f".{name}" or name.startswith("encoder.rqf") else base).append(p)
    groups = [{"params": base, "lr": cfg.lr, "weight_decay": cfg.weight_decay}]
    if rqf:
        groups.append({"params": rqf, "lr": cfg.lr * cfg.rqf_lr_factor, "weight_decay": 0.0})
    return torch.optim.AdamW(groups, eps=1e-8)


class GradAllReduce:
    """One flat all-reduce (average) of every parameter gradient across ranks."""

    def __init__(self, params, group=None):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self._flat = None

    def __call__(self) -> None:
        if self.world == 1:
            return
        views = []
        for p in self.params:
            g = p.grad
            if g is None:
                g = p.grad = torch.zeros_like(p)
            views.append(torch.view_as_real(g).reshape(-1) if g.is_complex() else g.reshape(-1))
        n = sum(v.numel() for v in views)
        if self._flat is None or self._flat.numel() != n:
            self._flat = torch.empty(n, dtype=torch.float32, device=views[0].device)
        torch.cat(views, out=self._flat)
        dist.all_reduce(self._flat, op=dist.ReduceOp.SUM, group=self.group)
        self._flat.div_(self.world)
        off = 0
        for v in views:
            v.copy_(self._flat[off:off + v.numel()].view_as(v))
            off += v.numel()


@torch.no_grad()
def clip_grad_norm_(params, max_norm: float) -> torch.Tensor:
    """torch.nn.utils.clip_grad_norm_ (train.py:clip_model_grad_norm_
    :777-789): total = ||(||g_p||)_p||, g *= min(1, max_norm / (total + 1e-6)).
    Complex gradients enter through their real views, as the reference's own
    MPS branch does, so all norms are one foreach launch instead of one
    complex reduction per parameter."""
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return torch.zeros(())
    if any(g.is_complex() and g.is_conj() for g in grads):
        return torch.nn.utils.clip_grad_norm_(params, max_norm)
    views = [torch.view_as_real(g) if g.is_complex() else g for g in grads]
    total = torch.linalg.vector_norm(torch.stack(torch._foreach_norm(views)))
    scale = (max_norm / (total + 1e-6)).clamp(max=1.0)
    torch._foreach_mul_(views, scale)
    return total


class TrainStep:
    """One optimisation step: returns the (detached) loss tensor on device."""

    def __init__(self, cfg: StepConfig, device, seed: int = 0):
        self.cfg = cfg
        self.model = build_model(cfg, device, seed)
        self.opt = build_optimizer(self.model, cfg)
        self.allreduce = GradAllReduce(self.model.parameters())

    def __call__(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        self.model.train()
        if cfg.scan_grad_mode == "tbptt1":  # per_step_cross_entropy (train.py:663-674)
            loss = self.model.per_step_loss(x, y, cfg.label_smoothing)
        else:
            loss = torch.nn.functional.cross_entropy(self.model(x), y,
                                                     label_smoothing=cfg.label_smoothing)
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        self.allreduce()
        clip_grad_norm_(list(self.model.parameters()), cfg.clip)
        self.opt.step()
        self.model.encoder.clamp_parameters()
        return loss.detach()
