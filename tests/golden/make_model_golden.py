"""Generate the model-level golden fixtures: the reference's own classifier.

Run in a container that has the reference tree (read-only) available:

    python tests/golden/make_model_golden.py --reference /path/to/prospective-rqf

Each case builds the REFERENCE model on CPU, with the reference's own code:

* rqf_models/backbones/rqf/pure.py:PureRQFEncoder (paper recipe: log
  parameters, ZOH, tau-mode prospective input, split-ReLU, skip connections,
  final_activation=False, complex_output=True), run on its CPU path
  (pure.py:444-465: per block the complex GEMM, the prospective two-tap scan
  of block.py:684-954 and the split activation);
* train.py:ComplexReadoutClassifier (:74-136) around it, the classifier the
  reference trains this encoder with.  train.py imports hydra at module level,
  which this container lacks, so the class definition alone is taken from the
  file's syntax tree and executed with torch.nn in scope; no other part of
  train.py runs.

then one forward and backward of the training loss of train.py:run_epoch
(:815-827): cross-entropy of the mean-pooled logits (full BPTT), or
per_step_cross_entropy (:663-674) of the per-step logits (TBPTT(1) with
per_step_loss).  The fixture holds the parameters (reference names), the
input, the labels, the logits, the loss and every parameter gradient, all
fp32 as the reference computes them.

Outputs: tests/golden/model_*.npz (small; committed).  Nothing at test time
reads the reference tree.
"""

from __future__ import annotations

import argparse
import ast
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

CASES = {
    # name: (hidden, depth, batch, time, readout hidden, classes, scan_grad_mode)
    "model_full": (64, 6, 2, 4000, 32, 35, "full"),
    "model_tbptt1": (64, 6, 2, 2000, 32, 35, "tbptt1"),
}


def _classifier_class(reference: str):
    """train.py:ComplexReadoutClassifier, executed from the file's syntax tree."""
    import torch
    import torch.nn as nn

    src = (Path(reference) / "train.py").read_text()
    tree = ast.parse(src)
    cls = [n for n in tree.body
           if isinstance(n, ast.ClassDef) and n.name == "ComplexReadoutClassifier"]
    if len(cls) != 1:
        raise SystemExit("ComplexReadoutClassifier not found in train.py")
    ns = {"nn": nn, "torch": torch}
    exec(compile(ast.Module(body=cls, type_ignores=[]), "train.py", "exec"), ns)
    return ns["ComplexReadoutClassifier"]


def _waveforms(batch, time, seed):
    """Sum of three sinusoids plus noise, clipped (the benchmark's waveform draw)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    t = torch.arange(time, dtype=torch.float64) / 16000.0
    freq = 50 + 3950 * torch.rand(batch, 3, 1, generator=g, dtype=torch.float64)
    amp = 0.1 + 0.4 * torch.rand(batch, 3, 1, generator=g, dtype=torch.float64)
    phase = 2 * torch.pi * torch.rand(batch, 3, 1, generator=g, dtype=torch.float64)
    x = (amp * torch.sin(2 * torch.pi * freq * t + phase)).sum(dim=1)
    x = x + 0.05 * torch.randn(batch, time, generator=g, dtype=torch.float64)
    return x.clamp(-1, 1).to(torch.float32)[:, :, None]


def make_case(out: Path, name: str, classifier_cls):
    import torch
    import torch.nn.functional as tnf

    from rqf_models.backbones.rqf.pure import PureRQFEncoder

    hidden, depth, batch, time, rh, classes, mode = CASES[name]
    torch.manual_seed(0)
    enc = PureRQFEncoder(
        input_dims=1, output_dims=8, hidden_dims=hidden, num_layers=depth,
        samp_frequency=16000.0, min_freq=1.0, max_freq=8000.0, tau=0.0003125,
        discretization="zoh", activation="split_relu", complex_weights=True,
        param_space="log", seq_duration=1.0, w_init="forward", final_activation=False,
        input_proj_bias=False, complex_output=True, prospective_input=True,
        prospective_mode="tau", skip_connection=True, scan_grad_mode=mode)
    per_step = mode == "tbptt1"
    model = classifier_cls(enc, hidden, classes, rh, 0.0, per_step)
    with torch.no_grad():  # a non-trivial output layer (the reference starts it near 0)
        model.head[3].weight.normal_(0.0, 0.1)
        model.head[3].bias.normal_(0.0, 0.1)
    model.train()
    x = _waveforms(batch, time, seed=11)
    y = torch.randint(0, classes, (batch,), generator=torch.Generator().manual_seed(12))
    logits = model(x)
    if per_step:
        bt, tt, cc = logits.shape
        loss = tnf.cross_entropy(logits.reshape(bt * tt, cc), y[:, None].expand(bt, tt).reshape(-1))
    else:
        loss = tnf.cross_entropy(logits, y)
    loss.backward()
    rec = {"x": x.numpy(), "y": y.numpy(), "logits": logits.detach().numpy(),
           "loss": np.float32(loss.item()),
           "config": np.array([hidden, depth, batch, time, rh, classes, int(per_step)])}
    for n, p in model.named_parameters():
        rec["param/" + n] = p.detach().numpy()
        if p.grad is not None:
            rec["grad/" + n] = p.grad.numpy()
    for n, b in model.named_buffers():
        rec["buffer/" + n] = b.numpy()
    np.savez_compressed(out / f"{name}.npz", **rec)
    print(name, "loss", loss.item(), "logits", tuple(logits.shape))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RQF_REFERENCE", ""))
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    if not args.reference:
        sys.exit("pass --reference <path to the reference project>")
    sys.path.insert(0, args.reference)
    import torch

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    cls = _classifier_class(args.reference)
    for name in CASES:
        make_case(Path(args.out), name, cls)


if __name__ == "__main__":
    main()
