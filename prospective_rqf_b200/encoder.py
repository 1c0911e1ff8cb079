"""Pure RQF encoder and complex readout driven by the B200 scan kernels.

A restatement of the reference's channel-outermost Pure RQF stack — the
callers on either side of the scan — so the training step can run (and be
timed) without the reference tree:

* ZOH prospective two-tap coefficients from log-space leaves
  (rqf_models/backbones/rqf/filter.py:RQF, _init_log_space :303-340,
  compute_two_tap_coefficients :510-664 ZOH branch, clamp_parameters :366-399,
  _expm1_div_x_complex :21-50);
* the (F,B,T) stack of rqf_models/backbones/rqf/pure.py:_forward_fbt_stack
  (:510-536) and PureRQFBlock._forward_fbt (:212-243): input projection on the
  tiny input axis, per block z = W @ h (complex GEMM), two-tap scan with the
  split-ReLU fused (fbt_recompute_scan) or the raw state for a last block
  without activation, complex skip h = out + h;
* power-preserving W init (rqf_models/backbones/rqf/utils/init.py:33-65);
* the per-timestep [Re; Im] MLP readout with mean-pooled logits
  (train.py:ComplexReadoutClassifier :74-136), evaluated channel-first so the
  (F,B,T) features need no (B,T,F) permute.

TBPTT(1) blocks own their projection GEMM (as rqf_models/ops/selective_scan.py
:_SelectiveLayerScan does for the selective path) so the lag-tap cotangent
reaches W only, without the reference's second forward GEMM W(x.detach())
(pure.py:184-187).
"""

from __future__ import annotations

import math
import os

import torch
import torch.nn as nn
from torch.autograd.function import once_differentiable

from . import ops

SPLIT_RELU_GAIN = 0.5     # utils/init.py RQF_ACTIVATION_GAINS["split_relu"]

# "tc": the block projections run on the split-TF32 tcgen05 GEMM
# (ops.projection); "torch": torch.matmul (cuBLAS fp32), as the reference does.
PROJECTION = os.environ.get("RQF_B200_PROJECTION", "tc")
# "auto": a block whose projection runs on the tcgen05 GEMM runs its scan in
# that GEMM's epilogue (ops.projection_block_scan) where that is expected to be
# faster (ops.block_scan_preferred); "1": wherever it applies (T a multiple of
# 128); "0": never — the projection, then the separate (F,B,T) scan kernel.
BLOCK_SCAN = os.environ.get("RQF_B200_BLOCK_SCAN", "auto")
# The same for the backward pairs of _PureStack (ops.projection_block_scan_backward):
# "auto" where ops.block_scan_backward_preferred expects it to pay, "1"
# wherever it applies, "0" never.
BLOCK_SCAN_BWD = os.environ.get("RQF_B200_BLOCK_SCAN_BWD", "auto")


def _block_scan_chosen(W, h) -> bool:
    """Whether the block z = W h runs its scan in the GEMM's epilogue, by
    BLOCK_SCAN (the same rule decides a backward pair: W the upper block's
    weight conjugate-transposed, h its z cotangent)."""
    mode = str(BLOCK_SCAN)
    return PROJECTION == "tc" and mode not in ("0", "False") and (
        ops.block_scan_preferred(W, h) if mode == "auto" else ops.block_scan_eligible(W, h))


def _backward_pair_chosen(W, gz) -> bool:
    """Whether the backward pair (W the upper block's weight, gz its z
    cotangent) runs as one ops.projection_block_scan_backward launch."""
    mode = str(BLOCK_SCAN_BWD)
    return PROJECTION == "tc" and mode not in ("0", "False") and (
        ops.block_scan_backward_preferred(W, gz) if mode == "auto"
        else ops.block_scan_eligible(W.mH, gz))


def _block_forward(W, h, C1, tap0, tap1, fuse_act, skip):
    """z = W h, then the (F,B,T) scan (act(y) + skip when skip is given):
    (out, saved) as ops._fbt_forward returns them."""
    if _block_scan_chosen(W, h):
        return ops.projection_block_scan(W, h, C1, tap0, tap1, fuse_act, skip)
    return ops._fbt_forward(C1, tap0, tap1, _project(W, h), fuse_act, skip)


def _weight_grad(gz, h):
    """gz @ h^H over the (d, batch*time) views: the projection's weight cotangent."""
    if PROJECTION == "tc" and gz.is_cuda:
        return ops.projection_weight_grad(gz, h)
    return gz.reshape(gz.shape[0], -1) @ h.reshape(h.shape[0], -1).mH


def _project(W, h, conj_transpose=False, acc=None, inplace=False):
    """op(W) @ h (+ acc) over the (d, batch*time) view of an (d, B, T) tensor;
    with `inplace` the sum may be accumulated into acc (which the caller
    gives up)."""
    if PROJECTION == "tc" and h.is_cuda:
        return ops.projection(W, h, conj_transpose, acc, inplace)
    d, B, T = h.shape
    opw = W.mH if conj_transpose else W
    if acc is None:
        return (opw @ h.reshape(d, B * T)).reshape(-1, B, T)
    return torch.addmm(acc.reshape(-1, B * T), opw, h.reshape(d, B * T)).reshape(-1, B, T)
# Inputs of at most this many channels take the low-rank first block (_InputBlock).
LOWRANK_MAX_INPUTS = 4
NOMINAL_FILTER_GAIN = 0.5  # utils/init.py NOMINAL_FILTER_GAIN


def rqf_forward_std(n_in: int, activation_gain: float) -> float:
    return 1.0 / math.sqrt(2.0 * n_in * NOMINAL_FILTER_GAIN * activation_gain)


def _expm1_div_x(x: torch.Tensor, threshold: float = 1e-4) -> torch.Tensor:
    """(e^x - 1)/x for complex x with the reference's 4th-order small branch."""
    small = x.abs() < threshold
    safe = torch.where(small, torch.ones_like(x), x)
    direct = (torch.exp(x) - 1.0) / safe
    taylor = 1.0 + x / 2 + x ** 2 / 6 + x ** 3 / 24 + x ** 4 / 120
    return torch.where(small, taylor, direct)


def two_tap_coefficients(log_theta: torch.Tensor, log_gamma: torch.Tensor, dt: float,
                         tau: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """ZOH prospective two-tap coefficients (tau mode, rho = 1) of log-space
    leaves of any shape (filter.py:510-664): a = (-gamma + i theta (1 - gamma))
    dt / tau, C1 = e^a, tap0 = gamma (dt/tau) (e^a - 1)/a + gamma C1,
    tap1 = -gamma C1.  CUDA leaves take the fused kernel pair
    (ops.TwoTapCoefficients); the torch expressions below are the same
    formulas."""
    if log_theta.is_cuda:
        return ops.TwoTapCoefficients.apply(log_theta, log_gamma, dt, tau)
    gamma = log_gamma.exp()
    theta = log_theta.exp()
    a = torch.complex(-gamma / tau, (theta / tau) * (1.0 - gamma)) * dt
    c1 = torch.exp(a)
    b_bar = (dt / tau) * _expm1_div_x(a)
    extra = gamma * c1  # gamma * rho * C1 with rho = 1
    tap0 = gamma * b_bar + extra
    tap1 = -extra
    return c1.to(torch.complex64), tap0.to(torch.complex64), tap1.to(torch.complex64)


def stacked_two_tap(layers) -> list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
    """two_tap() of every layer, computed once on the stacked (L, F) leaves
    when the layers share dt, tau and width: the same arithmetic, with one
    launch per op for the whole stack instead of one per layer (and likewise
    in the backward)."""
    layers = list(layers)
    same = len(layers) > 1 and all(
        r.dt == layers[0].dt and r.tau == layers[0].tau and
        r.log_theta.shape == layers[0].log_theta.shape for r in layers)
    if not same:
        return [r.two_tap() for r in layers]
    c1, t0, t1 = two_tap_coefficients(torch.stack([r.log_theta for r in layers]),
                                      torch.stack([r.log_gamma for r in layers]),
                                      layers[0].dt, layers[0].tau)
    return [(c1[i], t0[i], t1[i]) for i in range(len(layers))]


class RQFCoefficients(nn.Module):
    """Log-space RQF leaves (resonant recipe, seq_duration set) and their ZOH
    prospective two-tap coefficients (tau mode, rho = 1)."""

    def __init__(self, num_filters: int, dt: float, tau: float, seq_duration: float,
                 filter_max_freq_factor: float = 1.0, generator: torch.Generator | None = None):
        super().__init__()
        self.dt = float(dt)
        self.tau = float(tau)
        self.seq_duration = float(seq_duration)
        lo = math.log(2 * math.pi * tau / seq_duration)
        hi = math.log(2 * math.pi * filter_max_freq_factor)
        u = torch.rand(num_filters, generator=generator)
        log_theta = lo + u * (hi - lo)
        theta = log_theta.exp()
        gamma = (theta / (1.0 + theta)).clamp(1e-6, 1.0 - 1e-6)
        self.log_theta = nn.Parameter(log_theta)
        self.log_gamma = nn.Parameter(gamma.log())
        # theta band [2 pi tau / T, 2 pi tau * (1/tau)] and gamma band [1e-6, 1 - 1e-6]
        self._theta_bounds = (lo, math.log(2 * math.pi))
        self._gamma_bounds = (math.log(1e-6), math.log(1.0 - 1e-6))

    def two_tap(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        return two_tap_coefficients(self.log_theta, self.log_gamma, self.dt, self.tau)

    @torch.no_grad()
    def clamp_parameters(self) -> None:
        self.log_theta.clamp_(*self._theta_bounds)
        self.log_gamma.clamp_(*self._gamma_bounds)


class _TBPTTStack(torch.autograd.Function):
    """Consecutive TBPTT(1) layers as one autograd node.  Each layer: z = W @ h,
    the TBPTT(1) two-tap scan in (F,B,T), and the skip h_out = out + h fused
    into the scan's store.  The lag-tap cotangent updates W only — the
    reference gets the same by feeding the lag tap from a second GEMM
    W(x.detach()) (pure.py:184-187) — so the kernel hands back gz + gzw for
    the weight cotangent, and the input cotangent is W^H gz + g (g the skip's
    cotangent) in one GEMM, accumulated into the backward's own cotangent
    buffer after the top layer (ops.projection with inplace).  Arguments as
    _PureStack's."""

    @staticmethod
    def forward(ctx, h, acts, skips, *params):
        m = len(acts)
        Ws, c1s, t0s, t1s = (params[i * m:(i + 1) * m] for i in range(4))
        inputs, saved = [], []
        for i in range(m):
            inputs.append(h)
            h, sv = _block_forward(Ws[i], h, c1s[i], t0s[i], t1s[i], bool(acts[i]),
                                   h if skips[i] else None)
            saved.extend(sv)
        ctx.save_for_backward(*inputs, *Ws, *saved)
        ctx.acts, ctx.skips = tuple(map(bool, acts)), tuple(map(bool, skips))
        return h

    @staticmethod
    @once_differentiable
    def backward(ctx, g):
        m = len(ctx.acts)
        st = ctx.saved_tensors
        inputs, Ws = st[:m], st[m:2 * m]
        saved = [st[2 * m + 5 * i:2 * m + 5 * i + 5] for i in range(m)]
        need = ctx.needs_input_grad
        gW, gc1, gt0, gt1 = ([None] * m for _ in range(4))
        g = ops._c64(g)
        for i in range(m - 1, -1, -1):
            gc1[i], gt0[i], gt1[i], gz, gsum = ops._tbptt_backward_wsum(saved[i], g,
                                                                        ctx.acts[i])
            if need[3 + i]:
                gW[i] = _weight_grad(gsum, inputs[i])
            del gsum
            if i > 0 or need[0]:
                acc = g if ctx.skips[i] else None
                g = _project(Ws[i], gz, conj_transpose=True, acc=acc, inplace=i < m - 1)
        return (g if need[0] else None, None, None, *gW, *gc1, *gt0, *gt1)


class _PureBlock(torch.autograd.Function):
    """One full-BPTT Pure RQF block in (F,B,T): z = W @ h, two-tap scan with
    split-ReLU (or raw), and the complex skip h_out = out + h fused into the
    scan's store (pure.py:_forward_fbt :212-243 and :535).  Backward: the
    fused scan VJP on the output cotangent g, then one accumulating GEMM
    gh = W^H gz + g (the skip's cotangent is g) and gW = gz h^H, all three on
    the split-TF32 tcgen05 GEMMs (ops.projection, ops.projection_weight_grad)."""

    @staticmethod
    def forward(ctx, h, W, C1, tap0, tap1, fuse_act, skip):
        out, saved = _block_forward(W, h, C1, tap0, tap1, bool(fuse_act), h if skip else None)
        ctx.save_for_backward(h, W, *saved)
        ctx.fuse_act, ctx.skip = bool(fuse_act), bool(skip)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, g):
        h, W, *saved = ctx.saved_tensors
        gc1, gt0, gt1, gz = ops._fbt_backward(saved, g, ctx.fuse_act)
        need = ctx.needs_input_grad
        gh = None
        if need[0]:
            gh = _project(W, gz, conj_transpose=True, acc=ops._c64(g) if ctx.skip else None)
        gW = _weight_grad(gz, h) if need[1] else None
        return gh, gW, gc1, gt0, gt1, None, None


class _PureStack(torch.autograd.Function):
    """Consecutive full-BPTT Pure RQF blocks (pure.py:_forward_fbt_stack
    :530-536, each block as in _PureBlock) as one autograd node, so that the
    backward can hand each block's output cotangent straight to the scan VJP
    of the block below inside one launch: for blocks i-1 < i,
    ops.projection_block_scan_backward computes g_{i-1} = W_i^H gz_i + g_i
    (g_i the skip's cotangent) and, in the same GEMM's epilogue, block i-1's
    scan VJP of it from its saved context (every (F,B,T) forward saves the
    entry states it replays), so g_{i-1} is not read back.  Where that launch
    is not expected to pay (_backward_pair_chosen), the pair takes the
    separate GEMM and (F,B,T) backward, as _PureBlock does.  Arguments: h, then per-block tuples of
    flags (fuse_act, skip), then the blocks' W, C1, tap0 and tap1 in that
    order."""

    @staticmethod
    def forward(ctx, h, acts, skips, *params):
        m = len(acts)
        Ws, c1s, t0s, t1s = (params[i * m:(i + 1) * m] for i in range(4))
        inputs, saved = [], []
        for i in range(m):
            inputs.append(h)
            h, sv = _block_forward(Ws[i], h, c1s[i], t0s[i], t1s[i], bool(acts[i]),
                                   h if skips[i] else None)
            saved.extend(sv)
        ctx.save_for_backward(*inputs, *Ws, *saved)
        ctx.acts, ctx.skips = tuple(map(bool, acts)), tuple(map(bool, skips))
        return h

    @staticmethod
    @once_differentiable
    def backward(ctx, g):
        m = len(ctx.acts)
        st = ctx.saved_tensors
        inputs, Ws = st[:m], st[m:2 * m]
        saved = [st[2 * m + 5 * i:2 * m + 5 * i + 5] for i in range(m)]
        need = ctx.needs_input_grad
        gW, gc1, gt0, gt1 = ([None] * m for _ in range(4))
        g = ops._c64(g)
        vjp = ops._fbt_backward(saved[m - 1], g, ctx.acts[m - 1])
        for i in range(m - 1, -1, -1):
            gc1[i], gt0[i], gt1[i], gz = vjp
            acc = g if ctx.skips[i] else None
            if i > 0 and _backward_pair_chosen(Ws[i], gz):
                g, vjp = ops.projection_block_scan_backward(Ws[i], gz, acc, saved[i - 1],
                                                            ctx.acts[i - 1])
            elif i > 0 or need[0]:
                # after the top block, g is this backward's own buffer: sum into it
                g = _project(Ws[i], gz, conj_transpose=True, acc=acc, inplace=i < m - 1)
                if i > 0:
                    vjp = ops._fbt_backward(saved[i - 1], g, ctx.acts[i - 1])
            if need[3 + i]:
                gW[i] = _weight_grad(gz, inputs[i])
        return (g if need[0] else None, None, None, *gW, *gc1, *gt0, *gt1)


class _InputBlock(torch.autograd.Function):
    """The input projection and the first full-BPTT block together
    (pure.py:_forward_fbt_stack :522-534 and the block's _forward_fbt
    :212-243).  h0 = w_in x (+ b_in) has rank <= I = input_dims, so the
    block's projection z0 = W h0 = (W w_in) x (+ W b_in) needs no F x F GEMM
    (rqf_lowrank_drive writes z0 and h0 in one pass), and neither do its
    cotangents, with G = gz0 [x; 1]^T (rqf_rowdot, one pass over gz0):
      gW = gz0 h0^H = G [w_in, b_in]^T                      (h0 is real)
      grad [w_in, b_in] = Re(g_h0 [x; 1]^T),  g_h0 = W^H gz0 + g (skip),
    i.e. Re(W^H G + g [x; 1]^T), the second term one pass over g.  The
    reference's _Layer0RealScan (fbt_scan_kernel.py:899-1032) takes the same
    block's real input as a stacked real GEMM; the rank of h0 removes the
    F x F GEMM altogether.  x itself
    gets no gradient (the encoder routes inputs that need one through the
    general blocks)."""

    @staticmethod
    def forward(ctx, x_cf, w_in, b_in, W, C1, tap0, tap1, fuse_act, skip, B, T):
        F = W.shape[0]
        beta = W @ b_in.to(torch.complex64) if b_in is not None else None
        U = W @ w_in.to(torch.complex64)
        ctx.rank1 = w_in.shape[1] == 1 and ops.rank1_supported(F, B, T)
        if ctx.rank1:  # the drive and skip made inside the scan from x
            out, saved = ops.rank1_block_forward(U[:, 0], beta, w_in[:, 0] if skip else None,
                                                 b_in, x_cf.view(B, T), C1, tap0, tap1,
                                                 bool(fuse_act))
        else:
            z, h0 = ops.lowrank_drive(U, x_cf, beta, w_in if skip else None, b_in)
            out, saved = ops._fbt_forward(C1, tap0, tap1, z.view(F, B, T), bool(fuse_act),
                                          h0.view(F, B, T) if skip else None)
        ctx.save_for_backward(x_cf, w_in, b_in, W, *[t for t in saved if t is not None])
        ctx.has_beta = beta is not None
        ctx.fuse_act, ctx.skip = bool(fuse_act), bool(skip)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, g):
        x_cf, w_in, b_in, W, *saved = ctx.saved_tensors
        need = ctx.needs_input_grad
        I, has_b = w_in.shape[1], b_in is not None
        Gs = None
        if ctx.rank1:
            c1, t0, t1, u, *rest = saved
            beta = rest.pop(0) if ctx.has_beta else None
            xx, carries = rest
            gc1, gt0, gt1, G, Gs = ops.rank1_block_backward(
                (c1, t0, t1, u, beta, xx, carries), g, ctx.fuse_act, has_b, ctx.skip)
        else:
            gc1, gt0, gt1, gz = ops._fbt_backward(saved, g, ctx.fuse_act)
            G = ops.rowdot(gz, x_cf, with_sum=has_b)  # (F, I + has_b)
            if ctx.skip:
                Gs = ops.rowdot(g, x_cf, with_sum=has_b)
        gW = gw_in = gb_in = None
        if need[3]:
            rows = torch.cat([w_in, b_in[:, None]], dim=1) if has_b else w_in
            gW = G @ rows.t().to(torch.complex64)
        if need[1] or need[2]:
            gh = W.mH @ G
            if ctx.skip:
                gh = gh + Gs
            gw_in = gh[:, :I].real.contiguous() if need[1] else None
            gb_in = gh[:, I].real.contiguous() if (has_b and need[2]) else None
        return None, gw_in, gb_in, gW, gc1, gt0, gt1, None, None, None, None


class _InputTBPTT(torch.autograd.Function):
    """The input projection and the first TBPTT(1) layer together, with the
    skip add (the TBPTT counterpart of _InputBlock; pure.py:184-187 for the
    lag tap).  z0 = (W w_in) x (+ W b_in) from rqf_lowrank_drive, the TBPTT(1)
    scan, then out = y + h0.  With G = gz0 [x; 1]^T and Gs = (gz0 + gzw) [x; 1]^T
    (the kernel returns gz0 + gzw):
      gW = (gz0 + gzw) h0^H = Gs [w_in, b_in]^T
      grad [w_in, b_in] = Re(W^H G + g [x; 1]^T)   (the lag cotangent updates W only).

    The forward is the full-BPTT block's: with one input channel it runs on
    the rank-1 kernel (z0 and the skip made from x inside the scan, the skip
    add fused), and so does the backward (rqf_fbt_rank1_tbptt_backward: the
    states replayed from the saved entries with z0 made from x, and G, Gs and
    the sums of gz0 + gzw returned as row sums instead of gz0 and gz0 + gzw)."""

    @staticmethod
    def forward(ctx, x_cf, w_in, b_in, W, C1, tap0, tap1, fuse_act, skip, B, T):
        F = W.shape[0]
        beta = W @ b_in.to(torch.complex64) if b_in is not None else None
        U = W @ w_in.to(torch.complex64)
        ctx.rank1 = w_in.shape[1] == 1 and ops.rank1_supported(F, B, T)
        ctx.fuse_act, ctx.skip = bool(fuse_act), bool(skip)
        if ctx.rank1:
            out, saved = ops.rank1_block_forward(U[:, 0], beta, w_in[:, 0] if skip else None,
                                                 b_in, x_cf.view(B, T), C1, tap0, tap1,
                                                 bool(fuse_act))
            ctx.has_beta = beta is not None
            ctx.save_for_backward(x_cf, w_in, b_in, W, *[t for t in saved if t is not None])
            return out
        z, h0 = ops.lowrank_drive(U, x_cf, beta, w_in if skip else None, b_in)
        y, saved = ops._fbt_forward(C1, tap0, tap1, z.view(F, B, T), bool(fuse_act))
        ctx.save_for_backward(x_cf, w_in, b_in, W, *saved)
        return y + h0.view(F, B, T) if skip else y

    @staticmethod
    @once_differentiable
    def backward(ctx, g):
        x_cf, w_in, b_in, W, *saved = ctx.saved_tensors
        need = ctx.needs_input_grad
        I, has_b = w_in.shape[1], b_in is not None
        if ctx.rank1:
            c1, t0, t1, u, *rest = saved
            beta = rest.pop(0) if ctx.has_beta else None
            xx, carries = rest
            gc1, gt0, gt1, G, Gw, Gs = ops.rank1_tbptt_backward(
                (c1, t0, t1, u, beta, xx, carries), g, ctx.fuse_act, has_b, ctx.skip)
        else:
            gc1, gt0, gt1, gz, gsum = ops._tbptt_backward_wsum(saved, g, ctx.fuse_act)
            G = ops.rowdot(gz, x_cf, with_sum=has_b)
            Gw = ops.rowdot(gsum, x_cf, with_sum=has_b) if need[3] else None
            Gs = ops.rowdot(g, x_cf, with_sum=has_b) if ctx.skip else None
        gW = gw_in = gb_in = None
        if need[3]:
            rows = torch.cat([w_in, b_in[:, None]], dim=1) if has_b else w_in
            gW = Gw @ rows.t().to(torch.complex64)
        if need[1] or need[2]:
            gh = W.mH @ G
            if ctx.skip:
                gh = gh + Gs
            gw_in = gh[:, :I].real.contiguous() if need[1] else None
            gb_in = gh[:, I].real.contiguous() if (has_b and need[2]) else None
        return None, gw_in, gb_in, gW, gc1, gt0, gt1, None, None, None, None


class PureRQFEncoderB200(nn.Module):
    """Pure RQF encoder in (F,B,T) layout on the B200 scan kernels.

    forward(x: (B,T,input_dims) real) -> complex (F,B,T) features."""

    def __init__(self, input_dims: int = 1, hidden_dims: int = 128, num_layers: int = 6,
                 samp_frequency: float = 16000.0, tau: float = 0.0003125,
                 seq_duration: float = 1.0, skip_connection: bool = True,
                 final_activation: bool = False, input_proj_bias: bool = False,
                 scan_grad_mode: str = "full", seed: int = 0):
        super().__init__()
        if scan_grad_mode not in ("full", "tbptt1"):
            raise ValueError(f"scan_grad_mode must be 'full' or 'tbptt1', got {scan_grad_mode!r}")
        g = torch.Generator().manual_seed(seed)
        self.hidden = hidden_dims
        self.skip = skip_connection
        self.final_activation = final_activation
        self.scan_grad_mode = scan_grad_mode
        self.input_proj = nn.Linear(input_dims, hidden_dims, bias=input_proj_bias)
        dt = 1.0 / samp_frequency
        self.rqf = nn.ModuleList(
            RQFCoefficients(hidden_dims, dt, tau, seq_duration, generator=g)
            for _ in range(num_layers))
        ws = []
        for i in range(num_layers):
            std = rqf_forward_std(hidden_dims, 1.0 if i == 0 else SPLIT_RELU_GAIN)
            re = torch.randn(hidden_dims, hidden_dims, generator=g) * std
            im = torch.randn(hidden_dims, hidden_dims, generator=g) * std
            ws.append(nn.Parameter(torch.complex(re, im)))
        self.W = nn.ParameterList(ws)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, I = x.shape
        x_cf = x.permute(2, 0, 1).reshape(I, B * T)
        w_in, b_in = self.input_proj.weight, self.input_proj.bias
        n = len(self.W)
        coeffs = stacked_two_tap(self.rqf)
        first = 0
        if (PROJECTION == "tc" and x.is_cuda and n > 0 and I <= LOWRANK_MAX_INPUTS
                and (B * T) % 2 == 0 and not x.requires_grad):
            c1, t0, t1 = coeffs[0]
            W = self.W[0]
            block = _InputTBPTT if self.scan_grad_mode == "tbptt1" else _InputBlock
            h = block.apply(x_cf, w_in, b_in, W, c1, t0, t1, self.final_activation or n > 1,
                            self.skip and W.shape[0] == W.shape[1], B, T)
            first = 1
        else:
            proj = w_in @ x_cf if b_in is None else torch.addmm(b_in[:, None], w_in, x_cf)
            h = proj.reshape(-1, B, T).to(torch.complex64)
        blocks = range(first, n)
        acts = tuple(self.final_activation or i + 1 < n for i in blocks)
        skips = tuple(self.skip and self.W[i].shape[0] == self.W[i].shape[1] for i in blocks)
        if len(blocks) > 0:
            stack = _TBPTTStack if self.scan_grad_mode == "tbptt1" else _PureStack
            h = stack.apply(h, acts, skips, *(self.W[i] for i in blocks),
                            *(coeffs[i][0] for i in blocks), *(coeffs[i][1] for i in blocks),
                            *(coeffs[i][2] for i in blocks))
        return h

    @torch.no_grad()
    def clamp_parameters(self) -> None:
        for r in self.rqf:
            r.clamp_parameters()


class _ReadoutHidden(torch.autograd.Function):
    """hid = relu(W1 @ [Re h; Im h] + b1) over the (F, B*T) view of h, on the
    split-TF32 tensor-core projections (the real-output forward and the
    real-operand cotangents; used for per-step logits).

    With V = W1[:, :F] - i W1[:, F:] (complex H x F), W1 @ [Re h; Im h] is
    Re(V h), computed directly (rqf_projection_real_out); with the real
    cotangent g the input cotangent is V^H g (rqf_projection_real) and the
    weight cotangent P = g h^H (rqf_projection_weight_grad_real) gives
    [Re P, -Im P].  No [Re; Im] copy of h is made."""

    @staticmethod
    def forward(ctx, h, W1, b1):
        F = h.shape[0]
        V = torch.complex(W1[:, :F], -W1[:, F:]).contiguous()
        # bias and ReLU in one pass over the projection, the decisions kept as bits
        hid, mask = ops.readout_bias_relu(ops.projection_real_out(V, h), b1)
        ctx.save_for_backward(h, V, mask)
        return hid

    @staticmethod
    @once_differentiable
    def backward(ctx, ghid):
        h, V, mask = ctx.saved_tensors
        need = ctx.needs_input_grad
        # real: the real-operand forms of both cotangent GEMMs
        g, rowsum = ops.readout_bias_relu_backward(ghid, mask)
        gh = ops.projection_real(V, g, conj_transpose=True) if need[0] else None
        gW1 = None
        if need[1]:
            P = ops.projection_weight_grad_real(g, h)
            gW1 = torch.cat([P.real, -P.imag], dim=1)
        gb1 = rowsum.sum(dim=1) if need[2] else None
        return gh, gW1, gb1


class _ReadoutPooled(torch.autograd.Function):
    """pooled = mean_t relu(W1 [Re h; Im h] + b1), (H, B), for the mean-pooled
    readout (train.py:ComplexReadoutClassifier :126-136): the real part
    Re(V h) of _ReadoutHidden's projection (rqf_projection_real_out, which
    computes only that), then one pass (rqf_readout_relu_pool) that
    keeps only the ReLU mask bits and the time-means.  Backward: the mask
    turns gpool into the real g = mask * gpool / T
    (rqf_readout_relu_pool_backward), which feeds the real-operand forms of
    the two projection cotangents (rqf_projection_real,
    rqf_projection_weight_grad_real); gb1 = sum_b gpool / T * (set bits of
    the (h, b) row)."""

    @staticmethod
    def forward(ctx, h, W1, b1):
        F = h.shape[0]
        V = torch.complex(W1[:, :F], -W1[:, F:]).contiguous()
        pooled, mask = ops.readout_relu_pool(ops.projection_real_out(V, h), b1)
        ctx.save_for_backward(h, V, mask)
        ctx.time = h.shape[2]
        return pooled

    @staticmethod
    @once_differentiable
    def backward(ctx, gpool):
        h, V, mask = ctx.saved_tensors
        need = ctx.needs_input_grad
        scale = gpool / ctx.time
        g, counts = ops.readout_relu_pool_backward(mask, scale, ctx.time)
        gh = ops.projection_real(V, g, conj_transpose=True) if need[0] else None
        gW1 = None
        if need[1]:
            P = ops.projection_weight_grad_real(g, h)
            gW1 = torch.cat([P.real, -P.imag], dim=1)
        gb1 = (scale * counts).sum(dim=1) if need[2] else None
        return gh, gW1, gb1


class ComplexReadout(nn.Module):
    """Per-timestep MLP on [Re h; Im h] with mean-pooled logits
    (train.py:ComplexReadoutClassifier, hidden_dims set).

    On CUDA with the tensor-core projections (the default), the output layer
    is applied to the time-mean of the hidden activations with mean pooling:
    mean_t(W2 hid_t + b2) = W2 mean_t(hid_t) + b2, the same logits without
    the per-step output GEMM; the hidden layer then runs as _ReadoutPooled
    (no per-step activations are kept, only the ReLU mask bits).  Per-step
    logits run _ReadoutHidden."""

    def __init__(self, features: int, num_classes: int, hidden_dims: int = 256, seed: int = 1):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.fc1 = nn.Linear(2 * features, hidden_dims)
        self.fc2 = nn.Linear(hidden_dims, num_classes)
        with torch.no_grad():
            bound = 1.0 / math.sqrt(2 * features)
            self.fc1.weight.uniform_(-bound, bound, generator=g)
            self.fc1.bias.uniform_(-bound, bound, generator=g)
            self.fc2.weight.normal_(0.0, 1e-3, generator=g)
            self.fc2.bias.zero_()

    def forward(self, h: torch.Tensor, per_step: bool = False) -> torch.Tensor:
        F, B, T = h.shape
        if PROJECTION == "tc" and h.is_cuda:
            if not per_step:
                pooled = _ReadoutPooled.apply(h, self.fc1.weight, self.fc1.bias)  # (H, B)
                return torch.addmm(self.fc2.bias[:, None], self.fc2.weight, pooled).t()
            hid = _ReadoutHidden.apply(h, self.fc1.weight, self.fc1.bias)  # (H, B, T)
            logits = torch.addmm(self.fc2.bias[:, None], self.fc2.weight,
                                 hid.reshape(hid.shape[0], B * T))
            return logits.reshape(-1, B, T).permute(1, 2, 0)  # (B, T, C)
        feats = torch.cat([h.real, h.imag], dim=0).reshape(2 * F, B * T)
        hid = torch.relu(torch.addmm(self.fc1.bias[:, None], self.fc1.weight, feats))
        logits = torch.addmm(self.fc2.bias[:, None], self.fc2.weight, hid)  # (C, B*T)
        logits = logits.reshape(-1, B, T)
        if per_step:
            return logits.permute(1, 2, 0)  # (B, T, C)
        return logits.mean(dim=2).t()  # (B, C)


# Split of the sample reduction in the per-step output layer's weight
# cotangent (batched GEMMs over this many sample chunks, then their sum);
# 0: one GEMM over all samples.
OUTPUT_GRAD_SPLITS = int(os.environ.get("RQF_B200_OUTPUT_GRAD_SPLITS", "64"))


class _PerStepLogits(torch.autograd.Function):
    """logits = W2 @ hid + b2 over the (H, N) samples of the per-step readout,
    as torch.addmm; backward as addmm's, except that the weight cotangent
    dl @ hid^T, a reduction over all N samples with only C x H outputs,
    runs as OUTPUT_GRAD_SPLITS batched GEMMs over sample chunks and their sum
    (one GEMM of depth N leaves most SMs idle)."""

    @staticmethod
    def forward(ctx, hid, W2, b2):
        ctx.save_for_backward(hid, W2)
        return torch.addmm(b2[:, None], W2, hid)

    @staticmethod
    @once_differentiable
    def backward(ctx, dl):
        hid, W2 = ctx.saved_tensors
        need = ctx.needs_input_grad
        gh = W2.t() @ dl if need[0] else None
        gW = None
        if need[1]:
            (C, N), H, S = dl.shape, hid.shape[0], OUTPUT_GRAD_SPLITS
            if S > 1 and N % S == 0 and dl.is_contiguous() and hid.is_contiguous():
                n = N // S
                gW = torch.bmm(dl.view(C, S, n).transpose(0, 1),
                               hid.view(H, S, n).permute(1, 2, 0)).sum(dim=0)
            else:
                gW = dl @ hid.t()
        gb = dl.sum(dim=1) if need[2] else None
        return gh, gW, gb


class RQFClassifier(nn.Module):
    def __init__(self, encoder: PureRQFEncoderB200, num_classes: int, hidden_dims: int = 256):
        super().__init__()
        self.encoder = encoder
        self.readout = ComplexReadout(encoder.hidden, num_classes, hidden_dims)

    def forward(self, x: torch.Tensor, per_step: bool = False) -> torch.Tensor:
        return self.readout(self.encoder(x), per_step=per_step)

    def per_step_loss(self, x: torch.Tensor, y: torch.Tensor,
                      label_smoothing: float = 0.0) -> torch.Tensor:
        """train.py:per_step_cross_entropy (:663-674) of forward(x, per_step=True)
        against the batch labels y.  On the tensor-core path the logits stay in
        the output GEMM's (classes, batch*time) layout and the loss and its
        gradient run in one pass each (ops.per_step_cross_entropy)."""
        h = self.encoder(x)
        F, B, T = h.shape
        ro = self.readout
        if PROJECTION == "tc" and h.is_cuda:
            hid = _ReadoutHidden.apply(h, ro.fc1.weight, ro.fc1.bias)  # (H, B, T)
            logits = _PerStepLogits.apply(hid.reshape(hid.shape[0], B * T), ro.fc2.weight,
                                          ro.fc2.bias)                  # (C, B*T)
            return ops.per_step_cross_entropy(logits, y, B, T, label_smoothing)
        logits = ro(h, per_step=True)
        return torch.nn.functional.cross_entropy(
            logits.reshape(B * T, -1), y[:, None].expand(B, T).reshape(-1),
            label_smoothing=label_smoothing)
