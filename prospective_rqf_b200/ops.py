"""B200 drop-in for the rqf_models.ops scan entry points.

Each public callable keeps the name, signature, return convention and
gradient convention (PyTorch conjugate-Wirtinger, ``None`` for inputs that do
not need a gradient) of the reference callable it replaces; the compute runs
in librqf_b200.so through the C ABI of include/rqf_b200.h.  There is no CPU
or Triton fallback: non-CUDA inputs raise.

Reference callables (paths inside the reference project):
  _triton_chunked_scan              rqf_models/ops/chunked_scan_kernel.py:340
  _triton_chunked_scan_prospective  rqf_models/ops/chunked_scan_kernel.py:506
  fbt_prospective_scan              rqf_models/ops/fbt_scan_kernel.py:332
  fbt_recompute_scan                rqf_models/ops/fbt_scan_kernel.py:667
  fbt_layer0_real_scan              rqf_models/ops/fbt_scan_kernel.py:1005
  sequential_scan / parallel_scan   rqf_models/ops/scan.py:290 / :435 (CUDA branch)
  sequential_scan_abs               rqf_models/ops/scan.py:381
  _sequential_scan_forward_abs_raw_block_f        triton_scan_kernel.py:507
  _sequential_scan_real_forward_abs_raw_block_f   triton_scan_kernel.py:1531
  _triton_sequential_scan_multi_osc (+ _real, parallel, abs forms)
                                    triton_scan_kernel.py:2499, :3071, :4106, :2019, :2688
New (no single reference callable; replaces the autograd surrogate of
rqf_models/backbones/rqf/block.py:_scan_two_tap_with_grad_mode :904-954 and
_scan_with_grad_mode :882-902):
  tbptt1_two_tap_scan, tbptt1_scan
"""

from __future__ import annotations

import contextlib
import ctypes
import os

import torch
from torch.autograd.function import once_differentiable

from . import _abi, _timing

_SYNC_CHECK = os.environ.get("RQF_B200_SYNC_CHECK", "0") == "1"

__all__ = [
    "_triton_chunked_scan",
    "_triton_chunked_scan_prospective",
    "fbt_prospective_scan",
    "fbt_recompute_scan",
    "fbt_layer0_real_scan",
    "tbptt1_two_tap_scan",
    "tbptt1_scan",
    "sequential_scan",
    "parallel_scan",
    "sequential_scan_abs",
    "selective_forward",
    "selective_backward",
    "selective_layer_scan",
]


# ------------------------------------------------------------------ helpers
def _c64(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.complex64:
        t = t.to(torch.complex64)
    return t.resolve_conj().resolve_neg().contiguous()


def _require_cuda(*ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "prospective_rqf_b200 runs on CUDA tensors only (no CPU fallback); "
                f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _coef(t: torch.Tensor, n: int, name: str) -> torch.Tensor:
    t = _c64(t)
    if t.dim() != 1 or t.shape[0] != n:
        raise ValueError(f"{name} must have shape ({n},), got {tuple(t.shape)}")
    return t


def _scratch(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def _carries(n: int, device) -> torch.Tensor:
    return torch.empty(max(int(n), 1), dtype=torch.complex64, device=device)


def _done(device) -> None:
    if _SYNC_CHECK:
        _abi.check_device_errors(device)


def _nbytes(*tensors) -> int:
    """Algorithmic bytes of one launch: each large operand read or written once."""
    return sum(t.numel() * t.element_size() for t in tensors if t is not None)


# (B,T,F) kernel family for the next forwards: 0 automatic (by the number of
# chains of batch x 32 channels), 1 streaming, 2 tile-resident.  Every forward
# records the value it was given in its saved context and its backward passes
# that same value, so the two always use the same family (their saved entry
# states differ).
_BTF_PATH = 0


@contextlib.contextmanager
def btf_kernel_family(path: int):
    """Force one (B,T,F) kernel family for the forwards run inside (tests,
    microbenchmarks); 0 restores the automatic choice."""
    global _BTF_PATH
    if path not in (0, 1, 2):
        raise ValueError(f"path must be 0, 1 or 2, got {path!r}")
    prev, _BTF_PATH = _BTF_PATH, int(path)
    try:
        yield
    finally:
        _BTF_PATH = prev


def _shape3(x: torch.Tensor, what: str):
    if x.dim() != 3:
        raise ValueError(f"{what} must be 3-D, got shape {tuple(x.shape)}")
    return tuple(int(s) for s in x.shape)


# ------------------------------------------------------ (B,T,F) plain scan
class _ChunkedScanFunction(torch.autograd.Function):
    """y[t] = C1*y[t-1] + C2*u[t] on (B,T,F); saves C1, C2, u and one carry per
    tile (chunked_scan_kernel.py:_ChunkedScanFunction :306-337 saves the full
    output instead)."""

    @staticmethod
    def forward(ctx, C1, C2, u):
        dev = _require_cuda(C1, C2, u)
        real = not u.is_complex()
        uu = u.to(torch.float32).contiguous() if real else _c64(u)
        B, T, F = _shape3(uu, "u")
        c1, c2 = _coef(C1, F, "C1"), _coef(C2, F, "C2")
        lib = _abi.load()
        y = torch.empty((B, T, F), dtype=torch.complex64, device=dev)
        carries = _carries(lib.rqf_btf_carry_count(B, T, F), dev)
        scratch = _scratch(lib.rqf_btf_scratch_bytes(B, T, F), dev)
        with _timing.launch("rqf_chunked_scan_forward", B * T * F, _nbytes(uu, y)):
            _abi.check(lib.rqf_chunked_scan_forward(
                _abi.ptr(c1), _abi.ptr(c2), _abi.ptr(uu), int(real), _abi.ptr(y), _abi.ptr(carries),
                _abi.ptr(scratch), B, T, F, _BTF_PATH, _abi.stream_of(uu)),
                "rqf_chunked_scan_forward")
        _done(dev)
        ctx.save_for_backward(c1, c2, uu, carries)
        ctx.real, ctx.path = real, _BTF_PATH
        return y

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        c1, c2, uu, carries = ctx.saved_tensors
        B, T, F = uu.shape
        dev = uu.device
        gy = _c64(grad_output)
        lib = _abi.load()
        gu = torch.empty_like(uu)
        gc1 = torch.empty_like(c1)
        gc2 = torch.empty_like(c2)
        scratch = _scratch(lib.rqf_btf_scratch_bytes(B, T, F), dev)
        with _timing.launch("rqf_chunked_scan_backward", B * T * F, _nbytes(uu, gy, gu)):
            _abi.check(lib.rqf_chunked_scan_backward(
                _abi.ptr(c1), _abi.ptr(c2), _abi.ptr(uu), int(ctx.real), _abi.ptr(carries),
                _abi.ptr(gy), _abi.ptr(gu), _abi.ptr(gc1), _abi.ptr(gc2), _abi.ptr(scratch),
                B, T, F, ctx.path, _abi.stream_of(gy)), "rqf_chunked_scan_backward")
        _done(dev)
        need = ctx.needs_input_grad
        return (gc1 if need[0] else None, gc2 if need[1] else None, gu if need[2] else None)


def _triton_chunked_scan(C1: torch.Tensor, C2: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """x[n] = C1*x[n-1] + C2*u[n] on (batch, time, filters) — drop-in for
    rqf_models/ops/chunked_scan_kernel.py:_triton_chunked_scan (:340).  A real
    ``u`` is scanned without promotion (same values as scan.py:366's cast)."""
    return _ChunkedScanFunction.apply(C1, C2, u)


# ------------------------------------------------ (B,T,F) two-tap scan
class _ChunkedProspectiveScanFunction(torch.autograd.Function):
    """y[n] = C1 y[n-1] + tap0 x[n] + tap1 x[n-1] on (B,T,F)
    (chunked_scan_kernel.py:_ChunkedProspectiveScanFunction :474-503)."""

    @staticmethod
    def forward(ctx, C1, tap0, tap1, x):
        dev = _require_cuda(C1, tap0, tap1, x)
        xx = _c64(x)
        B, T, F = _shape3(xx, "x")
        c1, t0, t1 = _coef(C1, F, "C1"), _coef(tap0, F, "tap0"), _coef(tap1, F, "tap1")
        lib = _abi.load()
        y = torch.empty((B, T, F), dtype=torch.complex64, device=dev)
        carries = _carries(lib.rqf_btf_carry_count(B, T, F), dev)
        scratch = _scratch(lib.rqf_btf_scratch_bytes(B, T, F), dev)
        with _timing.launch("rqf_chunked_prospective_forward", B * T * F, _nbytes(xx, y)):
            _abi.check(lib.rqf_chunked_prospective_forward(
                _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1), _abi.ptr(xx), _abi.ptr(y), _abi.ptr(carries),
                _abi.ptr(scratch), B, T, F, _BTF_PATH, _abi.stream_of(xx)),
                "rqf_chunked_prospective_forward")
        _done(dev)
        ctx.save_for_backward(c1, t0, t1, xx, carries)
        ctx.path = _BTF_PATH
        return y

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        c1, t0, t1, xx, carries = ctx.saved_tensors
        B, T, F = xx.shape
        dev = xx.device
        gy = _c64(grad_output)
        lib = _abi.load()
        gx = torch.empty_like(xx)
        gc1, gt0, gt1 = torch.empty_like(c1), torch.empty_like(t0), torch.empty_like(t1)
        scratch = _scratch(lib.rqf_btf_scratch_bytes(B, T, F), dev)
        with _timing.launch("rqf_chunked_prospective_backward", B * T * F, _nbytes(xx, gy, gx)):
            _abi.check(lib.rqf_chunked_prospective_backward(
                _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1), _abi.ptr(xx), _abi.ptr(carries),
                _abi.ptr(gy), _abi.ptr(gx), _abi.ptr(gc1), _abi.ptr(gt0), _abi.ptr(gt1),
                _abi.ptr(scratch), B, T, F, ctx.path, _abi.stream_of(gy)),
                "rqf_chunked_prospective_backward")
        _done(dev)
        need = ctx.needs_input_grad
        return (gc1 if need[0] else None, gt0 if need[1] else None, gt1 if need[2] else None,
                gx if need[3] else None)


def _triton_chunked_scan_prospective(C1, tap0, tap1, x):
    """Fused two-tap prospective scan on (batch, time, filters) — drop-in for
    rqf_models/ops/chunked_scan_kernel.py:_triton_chunked_scan_prospective (:506)."""
    return _ChunkedProspectiveScanFunction.apply(C1, tap0, tap1, x)


# ------------------------------------------------ (F,B,T) two-tap scan
def _fbt_forward(C1, tap0, tap1, x_fbt, fuse_act: bool, skip=None):
    """(F,B,T) two-tap scan; with `skip`, returns act(y) + skip (fused)."""
    dev = _require_cuda(C1, tap0, tap1, x_fbt, skip)
    z = _c64(x_fbt)
    F, B, T = _shape3(z, "x_fbt")
    c1, t0, t1 = _coef(C1, F, "C1"), _coef(tap0, F, "tap0"), _coef(tap1, F, "tap1")
    sk = None
    if skip is not None:
        sk = _c64(skip)
        if sk.shape != z.shape:
            raise ValueError(f"skip must have shape {tuple(z.shape)}, got {tuple(sk.shape)}")
    lib = _abi.load()
    out = torch.empty((F, B, T), dtype=torch.complex64, device=dev)
    carries = _carries(lib.rqf_fbt_carry_count(F, B, T), dev)
    scratch = _scratch(lib.rqf_fbt_scratch_bytes(F, B, T), dev)
    name = "rqf_fbt_prospective_forward" if sk is None else "rqf_fbt_block_forward"
    with _timing.launch(name, B * T * F, _nbytes(z, sk, out)):
        _abi.check(lib.rqf_fbt_block_forward(
            _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1), _abi.ptr(z), _abi.ptr(sk), _abi.ptr(out),
            _abi.ptr(carries), _abi.ptr(scratch), F, B, T, int(bool(fuse_act)),
            _abi.stream_of(z)), "rqf_fbt_block_forward")
    _done(dev)
    return out, (c1, t0, t1, z, carries)


def block_scan_eligible(W: torch.Tensor, h: torch.Tensor) -> bool:
    """Whether projection_block_scan takes this block: complex W (F, K) on
    the GPU against h (K, B, T) with T a multiple of 128 (the GEMM's sample
    tile) and B*T below 2^30."""
    return (W.is_cuda and h.is_cuda and W.dim() == 2 and h.dim() == 3
            and int(W.shape[1]) == int(h.shape[0]) and int(h.shape[0]) > 0
            and int(h.shape[2]) % 128 == 0 and int(h.shape[1]) * int(h.shape[2]) < (1 << 30))


def block_scan_preferred(W: torch.Tensor, h: torch.Tensor) -> bool:
    """Whether the fused block forward is expected to beat the projection
    followed by the separate scan.  The fused launch carries the scan state
    from each 128-sample tile to the next along time, so every (128-filter
    block, batch row) chain is a sequence of dependent tile epilogues; it
    wins when those chains nearly fill the device's CTA pairs (measured at
    F = K = 256, T = 16000: 1.40 ms fused against 1.55 ms unfused at B = 32,
    64 chains on 74 pairs; 1.17 against 0.76 ms at B = 16) and when K is
    large enough for the tensor-core work of a tile to cover its epilogue."""
    if not block_scan_eligible(W, h):
        return False
    F, K = int(W.shape[0]), int(W.shape[1])
    chains = -(-F // 128) * int(h.shape[1])
    pairs = torch.cuda.get_device_properties(h.device).multi_processor_count // 2
    return K >= 128 and 5 * chains >= 4 * pairs


def projection_block_scan(W, h, C1, tap0, tap1, fuse_act: bool, skip=None):
    """One Pure RQF block forward in one launch (rqf_projection_block_scan):
    z = W h (pure.py:223) on the split-TF32 tensor-core GEMM, whose epilogue
    runs the (F,B,T) two-tap scan of z along time, the split-ReLU and the
    skip add (pure.py:529-535) tile by tile.  Returns (out, saved) exactly as
    _fbt_forward(C1, tap0, tap1, W h, fuse_act, skip) does, so _fbt_backward
    and _tbptt_backward take ``saved`` unchanged.  Requires
    block_scan_eligible(W, h)."""
    dev = _require_cuda(W, h, C1, tap0, tap1, skip)
    w = _c64(W)
    x = _c64(h)
    if not block_scan_eligible(w, x):
        raise ValueError(f"projection_block_scan: W {tuple(w.shape)} and h {tuple(x.shape)} "
                         "need h (K, B, T) with T a multiple of 128")
    F, K = int(w.shape[0]), int(w.shape[1])
    _, B, T = (int(d) for d in x.shape)
    c1, t0, t1 = _coef(C1, F, "C1"), _coef(tap0, F, "tap0"), _coef(tap1, F, "tap1")
    sk = None
    if skip is not None:
        sk = _c64(skip)
        if tuple(sk.shape) != (F, B, T):
            raise ValueError(f"skip must have shape {(F, B, T)}, got {tuple(sk.shape)}")
    lib = _abi.load()
    z = torch.empty((F, B, T), dtype=torch.complex64, device=dev)
    out = torch.empty((F, B, T), dtype=torch.complex64, device=dev)
    carries = _carries(lib.rqf_fbt_carry_count(F, B, T), dev)
    ws = _scratch(lib.rqf_projection_block_scan_workspace_bytes(F, K, B, T), dev)
    with _timing.launch("rqf_projection_block_scan", F * B * T, _nbytes(x, z, sk, out),
                        8 * F * K * B * T):
        _abi.check(lib.rqf_projection_block_scan(
            _abi.ptr(w), _abi.ptr(x), _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1), _abi.ptr(sk),
            _abi.ptr(z), _abi.ptr(out), _abi.ptr(carries), _abi.ptr(ws), F, K, B, T,
            int(bool(fuse_act)), _abi.stream_of(x)), "rqf_projection_block_scan")
    _done(dev)
    return out, (c1, t0, t1, z, carries)


def block_scan_backward_preferred(W: torch.Tensor, gz: torch.Tensor) -> bool:
    """Whether projection_block_scan_backward is expected to beat the
    input-cotangent GEMM followed by the separate (F,B,T) backward (W (k, F)
    the upper block's weight, gz (k, B, T) its z cotangent): nowhere
    measured so far.  At F = k = 256, T = 16000 the fused launch takes
    2.25 ms at B = 32 against 1.30 + 0.55 ms for the two launches, and
    2.29 ms against 0.65 + 0.28 ms at B = 16: its epilogue (the replay, the
    reverse adjoint and the coefficient sums of 16 rows per warp, one warp
    per TMEM lane quarter) needs ~12 us per tile, longer than the tile's
    tensor-core work (~11 us), and the chains along time serialise it."""
    return False


def projection_block_scan_backward(W, gz_above, acc, saved, fuse_act: bool):
    """The lower block's output cotangent and scan VJP in one launch
    (rqf_projection_block_scan_backward): g = W^H gz_above + acc on the
    split-TF32 tensor-core GEMM (the autograd of pure.py:223's matmul for
    the upper block, acc the skip's cotangent), and in its epilogue the
    lower block's (F,B,T) scan VJP of g from its saved context ``saved``
    (c1, tap0, tap1, z, carries), which must come from projection_block_scan
    or the row kernels (every 8-sample entry state saved).  Returns
    (g, (gc1, gt0, gt1, gz)) with the second tuple as _fbt_backward(saved, g,
    fuse_act) returns it."""
    c1, t0, t1, z, carries = saved
    dev = _require_cuda(W, gz_above, acc, z)
    w = _c64(W)
    x = _c64(gz_above)
    F, B, T = (int(d) for d in z.shape)
    k = int(w.shape[0])
    if w.dim() != 2 or int(w.shape[1]) != F or tuple(x.shape) != (k, B, T):
        raise ValueError(f"projection_block_scan_backward: W {tuple(w.shape)}, gz {tuple(x.shape)} "
                         f"and z {tuple(z.shape)} do not chain")
    if not block_scan_eligible(w.mH, x):
        raise ValueError("projection_block_scan_backward needs T a multiple of 128")
    a = None
    if acc is not None:
        a = _c64(acc)
        if tuple(a.shape) != (F, B, T):
            raise ValueError(f"acc must have shape {(F, B, T)}, got {tuple(a.shape)}")
    lib = _abi.load()
    g = torch.empty_like(z)
    gz = torch.empty_like(z)
    gc1, gt0, gt1 = torch.empty_like(c1), torch.empty_like(t0), torch.empty_like(t1)
    ws = _scratch(lib.rqf_projection_block_scan_backward_workspace_bytes(F, k, B, T), dev)
    with _timing.launch("rqf_projection_block_scan_backward", F * B * T,
                        _nbytes(x, a, z, g, gz), 8 * F * k * B * T):
        _abi.check(lib.rqf_projection_block_scan_backward(
            _abi.ptr(w), _abi.ptr(x), _abi.ptr(a), _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1),
            _abi.ptr(z), _abi.ptr(carries), _abi.ptr(g), _abi.ptr(gz), _abi.ptr(gc1),
            _abi.ptr(gt0), _abi.ptr(gt1), _abi.ptr(ws), F, k, B, T, int(bool(fuse_act)),
            _abi.stream_of(x)), "rqf_projection_block_scan_backward")
    _done(dev)
    return g, (gc1, gt0, gt1, gz)


def _fbt_backward(saved, grad_output, fuse_act: bool):
    c1, t0, t1, z, carries = saved
    F, B, T = z.shape
    dev = z.device
    gy = _c64(grad_output)
    lib = _abi.load()
    gz = torch.empty_like(z)
    gc1, gt0, gt1 = torch.empty_like(c1), torch.empty_like(t0), torch.empty_like(t1)
    scratch = _scratch(lib.rqf_fbt_scratch_bytes(F, B, T), dev)
    with _timing.launch("rqf_fbt_prospective_backward", B * T * F, _nbytes(z, gy, gz)):
        _abi.check(lib.rqf_fbt_prospective_backward(
            _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1), _abi.ptr(z), _abi.ptr(carries), _abi.ptr(gy),
            _abi.ptr(gz), _abi.ptr(gc1), _abi.ptr(gt0), _abi.ptr(gt1), _abi.ptr(scratch), F, B, T,
            int(bool(fuse_act)), _abi.stream_of(gy)), "rqf_fbt_prospective_backward")
    _done(dev)
    return gc1, gt0, gt1, gz


class _FBTProspectiveScan(torch.autograd.Function):
    """(F,B,T) two-tap scan, split-ReLU output when ``fuse_act``
    (fbt_scan_kernel.py:_FBTProspectiveScan :245-329).  Saves only the tile
    carries; the backward recomputes the raw state."""

    @staticmethod
    def forward(ctx, C1, tap0, tap1, x_fbt, fuse_act):
        out, saved = _fbt_forward(C1, tap0, tap1, x_fbt, bool(fuse_act))
        ctx.save_for_backward(*saved)
        ctx.fuse_act = bool(fuse_act)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        gc1, gt0, gt1, gz = _fbt_backward(ctx.saved_tensors, grad_output, ctx.fuse_act)
        need = ctx.needs_input_grad
        return (gc1 if need[0] else None, gt0 if need[1] else None, gt1 if need[2] else None,
                gz if need[3] else None, None)


class _FBTRecompute(torch.autograd.Function):
    """Split-ReLU (F,B,T) two-tap scan storing only per-tile carries
    (fbt_scan_kernel.py:_FBTRecompute :575-664)."""

    @staticmethod
    def forward(ctx, C1, tap0, tap1, x_fbt):
        out, saved = _fbt_forward(C1, tap0, tap1, x_fbt, True)
        ctx.save_for_backward(*saved)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        gc1, gt0, gt1, gz = _fbt_backward(ctx.saved_tensors, grad_output, True)
        need = ctx.needs_input_grad
        return (gc1 if need[0] else None, gt0 if need[1] else None, gt1 if need[2] else None,
                gz if need[3] else None)


def fbt_prospective_scan(C1, tap0, tap1, x_fbt, fuse_act: bool = False):
    """Fused two-tap prospective scan in channel-outermost (filters, batch,
    time) layout — drop-in for rqf_models/ops/fbt_scan_kernel.py:
    fbt_prospective_scan (:332).  Returns split-ReLU(y) when ``fuse_act``,
    else the raw state y."""
    return _FBTProspectiveScan.apply(C1, tap0, tap1, x_fbt, fuse_act)


def fbt_recompute_scan(C1, tap0, tap1, x_fbt):
    """Split-ReLU two-tap scan with recompute-in-backward — drop-in for
    rqf_models/ops/fbt_scan_kernel.py:fbt_recompute_scan (:667)."""
    return _FBTRecompute.apply(C1, tap0, tap1, x_fbt)


# ------------------------------------- real-input first layer, (F,B,T)
class _Layer0RealScan(torch.autograd.Function):
    """z = (Wr + i Wi) h for a real h, then the split-ReLU recompute scan
    (fbt_scan_kernel.py:_Layer0RealScan :899-996).  The projection is the
    real-operand tensor-core GEMM (rqf_projection_real: a complex W against a
    real h, half the work of the complex product) writing z interleaved, so
    the scan reads it as any other layer; backward:
      grad [Wr; Wi] = [Re P; Im P],  P = gz h^T = (h gz^H)^H   (rqf_projection_weight_grad_real)
      grad h        = Re(W^H gz)                               (rqf_projection_real_out)."""

    @staticmethod
    def forward(ctx, w_stacked, h_real, C1, tap0, tap1, batch):
        dev = _require_cuda(w_stacked, h_real, C1, tap0, tap1)
        ws = w_stacked.detach().to(torch.float32)
        if ws.dim() != 2 or ws.shape[0] % 2:
            raise ValueError(f"w_stacked must be (2*filters, d_model), got {tuple(ws.shape)}")
        F = ws.shape[0] // 2
        h = h_real.detach().to(torch.float32).contiguous()
        if h.dim() != 2 or h.shape[0] != ws.shape[1]:
            raise ValueError(f"h_real must be ({ws.shape[1]}, batch*time), got {tuple(h.shape)}")
        batch = int(batch)
        cols = int(h.shape[1])
        if batch <= 0 or cols % batch:
            raise ValueError(f"{cols} columns do not split into batch {batch}")
        W = torch.complex(ws[:F], ws[F:]).contiguous()
        z = projection_real(W, h).view(F, batch, cols // batch)
        out, saved = _fbt_forward(C1, tap0, tap1, z, True)
        ctx.save_for_backward(W, h, *saved)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_act):
        W, h, *saved = ctx.saved_tensors
        gc1, gt0, gt1, gz = _fbt_backward(saved, grad_act, True)
        need = ctx.needs_input_grad
        F = W.shape[0]
        g_ws = g_h = None
        if need[0]:
            Pt = projection_weight_grad_real(h, gz.reshape(F, -1))  # h gz^H = P^H, (d, F)
            g_ws = torch.cat([Pt.real.t(), -Pt.imag.t()], dim=0).contiguous()
        if need[1]:
            g_h = projection_real_out(W.mH.contiguous(), gz.reshape(F, -1))
        return (g_ws, g_h, gc1 if need[2] else None, gt0 if need[3] else None,
                gt1 if need[4] else None, None)


def fbt_layer0_real_scan(w_stacked, h_real, C1, tap0, tap1, batch):
    """Real-input first-layer projection + split-ReLU prospective scan —
    drop-in for rqf_models/ops/fbt_scan_kernel.py:fbt_layer0_real_scan
    (:1005): w_stacked (2F, d) real [Wr; Wi], h_real (d, batch*time) real;
    returns the complex (F, batch, time) split-ReLU output."""
    return _Layer0RealScan.apply(w_stacked, h_real, C1, tap0, tap1, batch)


# ------------------------------------------------------------- TBPTT(1)
class _TBPTT1TwoTap(torch.autograd.Function):
    """Forward = the exact two-tap scan; backward = the TBPTT(1) surrogate of
    block.py:_scan_two_tap_with_grad_mode (:938-954) in one pointwise kernel:
    grad_u = conj(tap0) g (+ conj(tap1) g[t+1] when u is its own lag source),
    grad_delayed_u[t] = conj(tap1) g[t+1], coefficient grads summed with the
    recurrent state detached."""

    @staticmethod
    def forward(ctx, C1, tap0, tap1, u, delayed_u, layout, fuse_act):
        if layout not in ("btf", "fbt"):
            raise ValueError(f"layout must be 'btf' or 'fbt', got {layout!r}")
        if layout == "btf" and fuse_act:
            raise ValueError("fuse_act is supported for the (F,B,T) layout only")
        if delayed_u is not None and delayed_u.shape != u.shape:
            raise ValueError(
                f"delayed_u must have shape {tuple(u.shape)}, got {tuple(delayed_u.shape)}")
        dev = _require_cuda(C1, tap0, tap1, u, delayed_u)
        lib = _abi.load()
        if layout == "fbt":
            out, saved = _fbt_forward(C1, tap0, tap1, u, bool(fuse_act))
            c1, t0, t1, z, carries = saved
            dims = tuple(z.shape)
        else:
            z = _c64(u)
            B, T, F = _shape3(z, "u")
            c1, t0, t1 = _coef(C1, F, "C1"), _coef(tap0, F, "tap0"), _coef(tap1, F, "tap1")
            out = torch.empty((B, T, F), dtype=torch.complex64, device=dev)
            carries = _carries(lib.rqf_btf_carry_count(B, T, F), dev)
            scratch = _scratch(lib.rqf_btf_scratch_bytes(B, T, F), dev)
            with _timing.launch("rqf_chunked_prospective_forward", B * T * F, _nbytes(z, out)):
                _abi.check(lib.rqf_chunked_prospective_forward(
                    _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1), _abi.ptr(z), _abi.ptr(out),
                    _abi.ptr(carries), _abi.ptr(scratch), B, T, F, _BTF_PATH, _abi.stream_of(z)),
                    "rqf_chunked_prospective_forward")
            _done(dev)
            dims = (B, T, F)
        ctx.save_for_backward(c1, t0, t1, z, carries)
        ctx.layout, ctx.fuse_act, ctx.dims = layout, bool(fuse_act), dims
        ctx.has_lag, ctx.path = delayed_u is not None, _BTF_PATH
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        gc1, gt0, gt1, gz, gzw = _tbptt_backward(ctx.saved_tensors, ctx.layout, ctx.dims,
                                                 grad_output, ctx.fuse_act, ctx.path)
        need = ctx.needs_input_grad
        if ctx.has_lag:
            gu, gd = gz, gzw
        else:
            gu, gd = gz.add_(gzw), None
        return (gc1 if need[0] else None, gt0 if need[1] else None, gt1 if need[2] else None,
                gu if need[3] else None, gd if (need[4] and gd is not None) else None, None, None)


def _tbptt_backward(saved, layout, dims, grad_output, fuse_act, path=0):
    """TBPTT(1) surrogate VJP kernel: returns (gc1, gtap0, gtap1, gz, gzw)."""
    c1, t0, t1, z, carries = saved
    dev = z.device
    gy = _c64(grad_output)
    lib = _abi.load()
    gz = torch.empty_like(z)
    gzw = torch.empty_like(z)
    gc1, gt0, gt1 = torch.empty_like(c1), torch.empty_like(t0), torch.empty_like(t1)
    d0, d1, d2 = dims
    if layout == "fbt":
        scratch = _scratch(lib.rqf_fbt_scratch_bytes(d0, d1, d2), dev)
    else:
        scratch = _scratch(lib.rqf_btf_scratch_bytes(d0, d1, d2), dev)
    with _timing.launch("rqf_tbptt1_two_tap_backward", d0 * d1 * d2, _nbytes(z, gy, gz, gzw)):
        _abi.check(lib.rqf_tbptt1_two_tap_backward(
            0 if layout == "btf" else 1, _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1),
            _abi.ptr(z), _abi.ptr(carries), _abi.ptr(gy), _abi.ptr(gz), _abi.ptr(gzw),
            _abi.ptr(gc1), _abi.ptr(gt0), _abi.ptr(gt1), _abi.ptr(scratch), d0, d1, d2,
            int(bool(fuse_act)), int(path), _abi.stream_of(gy)), "rqf_tbptt1_two_tap_backward")
    _done(dev)
    return gc1, gt0, gt1, gz, gzw


def _tbptt_backward_wsum(saved, grad_output, fuse_act):
    """The (F,B,T) TBPTT(1) surrogate VJP with the two tap cotangents also
    summed (rqf_fbt_tbptt1_backward_wsum): (gc1, gtap0, gtap1, gz, gz + gzw),
    for a lag source that is the same projection as z."""
    c1, t0, t1, z, carries = saved
    F, B, T = z.shape
    dev = z.device
    gy = _c64(grad_output)
    lib = _abi.load()
    gz = torch.empty_like(z)
    gsum = torch.empty_like(z)
    gc1, gt0, gt1 = torch.empty_like(c1), torch.empty_like(t0), torch.empty_like(t1)
    scratch = _scratch(lib.rqf_fbt_scratch_bytes(F, B, T), dev)
    with _timing.launch("rqf_tbptt1_two_tap_backward", F * B * T, _nbytes(z, gy, gz, gsum)):
        _abi.check(lib.rqf_fbt_tbptt1_backward_wsum(
            _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1), _abi.ptr(z), _abi.ptr(carries),
            _abi.ptr(gy), _abi.ptr(gz), _abi.ptr(gsum), _abi.ptr(gc1), _abi.ptr(gt0),
            _abi.ptr(gt1), _abi.ptr(scratch), F, B, T, int(bool(fuse_act)),
            _abi.stream_of(gy)), "rqf_fbt_tbptt1_backward_wsum")
    _done(dev)
    return gc1, gt0, gt1, gz, gsum


def tbptt1_two_tap_scan(u, C1, tap0, tap1, *, delayed_u=None, layout: str = "btf",
                        fuse_act: bool = False):
    """TBPTT(1) two-tap scan: forward value of the exact recurrence
    h[n] = C1 h[n-1] + tap0 u[n] + tap1 u[n-1]; gradients of the one-step
    rebuild with h[n-1] detached, as block.py:_scan_two_tap_with_grad_mode
    (:904-954) builds them in autograd.  ``delayed_u`` is the lag-tap source
    (e.g. W(x.detach())); ``layout`` "btf" (batch, time, filters) or "fbt"
    (filters, batch, time); ``fuse_act`` applies split-ReLU (fbt only)."""
    return _TBPTT1TwoTap.apply(C1, tap0, tap1, u, delayed_u, layout, fuse_act)


def tbptt1_scan(u, C1, C2):
    """TBPTT(1) single-tap scan x[n] = C1 x[n-1] + C2 u[n] with the surrogate
    gradients of block.py:_scan_with_grad_mode (:882-902)."""
    return _TBPTT1TwoTap.apply(C1, C2, torch.zeros_like(_c64(C2)), u, None, "btf", False)


# --------------------------------------------- scan.py dispatch mirrors
def _prepare(C1, C2, u, B):
    if not C1.is_complex():
        C1 = C1.to(torch.cfloat)
    if not C2.is_complex():
        C2 = C2.to(torch.cfloat)
    num_filters = C1.shape[0]
    if B is not None:
        # (C2 ⊙ B) @ u == C2 * (B @ u): project, then scan with gain C2.
        u_c = u.to(torch.cfloat) if not u.is_complex() else u
        u = torch.einsum("nf,btf->btn", B.to(torch.cfloat), u_c)
    elif u.shape[-1] == 1 and num_filters > 1:
        u = u.expand(-1, -1, num_filters).contiguous()
    return C1, C2, u


def sequential_scan(C1, C2, u, B=None):
    """CUDA branch of rqf_models/ops/scan.py:sequential_scan (:290-378):
    x[n] = C1 x[n-1] + C2 u[n] (or (C2 ⊙ B) @ u[n]); real u is scanned
    without materialising its zero imaginary part."""
    C1, C2, u = _prepare(C1, C2, u, B)
    return _triton_chunked_scan(C1, C2, u)


def parallel_scan(C1, C2, u, B=None):
    """CUDA branch of rqf_models/ops/scan.py:parallel_scan (:435-529); the
    reference routes it to the same chunked kernel (:504-509)."""
    return sequential_scan(C1, C2, u, B)


def _scan_abs(C1, C2, u) -> torch.Tensor:
    """|y| of y[t] = C1*y[t-1] + C2*u[t] on (B,T,F), written by the scan's own
    epilogue (no complex output, no saved context); float32 (B,T,F)."""
    dev = _require_cuda(C1, C2, u)
    real = not u.is_complex()
    uu = u.to(torch.float32).contiguous() if real else _c64(u)
    B, T, F = _shape3(uu, "u")
    c1, c2 = _coef(C1, F, "C1"), _coef(C2, F, "C2")
    lib = _abi.load()
    y = torch.empty((B, T, F), dtype=torch.float32, device=dev)
    scratch = _scratch(lib.rqf_btf_scratch_bytes(B, T, F), dev)
    with _timing.launch("rqf_chunked_scan_abs_forward", B * T * F, _nbytes(uu, y)):
        _abi.check(lib.rqf_chunked_scan_abs_forward(
            _abi.ptr(c1), _abi.ptr(c2), _abi.ptr(uu), int(real), _abi.ptr(y), _abi.ptr(scratch),
            B, T, F, _BTF_PATH, _abi.stream_of(uu)), "rqf_chunked_scan_abs_forward")
    _done(dev)
    return y


def _sequential_scan_forward_abs_raw_block_f(C1, C2, u):
    """Drop-in for rqf_models/ops/triton_scan_kernel.py:
    _sequential_scan_forward_abs_raw_block_f (:507): |scan| of complex u."""
    if not u.is_complex():
        raise ValueError("_sequential_scan_forward_abs_raw_block_f expects complex input")
    return _scan_abs(C1, C2, u)


def _sequential_scan_real_forward_abs_raw_block_f(C1, C2, u):
    """Drop-in for triton_scan_kernel.py:_sequential_scan_real_forward_abs_raw_block_f
    (:1531): |scan| of real u (float32)."""
    if u.is_complex():
        raise ValueError("_sequential_scan_real_forward_abs_raw_block_f expects real input")
    return _scan_abs(C1, C2, u)


def _triton_sequential_scan_b_matrix(C1, C2, u, B):
    """Drop-in for triton_scan_kernel.py:_triton_sequential_scan_b_matrix (:3375):
    x[n] = C1 x[n-1] + (C2 ⊙ B) @ u[n], B real (F, I), u (batch, time, I).  The
    input projection B @ u runs as one library GEMM over all (batch, time) rows
    and the recurrence on this backend's (B,T,F) scan with gain C2; autograd
    gives the reference's gradients (grad_B real: the real part of the
    complex one, as its backward takes)."""
    return sequential_scan(C1, C2, u, B)


def sequential_scan_abs(C1, C2, u, B=None):
    """|sequential_scan(...)| (rqf_models/ops/scan.py:381-432).  Without a B
    matrix and with no gradient required, the magnitude is written by the scan
    kernel's epilogue (half the output bytes, no separate abs pass), as the
    reference's fast path; otherwise the complex scan runs and .abs() follows."""
    needs_grad = torch.is_grad_enabled() and (
        u.requires_grad or getattr(C1, "requires_grad", False)
        or getattr(C2, "requires_grad", False) or (B is not None and B.requires_grad))
    if B is not None or needs_grad or not u.is_cuda:
        return sequential_scan(C1, C2, u, B).abs()
    C1, C2, u = _prepare(C1, C2, u, None)
    return _scan_abs(C1, C2, u)


# ------------------------------------------- multi-oscillator scans
def _mosc_pow2(n: int) -> bool:
    return 1 <= n <= 32 and (n & (n - 1)) == 0


def _cw_complex(c_weights: torch.Tensor) -> torch.Tensor:
    """The reference's real (scan_filters, 2) C-weights as complex64 (scan_filters,)."""
    return torch.view_as_complex(c_weights.detach().to(torch.float32).contiguous())


class _MultiOscScan(torch.autograd.Function):
    """out[t, f] = sum_k cw_{f n + k} x_{f n + k}[t] with x_s[t] = C1_s x_s[t-1] +
    C2_s u[t, s / n]: the fused multi-oscillator scan of
    triton_scan_kernel.py:_SequentialScanMultiOscFunction (:2413-2496), one
    lane per oscillator and the C-weight sum in the epilogue, so neither the
    repeated input nor the (B,T,F*n) states are materialised.  Saves C1, C2,
    the C-weights, u and one carry per 64-step sub-tile per oscillator."""

    @staticmethod
    def forward(ctx, C1, C2, u, c_weights, num_osc):
        dev = _require_cuda(C1, C2, u, c_weights)
        real = not u.is_complex()
        uu = u.to(torch.float32).contiguous() if real else _c64(u)
        B, T, F = _shape3(uu, "u")
        n = int(num_osc)
        c1, c2 = _coef(C1, F * n, "C1"), _coef(C2, F * n, "C2")
        cw = _coef(_cw_complex(c_weights), F * n, "c_weights")
        lib = _abi.load()
        out = torch.empty((B, T, F), dtype=torch.complex64, device=dev)
        carries = _carries(lib.rqf_multi_osc_carry_count(B, T, F, n), dev)
        scratch = _scratch(lib.rqf_multi_osc_scratch_bytes(B, T, F, n), dev)
        with _timing.launch("rqf_multi_osc_forward", B * T * F * n, _nbytes(uu, out)):
            _abi.check(lib.rqf_multi_osc_forward(
                _abi.ptr(c1), _abi.ptr(c2), _abi.ptr(cw), _abi.ptr(uu), int(real), _abi.ptr(out),
                0, _abi.ptr(carries), _abi.ptr(scratch), B, T, F, n, _abi.stream_of(uu)),
                "rqf_multi_osc_forward")
        _done(dev)
        ctx.save_for_backward(c1, c2, cw, uu, carries)
        ctx.real, ctx.n = real, n
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        c1, c2, cw, uu, carries = ctx.saved_tensors
        B, T, F = uu.shape
        n = ctx.n
        dev = uu.device
        gy = _c64(grad_output)
        lib = _abi.load()
        gu = torch.empty_like(uu)
        gc1, gc2, gcw = torch.empty_like(c1), torch.empty_like(c2), torch.empty_like(cw)
        scratch = _scratch(lib.rqf_multi_osc_scratch_bytes(B, T, F, n), dev)
        with _timing.launch("rqf_multi_osc_backward", B * T * F * n, _nbytes(uu, gy, gu)):
            _abi.check(lib.rqf_multi_osc_backward(
                _abi.ptr(c1), _abi.ptr(c2), _abi.ptr(cw), _abi.ptr(uu), int(ctx.real),
                _abi.ptr(carries), _abi.ptr(gy), _abi.ptr(gu), _abi.ptr(gc1), _abi.ptr(gc2),
                _abi.ptr(gcw), _abi.ptr(scratch), B, T, F, n, _abi.stream_of(gy)),
                "rqf_multi_osc_backward")
        _done(dev)
        need = ctx.needs_input_grad
        return (gc1 if need[0] else None, gc2 if need[1] else None, gu if need[2] else None,
                torch.view_as_real(gcw) if need[3] else None, None)


def _multi_osc_composed(C1, C2, u, c_weights, num_osc):
    """Any oscillator count: the scan over the repeated input, then the
    C-weighted sum (the reference's unfused path, block.py:_c_weighted_sum)."""
    B, T, F = u.shape
    y = sequential_scan(C1, C2, u.repeat_interleave(num_osc, dim=-1))
    cw = torch.view_as_complex(c_weights.to(torch.float32).contiguous())
    return (y.view(B, T, F, num_osc) * cw.view(F, num_osc)).sum(dim=-1)


def _triton_sequential_scan_multi_osc(C1, C2, u, c_weights, num_osc):
    """Drop-in for triton_scan_kernel.py:_triton_sequential_scan_multi_osc (:2499)."""
    if _mosc_pow2(int(num_osc)):
        return _MultiOscScan.apply(C1, C2, u, c_weights, int(num_osc))
    return _multi_osc_composed(C1, C2, u, c_weights, int(num_osc))


def _triton_sequential_scan_multi_osc_real(C1, C2, u, c_weights, num_osc):
    """Drop-in for triton_scan_kernel.py:_triton_sequential_scan_multi_osc_real
    (:3071): real u, scanned without materialising its imaginary part."""
    if u.is_complex():
        raise ValueError("_triton_sequential_scan_multi_osc_real expects real input")
    return _triton_sequential_scan_multi_osc(C1, C2, u, c_weights, num_osc)


def _triton_parallel_scan_multi_osc(C1, C2, u, c_weights, num_osc):
    """Drop-in for triton_scan_kernel.py:_triton_parallel_scan_multi_osc
    (:4106); the same values as the sequential form."""
    return _triton_sequential_scan_multi_osc(C1, C2, u, c_weights, num_osc)


def _multi_osc_abs(C1, C2, u, cw_complex, num_osc):
    n = int(num_osc)
    dev = _require_cuda(C1, C2, u)
    if not _mosc_pow2(n):
        return _multi_osc_composed(C1, C2, u, torch.view_as_real(cw_complex), n).abs()
    real = not u.is_complex()
    uu = u.to(torch.float32).contiguous() if real else _c64(u)
    B, T, F = _shape3(uu, "u")
    c1, c2 = _coef(C1, F * n, "C1"), _coef(C2, F * n, "C2")
    cw = _coef(cw_complex, F * n, "c_weights")
    lib = _abi.load()
    out = torch.empty((B, T, F), dtype=torch.float32, device=dev)
    scratch = _scratch(lib.rqf_multi_osc_scratch_bytes(B, T, F, n), dev)
    with _timing.launch("rqf_multi_osc_forward", B * T * F * n, _nbytes(uu, out)):
        _abi.check(lib.rqf_multi_osc_forward(
            _abi.ptr(c1), _abi.ptr(c2), _abi.ptr(cw), _abi.ptr(uu), int(real), _abi.ptr(out), 1,
            None, _abi.ptr(scratch), B, T, F, n, _abi.stream_of(uu)), "rqf_multi_osc_forward")
    _done(dev)
    return out


def _sequential_scan_multi_osc_forward_abs_raw(C1, C2, u, cw_real, cw_imag, num_osc):
    """Drop-in for triton_scan_kernel.py:_sequential_scan_multi_osc_forward_abs_raw
    (:2019): |C-weighted multi-oscillator scan|, no autograd."""
    cw = torch.complex(cw_real.to(torch.float32), cw_imag.to(torch.float32)).contiguous()
    return _multi_osc_abs(C1, C2, u, cw, num_osc)


def _sequential_scan_multi_osc_real_forward_abs_raw(C1, C2, u, c_weights, num_osc):
    """Drop-in for triton_scan_kernel.py:_sequential_scan_multi_osc_real_forward_abs_raw
    (:2688): real u, |output|, no autograd."""
    if u.is_complex():
        raise ValueError("_sequential_scan_multi_osc_real_forward_abs_raw expects real input")
    return _multi_osc_abs(C1, C2, u, _cw_complex(c_weights), num_osc)


# ------------------------------------------------------ selective scan
_SEL_FIELDS = ("gamma_logits", "warp_logits", "write_logits", "bias", "theta", "groups",
               "minimum", "span", "step", "horizon", "theta_minimum", "theta_maximum")


def _sel_options(opt) -> "_abi.SelectiveOptions":
    o = _abi.SelectiveOptions()
    (o.has_gamma, o.has_warp, o.has_write, o.log_shift) = (int(bool(v)) for v in opt[:4])
    o.gamma_scale, o.warp_scale = float(opt[4]), float(opt[5])
    o.prospective, o.gamma_horizon, o.write_sigmoid = (int(bool(v)) for v in opt[6:9])
    o.write_max, o.write_bias = float(opt[9]), float(opt[10])
    o.bound_warp = int(bool(opt[11]))
    return o


def _sel_tensors(inputs, device, logit_dtype=torch.float32):
    """Contiguous fp32 / int64 device tensors of a SelectiveScanInputs-like
    13-tuple (rqf_models/ops/selective_scan.py:10-23) and its C struct; the
    three logit tensors in `logit_dtype` (bf16 for the bf16 storage mode)."""
    opt = inputs[12]
    t = {}
    for i, name in enumerate(_SEL_FIELDS):
        v = inputs[i]
        if v is None or (name.endswith("_logits") and v.numel() == 0):
            t[name] = None
        elif name == "groups":
            t[name] = v.to(device=device, dtype=torch.int64).contiguous()
        elif name.endswith("_logits"):
            t[name] = v.to(device=device, dtype=logit_dtype).contiguous()
        else:
            t[name] = v.to(device=device, dtype=torch.float32).contiguous()
    if not opt[0]:
        t["gamma_logits"] = None
    if not opt[1]:
        t["warp_logits"], t["groups"] = None, None
    if not opt[2]:
        t["write_logits"] = None
    s = _abi.SelectiveInputs()
    for name in _SEL_FIELDS:
        setattr(s, name, None if t[name] is None else t[name].data_ptr())
    s.num_groups = int(t["warp_logits"].shape[0]) if t["warp_logits"] is not None else 0
    return t, s, _sel_options(opt)


def selective_forward(z, inputs, activate, write_raw, chunk=None):
    """Fused input-dependent ZOH scan — drop-in for
    rqf_models/ops/selective_scan_kernel.py:selective_forward (:491).
    Returns (raw | None, act | None, entries); `entries` holds this backend's
    per-tile entry states (opaque to the caller, passed back to
    selective_backward); `chunk` is accepted and unused (fixed tiles)."""
    dev = _require_cuda(z)
    if not activate and not write_raw:
        raise ValueError("selective scan requires at least one output")
    zz = _c64(z)
    F, B, T = _shape3(zz, "z")
    keep, sin, sopt = _sel_tensors(inputs, dev)
    lib = _abi.load()
    raw = torch.empty_like(zz) if write_raw else None
    act = torch.empty_like(zz) if activate else None
    entries = torch.empty((F * B, max(int(lib.rqf_selective_num_tiles(T)), 1)),
                          dtype=torch.complex64, device=dev)
    nb = _nbytes(zz, keep["gamma_logits"], keep["warp_logits"], keep["write_logits"], raw, act)
    with _timing.launch("rqf_selective_forward", F * B * T, nb):
        _abi.check(lib.rqf_selective_forward(
            _abi.ptr(zz), ctypes.byref(sin), ctypes.byref(sopt), _abi.ptr(raw), _abi.ptr(act),
            _abi.ptr(entries), F, B, T, _abi.stream_of(zz)), "rqf_selective_forward")
    _done(dev)
    del keep
    return raw, act, entries


def selective_backward(z, inputs, entries, gy, gx, activate, truncated, chunk=None):
    """Fused backward — drop-in for selective_scan_kernel.py:selective_backward
    (:517).  Returns (dz, dzw, dg, dd_group, dw, dbias, dtheta); dzw is dz
    unless truncated (TBPTT(1)), as in the reference."""
    dev = _require_cuda(z)
    zz = _c64(z)
    F, B, T = _shape3(zz, "z")
    keep, sin, sopt = _sel_tensors(inputs, dev)
    opt = inputs[12]
    lib = _abi.load()
    gyc = None if gy is None else _c64(gy)
    gxc = None if gx is None else _c64(gx)
    dz = torch.empty_like(zz)
    dzw = torch.empty_like(zz) if truncated else dz
    dg = torch.empty_like(keep["gamma_logits"]) if opt[0] else None
    dd = torch.empty_like(keep["warp_logits"]) if opt[1] else None
    dw = torch.empty_like(keep["write_logits"]) if opt[2] else None
    dbias = torch.empty(F, dtype=torch.float32, device=dev)
    dtheta = torch.empty(F, dtype=torch.float32, device=dev)
    scratch = _scratch(lib.rqf_selective_scratch_bytes(F, B, T, int(bool(opt[1]))), dev)
    nb = _nbytes(zz, keep["gamma_logits"], keep["warp_logits"], keep["write_logits"], gyc, gxc,
                 dz, dzw if truncated else None, dg, dd, dw)
    with _timing.launch("rqf_selective_backward", F * B * T, nb):
        _abi.check(lib.rqf_selective_backward(
            _abi.ptr(zz), ctypes.byref(sin), ctypes.byref(sopt), _abi.ptr(entries),
            _abi.ptr(gyc), _abi.ptr(gxc), int(bool(truncated)), _abi.ptr(dz),
            _abi.ptr(dzw if truncated else None), _abi.ptr(dg), _abi.ptr(dd), _abi.ptr(dw),
            _abi.ptr(dbias), _abi.ptr(dtheta), _abi.ptr(scratch), F, B, T, _abi.stream_of(zz)),
            "rqf_selective_backward")
    _done(dev)
    del keep
    return dz, dzw, dg, dd, dw, dbias, dtheta


def selective_forward_bf16(z, inputs, activate, write_raw):
    """The bf16 storage mode of selective_forward (rqf_selective_forward_bf16;
    no reference counterpart: the selective benchmark configuration's "bf16
    activations, fp32 state").  The logits of `inputs` are read as bf16 (converted if given in
    another dtype); raw and act are returned as bf16 (F, B, T, 2) [Re, Im]
    pairs.  z, the carries and all arithmetic stay fp32."""
    dev = _require_cuda(z)
    if not activate and not write_raw:
        raise ValueError("selective scan requires at least one output")
    zz = _c64(z)
    F, B, T = _shape3(zz, "z")
    keep, sin, sopt = _sel_tensors(inputs, dev, torch.bfloat16)
    lib = _abi.load()
    raw = torch.empty((F, B, T, 2), dtype=torch.bfloat16, device=dev) if write_raw else None
    act = torch.empty((F, B, T, 2), dtype=torch.bfloat16, device=dev) if activate else None
    entries = torch.empty((F * B, max(int(lib.rqf_selective_num_tiles(T)), 1)),
                          dtype=torch.complex64, device=dev)
    nb = _nbytes(zz, keep["gamma_logits"], keep["warp_logits"], keep["write_logits"], raw, act)
    with _timing.launch("rqf_selective_forward_bf16", F * B * T, nb):
        _abi.check(lib.rqf_selective_forward_bf16(
            _abi.ptr(zz), ctypes.byref(sin), ctypes.byref(sopt), _abi.ptr(raw), _abi.ptr(act),
            _abi.ptr(entries), F, B, T, _abi.stream_of(zz)), "rqf_selective_forward_bf16")
    _done(dev)
    del keep
    return raw, act, entries


def selective_backward_bf16(z, inputs, entries, gy, gx, activate, truncated):
    """The bf16 storage mode of selective_backward: the logit cotangents
    (dg, dd_group, dw) come back in bf16; dz, dzw, dbias and dtheta in fp32 as
    in selective_backward; gy / gx are complex64 cotangents."""
    dev = _require_cuda(z)
    zz = _c64(z)
    F, B, T = _shape3(zz, "z")
    keep, sin, sopt = _sel_tensors(inputs, dev, torch.bfloat16)
    opt = inputs[12]
    lib = _abi.load()
    gyc = None if gy is None else _c64(gy)
    gxc = None if gx is None else _c64(gx)
    dz = torch.empty_like(zz)
    dzw = torch.empty_like(zz) if truncated else dz
    dg = torch.empty_like(keep["gamma_logits"]) if opt[0] else None
    dd = torch.empty_like(keep["warp_logits"]) if opt[1] else None
    dw = torch.empty_like(keep["write_logits"]) if opt[2] else None
    dbias = torch.empty(F, dtype=torch.float32, device=dev)
    dtheta = torch.empty(F, dtype=torch.float32, device=dev)
    scratch = _scratch(lib.rqf_selective_scratch_bytes(F, B, T, int(bool(opt[1]))), dev)
    nb = _nbytes(zz, keep["gamma_logits"], keep["warp_logits"], keep["write_logits"], gyc, gxc,
                 dz, dzw if truncated else None, dg, dd, dw)
    with _timing.launch("rqf_selective_backward_bf16", F * B * T, nb):
        _abi.check(lib.rqf_selective_backward_bf16(
            _abi.ptr(zz), ctypes.byref(sin), ctypes.byref(sopt), _abi.ptr(entries),
            _abi.ptr(gyc), _abi.ptr(gxc), int(bool(truncated)), _abi.ptr(dz),
            _abi.ptr(dzw if truncated else None), _abi.ptr(dg), _abi.ptr(dd), _abi.ptr(dw),
            _abi.ptr(dbias), _abi.ptr(dtheta), _abi.ptr(scratch), F, B, T, _abi.stream_of(zz)),
            "rqf_selective_backward_bf16")
    _done(dev)
    del keep
    return dz, dzw, dg, dd, dw, dbias, dtheta


class _SelectiveLayerScan(torch.autograd.Function):
    """Owns the drive GEMM z = W @ x so the TBPTT(1) lag cotangent reaches W
    only (rqf_models/ops/selective_scan.py:_SelectiveLayerScan :107-170).
    The drive GEMM and its two cotangent GEMMs run on the split-TF32
    tensor-core projections (the reference: fp32 cuBLAS complex GEMMs)."""

    @staticmethod
    def forward(ctx, x, weight, *args):
        *tensors, options, truncated, activate, write_raw, chunk = args
        inputs = tuple(tensors) + (options,)
        z = projection(weight, x)
        raw, act, entries = selective_forward(z, inputs, activate, write_raw, chunk)
        ctx.save_for_backward(x, weight, z, entries, *[t for t in tensors if t is not None])
        ctx.none_mask = [t is None for t in tensors]
        ctx.options, ctx.truncated = options, truncated
        ctx.activate, ctx.chunk = activate, chunk
        ctx.set_materialize_grads(False)
        return raw, act

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_raw, grad_act):
        x, weight, z, entries, *present = ctx.saved_tensors
        it = iter(present)
        tensors = [None if none else next(it) for none in ctx.none_mask]
        inputs = tuple(tensors) + (ctx.options,)
        dx_drive, dw_drive, dg, dd, dw, dbias, dtheta = selective_backward(
            z, inputs, entries, grad_raw, grad_act, ctx.activate, ctx.truncated, ctx.chunk)
        need = ctx.needs_input_grad
        dx = projection(weight, dx_drive, conj_transpose=True) if need[0] else None
        dweight = projection_weight_grad(dw_drive, x) if need[1] else None
        grads = (dx, dweight, dg, dd, dw, dbias, dtheta) + (None,) * 12
        return tuple(g if need else None for g, need in zip(grads, ctx.needs_input_grad))


def selective_layer_scan(x, weight, inputs, *, truncated: bool = False, activate: bool = True,
                         write_raw: bool = True, use_kernel: bool = True, chunk=None):
    """Complex (I,B,T) selective layer on the B200 kernels — mirrors
    rqf_models/ops/selective_scan.py:selective_layer_scan (:173) for CUDA
    complex64 inputs (the reference's kernel-eligible case).  Returns
    (raw | None, act | None)."""
    if not activate and not write_raw:
        raise ValueError("selective scan requires at least one output")
    if not use_kernel:
        raise ValueError("use_kernel=False selects the reference's PyTorch path, which this "
                         "backend does not provide")
    if chunk is not None and (chunk < 1 or chunk & (chunk - 1)):
        raise ValueError("chunk must be a positive power of two")
    _require_cuda(x, weight)
    tensors = [v.contiguous() if isinstance(v, torch.Tensor) else v for v in inputs[:-1]]
    return _SelectiveLayerScan.apply(x.contiguous(), weight, *tensors, inputs[-1], truncated,
                                     activate, write_raw, chunk)


# ------------------------------------------------ complex projection GEMM
def projection(W: torch.Tensor, x: torch.Tensor, conj_transpose: bool = False,
               acc: torch.Tensor | None = None, inplace: bool = False) -> torch.Tensor:
    """out = op(W) @ x (+ acc) with x (K, ...) complex64, the trailing dims
    flattened to N: the Pure RQF block projection z = W h
    (rqf_models/backbones/rqf/pure.py:223, torch.matmul on the
    (d_model, batch*time) view) when op(W) = W with W (M, K), and its input
    cotangent W^H gz when ``conj_transpose`` (W is then (K, M)).  ``acc``
    (M, ...) is added in the epilogue (the skip cotangent); with ``inplace``
    the result is accumulated into ``acc`` itself when it is a contiguous
    complex64 tensor, by TMA reduce-adds (the epilogue reads no acc), and
    ``acc`` is returned.

    Runs the split-TF32 tcgen05 GEMM of rqf_projection (fp32-comparable;
    not differentiable itself — the callers own the autograd).  An odd N,
    which the kernel's TMA row pitch cannot express, runs torch.matmul on
    the GPU instead."""
    dev = _require_cuda(W, x, acc)
    w = _c64(W)
    xx = _c64(x)
    if w.dim() != 2 or xx.dim() < 1:
        raise ValueError("projection expects a 2-D W and an x of at least 1 dimension")
    K = int(xx.shape[0])
    M = int(w.shape[1] if conj_transpose else w.shape[0])
    if int(w.shape[0] if conj_transpose else w.shape[1]) != K:
        raise ValueError(f"W {tuple(w.shape)} does not match x {tuple(xx.shape)}"
                         f"{' (conj_transpose)' if conj_transpose else ''}")
    tail = tuple(xx.shape[1:])
    N = 1
    for d in tail:
        N *= int(d)
    out_shape = (M,) + tail
    a = None
    if acc is not None:
        a = _c64(acc)
        if tuple(a.shape) != out_shape:
            raise ValueError(f"acc must have shape {out_shape}, got {tuple(a.shape)}")
    if N % 2 == 1:
        opw = w.mH if conj_transpose else w
        out = (opw @ xx.reshape(K, N)).reshape(out_shape)
        return out if a is None else out.add_(a)
    lib = _abi.load()
    if inplace and a is not None and a is acc:  # acc already contiguous complex64
        out = a
    else:
        out = torch.empty(out_shape, dtype=torch.complex64, device=dev)
    ws = _scratch(lib.rqf_projection_workspace_bytes(M, K), dev)
    with _timing.launch("rqf_projection", M * N, _nbytes(xx, out, a), 8 * M * K * N):
        _abi.check(lib.rqf_projection(
            _abi.ptr(w), _abi.ptr(xx), _abi.ptr(a), _abi.ptr(out), M, K, N,
            int(bool(conj_transpose)), _abi.ptr(ws), _abi.stream_of(xx)), "rqf_projection")
    _done(dev)
    return out


def projection_weight_grad(gz: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """gW = gz @ x^H over the flattened trailing dims: the weight cotangent of
    the block projection z = W x (pure.py:223) given gz = dL/dz, with gz
    (M, ...) and x (K, ...) complex64.  Split-TF32 tcgen05 GEMM with a split
    reduction over samples summed in a fixed order
    (rqf_projection_weight_grad); an odd sample count runs torch.matmul."""
    dev = _require_cuda(gz, x)
    g = _c64(gz)
    xx = _c64(x)
    M, K = int(g.shape[0]), int(xx.shape[0])
    if tuple(g.shape[1:]) != tuple(xx.shape[1:]):
        raise ValueError(f"gz {tuple(g.shape)} and x {tuple(xx.shape)} differ in trailing dims")
    N = g.numel() // M if M else 0
    if N % 2 == 1:
        return g.reshape(M, N) @ xx.reshape(K, N).mH
    lib = _abi.load()
    gw = torch.empty((M, K), dtype=torch.complex64, device=dev)
    ws = _scratch(lib.rqf_projection_weight_grad_workspace_bytes(M, K, N), dev)
    with _timing.launch("rqf_projection_weight_grad", M * N, _nbytes(g, xx, gw), 8 * M * K * N):
        _abi.check(lib.rqf_projection_weight_grad(
            _abi.ptr(g), _abi.ptr(xx), _abi.ptr(gw), M, K, N, _abi.ptr(ws),
            _abi.stream_of(g)), "rqf_projection_weight_grad")
    _done(dev)
    return gw


# ------------------------------------------------ low-rank first block
def lowrank_drive(u: torch.Tensor, x: torch.Tensor, beta: torch.Tensor | None = None,
                  w_in: torch.Tensor | None = None, b_in: torch.Tensor | None = None):
    """The first block's drive over a low-rank input projection
    (pure.py:_forward_fbt_stack :522-534): z = u @ x (+ beta[:, None]) as
    complex64 (F, N), and, when w_in is given, h = (w_in @ x (+ b_in)) as
    complex64 with zero imaginary part, in one pass (rqf_lowrank_drive).
    u (F, I) complex, x (I, N) real with I <= 4 and N even."""
    dev = _require_cuda(u, x)
    uu = _c64(u)
    xx = x.detach().to(torch.float32).contiguous()
    F, I = int(uu.shape[0]), int(uu.shape[1])
    N = int(xx.shape[1])
    if xx.shape[0] != I:
        raise ValueError(f"u {tuple(uu.shape)} and x {tuple(xx.shape)} disagree on the rank")
    bb = _c64(beta) if beta is not None else None
    ww = w_in.detach().to(torch.float32).contiguous() if w_in is not None else None
    bi = b_in.detach().to(torch.float32).contiguous() if (w_in is not None and b_in is not None) else None
    z = torch.empty((F, N), dtype=torch.complex64, device=dev)
    h = torch.empty((F, N), dtype=torch.complex64, device=dev) if ww is not None else None
    lib = _abi.load()
    with _timing.launch("rqf_lowrank_drive", F * N, _nbytes(xx, z) + (h.numel() * 8 if h is not None else 0)):
        _abi.check(lib.rqf_lowrank_drive(
            _abi.ptr(uu), _abi.ptr(bb), _abi.ptr(ww), _abi.ptr(bi), _abi.ptr(xx), _abi.ptr(z),
            _abi.ptr(h), F, N, I, _abi.stream_of(z)), "rqf_lowrank_drive")
    _done(dev)
    return z, h


def rank1_supported(F: int, B: int, T: int) -> bool:
    """Whether the rank-1 first-block kernels take an (F, B, T) block on the
    current device (enough rows for the persistent row kernels, T a multiple
    of 4)."""
    return _abi.load().rqf_fbt_rank1_supported(int(F), int(B), int(T)) == 1


def rank1_block_forward(u, beta, w, bb, x, C1, tap0, tap1, fuse_act: bool):
    """The first Pure RQF block over a rank-1 input in one launch
    (rqf_fbt_rank1_forward): z = u x + beta and, when w is given, the skip
    h0 = w x + bb made inside the (F,B,T) row scan from x (B, T) float32;
    returns act(y) (+ h0) as complex64 (F, B, T) and the saved context
    (c1, tap0, tap1, u, beta, x, carries) for rank1_block_backward.  u,
    beta (F,) complex; w, bb (F,) real (beta, bb may be None)."""
    dev = _require_cuda(u, x, C1)
    xx = x.detach().to(torch.float32).contiguous()
    B, T = (int(d) for d in xx.shape)
    uu = _c64(u)
    F = int(uu.shape[0])
    c1, t0, t1 = _coef(C1, F, "C1"), _coef(tap0, F, "tap0"), _coef(tap1, F, "tap1")
    be = _c64(beta) if beta is not None else None
    ww = w.detach().to(torch.float32).contiguous() if w is not None else None
    bbv = bb.detach().to(torch.float32).contiguous() if (w is not None and bb is not None) else None
    lib = _abi.load()
    out = torch.empty((F, B, T), dtype=torch.complex64, device=dev)
    carries = _carries(lib.rqf_fbt_carry_count(F, B, T), dev)
    with _timing.launch("rqf_fbt_rank1_forward", F * B * T, _nbytes(xx, out)):
        _abi.check(lib.rqf_fbt_rank1_forward(
            _abi.ptr(uu), _abi.ptr(be), _abi.ptr(ww), _abi.ptr(bbv), _abi.ptr(xx), _abi.ptr(c1),
            _abi.ptr(t0), _abi.ptr(t1), _abi.ptr(out), _abi.ptr(carries), F, B, T,
            int(bool(fuse_act)), _abi.stream_of(xx)), "rqf_fbt_rank1_forward")
    _done(dev)
    return out, (c1, t0, t1, uu, be, xx, carries)


def rank1_block_backward(saved, grad_output, fuse_act: bool, with_sum: bool, skip: bool):
    """The rank-1 first block's backward (rqf_fbt_rank1_backward): the scan
    VJP of grad_output replayed from the saved context with z made from x,
    reduced to (gc1, gtap0, gtap1, G, Gs) where G = [sum gz x (, sum gz)] and
    Gs = [sum g x (, sum g)] over (b, t) are complex64 (F, 1 + with_sum) —
    what rowdot(gz, x, with_sum) and rowdot(g, x, with_sum) return — and Gs is
    None unless ``skip``.  grad_z itself is never formed."""
    c1, t0, t1, uu, be, xx, carries = saved
    F = int(uu.shape[0])
    B, T = (int(d) for d in xx.shape)
    dev = xx.device
    gy = _c64(grad_output)
    lib = _abi.load()
    gc1, gt0, gt1 = torch.empty_like(c1), torch.empty_like(t0), torch.empty_like(t1)
    G = torch.empty((F, 2), dtype=torch.complex64, device=dev)
    Gs = torch.empty((F, 2), dtype=torch.complex64, device=dev) if skip else None
    scratch = _scratch(lib.rqf_fbt_rank1_scratch_bytes(F, B, T), dev)
    with _timing.launch("rqf_fbt_rank1_backward", F * B * T, _nbytes(xx, gy)):
        _abi.check(lib.rqf_fbt_rank1_backward(
            _abi.ptr(uu), _abi.ptr(be), _abi.ptr(xx), _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1),
            _abi.ptr(carries), _abi.ptr(gy), _abi.ptr(G), _abi.ptr(Gs), _abi.ptr(gc1),
            _abi.ptr(gt0), _abi.ptr(gt1), _abi.ptr(scratch), F, B, T, int(bool(fuse_act)),
            int(bool(with_sum)), _abi.stream_of(gy)), "rqf_fbt_rank1_backward")
    _done(dev)
    n = 2 if with_sum else 1
    return gc1, gt0, gt1, G[:, :n], (Gs[:, :n] if Gs is not None else None)


def rank1_tbptt_backward(saved, grad_output, fuse_act: bool, with_sum: bool, skip: bool):
    """The TBPTT(1) surrogate backward of the rank-1 first block
    (rqf_fbt_rank1_tbptt_backward), from rank1_block_forward's saved context:
    (gc1, gtap0, gtap1, G, Gw, Gs) with G = [sum gz x (, sum gz)], Gw the same
    sums of gz + gzw (what _tbptt_backward_wsum's second output gives
    rowdot), Gs = [sum g x (, sum g)] or None unless ``skip``; complex64
    (F, 1 + with_sum).  Neither grad_z nor the lag cotangent is formed."""
    c1, t0, t1, uu, be, xx, carries = saved
    F = int(uu.shape[0])
    B, T = (int(d) for d in xx.shape)
    dev = xx.device
    gy = _c64(grad_output)
    lib = _abi.load()
    gc1, gt0, gt1 = torch.empty_like(c1), torch.empty_like(t0), torch.empty_like(t1)
    G = torch.empty((F, 2), dtype=torch.complex64, device=dev)
    Gw = torch.empty((F, 2), dtype=torch.complex64, device=dev)
    Gs = torch.empty((F, 2), dtype=torch.complex64, device=dev) if skip else None
    scratch = _scratch(lib.rqf_fbt_rank1_scratch_bytes(F, B, T), dev)
    with _timing.launch("rqf_fbt_rank1_tbptt_backward", F * B * T, _nbytes(xx, gy)):
        _abi.check(lib.rqf_fbt_rank1_tbptt_backward(
            _abi.ptr(uu), _abi.ptr(be), _abi.ptr(xx), _abi.ptr(c1), _abi.ptr(t0), _abi.ptr(t1),
            _abi.ptr(carries), _abi.ptr(gy), _abi.ptr(G), _abi.ptr(Gw), _abi.ptr(Gs),
            _abi.ptr(gc1), _abi.ptr(gt0), _abi.ptr(gt1), _abi.ptr(scratch), F, B, T,
            int(bool(fuse_act)), int(bool(with_sum)), _abi.stream_of(gy)),
            "rqf_fbt_rank1_tbptt_backward")
    _done(dev)
    n = 2 if with_sum else 1
    return gc1, gt0, gt1, G[:, :n], Gw[:, :n], (Gs[:, :n] if Gs is not None else None)


def rowdot(a: torch.Tensor, x: torch.Tensor | None, with_sum: bool = False) -> torch.Tensor:
    """out[:, j] = a @ x[j] for the real rows of x (I <= 4), then the row sums
    of a when with_sum: complex64 (F, I + with_sum), over the flattened
    trailing dims of a complex (F, ...).  Fixed-order reduction (rqf_rowdot)."""
    dev = _require_cuda(a)
    aa = _c64(a)
    F = int(aa.shape[0])
    N = aa.numel() // F if F else 0
    xx = x.detach().to(torch.float32).contiguous() if x is not None else None
    I = int(xx.shape[0]) if xx is not None else 0
    if xx is not None and xx.numel() != I * N:
        raise ValueError(f"x {tuple(xx.shape)} does not match {N} samples")
    J = I + int(bool(with_sum))
    out = torch.empty((F, J), dtype=torch.complex64, device=dev)
    lib = _abi.load()
    ws = _scratch(lib.rqf_rowdot_workspace_bytes(F, N, I, int(bool(with_sum))), dev)
    with _timing.launch("rqf_rowdot", F * N, _nbytes(aa) + (_nbytes(xx) if xx is not None else 0)):
        _abi.check(lib.rqf_rowdot(
            _abi.ptr(aa), _abi.ptr(xx), _abi.ptr(out), _abi.ptr(ws), F, N, I, int(bool(with_sum)),
            _abi.stream_of(aa)), "rqf_rowdot")
    _done(dev)
    return out


# ------------------------------------------------ mean-pooled readout hidden layer
class _PerStepCE(torch.autograd.Function):
    """The per-timestep cross entropy (train.py:per_step_cross_entropy
    :663-674) on logits in the readout GEMM's (classes, batch*time) layout:
    rqf_per_step_cross_entropy forward, rqf_per_step_cross_entropy_backward
    for the logits' gradient.  Labels and smoothing take no gradient."""

    @staticmethod
    def forward(ctx, logits, labels, batch, time, label_smoothing):
        ll = logits.detach().contiguous()
        yy = labels.detach().to(torch.int64).contiguous()
        C = int(ll.shape[0])
        dev = _require_cuda(ll, yy)
        lib = _abi.load()
        loss = torch.empty((), dtype=torch.float32, device=dev)
        scratch = _scratch(lib.rqf_per_step_cross_entropy_scratch_bytes(batch, time), dev)
        with _timing.launch("rqf_per_step_cross_entropy", batch * time, _nbytes(ll)):
            _abi.check(lib.rqf_per_step_cross_entropy(
                _abi.ptr(ll), _abi.ptr(yy), _abi.ptr(loss), _abi.ptr(scratch), C, batch, time,
                float(label_smoothing), _abi.stream_of(ll)), "rqf_per_step_cross_entropy")
        _done(dev)
        ctx.save_for_backward(ll, yy)
        ctx.dims = (batch, time, float(label_smoothing))
        return loss

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_loss):
        ll, yy = ctx.saved_tensors
        batch, time, eps = ctx.dims
        g = grad_loss.detach().to(torch.float32).contiguous()
        gl = torch.empty_like(ll)
        lib = _abi.load()
        with _timing.launch("rqf_per_step_cross_entropy_backward", batch * time,
                            2 * _nbytes(ll)):
            _abi.check(lib.rqf_per_step_cross_entropy_backward(
                _abi.ptr(ll), _abi.ptr(yy), _abi.ptr(g), _abi.ptr(gl), int(ll.shape[0]), batch,
                time, eps, _abi.stream_of(ll)), "rqf_per_step_cross_entropy_backward")
        _done(ll.device)
        return gl, None, None, None, None


def per_step_cross_entropy(logits_cn: torch.Tensor, labels: torch.Tensor, batch: int, time: int,
                           label_smoothing: float = 0.0) -> torch.Tensor:
    """Mean label-smoothed cross entropy of per-timestep logits given as
    float32 (classes, batch*time), sample b*time + t, labels (batch,) int64:
    the value of train.py:per_step_cross_entropy on the (batch, time,
    classes) view of the same logits, in one pass and without the view."""
    if logits_cn.dtype != torch.float32 or logits_cn.dim() != 2 or \
            logits_cn.shape[1] != batch * time or labels.shape != (batch,):
        raise ValueError(f"logits {tuple(logits_cn.shape)} {logits_cn.dtype}, labels "
                         f"{tuple(labels.shape)} do not match batch={batch}, time={time}")
    return _PerStepCE.apply(logits_cn, labels, int(batch), int(time), float(label_smoothing))


def readout_relu_pool(z: torch.Tensor, bias: torch.Tensor | None):
    """pooled = mean_t relu(z + bias[:, None, None]) as float32 (H, B), and
    the ReLU mask as int32 words (H, B, ceil(T/32)), bit t % 32 of word t / 32,
    from the float32 (H, B, T) pre-activation z = Re(V h) in one pass
    (rqf_readout_relu_pool; train.py:ComplexReadoutClassifier :74-136 with
    mean pooling)."""
    dev = _require_cuda(z)
    zz = z.detach().to(torch.float32).contiguous()
    H, B, T = (int(d) for d in zz.shape)
    words = (T + 31) // 32
    mask = torch.empty((H, B, words), dtype=torch.int32, device=dev)
    pooled = torch.empty((H, B), dtype=torch.float32, device=dev)
    bb = bias.detach().to(torch.float32).contiguous() if bias is not None else None
    lib = _abi.load()
    with _timing.launch("rqf_readout_relu_pool", H * B * T, _nbytes(zz, mask)):
        _abi.check(lib.rqf_readout_relu_pool(_abi.ptr(zz), _abi.ptr(bb), _abi.ptr(mask),
                                             _abi.ptr(pooled), H, B, T, _abi.stream_of(zz)),
                   "rqf_readout_relu_pool")
    _done(dev)
    return pooled, mask


def readout_relu_pool_backward(mask: torch.Tensor, scale: torch.Tensor, time: int):
    """g = mask * scale[:, :, None] as float32 (H, B, T) (the real cotangent
    of the readout's hidden layer) and the set-bit count per (h, b) row
    (rqf_readout_relu_pool_backward)."""
    dev = _require_cuda(mask, scale)
    mask = mask.contiguous()
    H, B, words = (int(d) for d in mask.shape)
    if words != (time + 31) // 32:
        raise ValueError(f"mask of {words} words does not cover {time} steps")
    ss = scale.detach().to(torch.float32).contiguous()
    gc = torch.empty((H, B, time), dtype=torch.float32, device=dev)
    counts = torch.empty((H, B), dtype=torch.float32, device=dev)
    lib = _abi.load()
    with _timing.launch("rqf_readout_relu_pool_backward", H * B * time, _nbytes(mask, gc)):
        _abi.check(lib.rqf_readout_relu_pool_backward(
            _abi.ptr(mask), _abi.ptr(ss), _abi.ptr(gc), _abi.ptr(counts), H, B, time,
            _abi.stream_of(gc)), "rqf_readout_relu_pool_backward")
    _done(dev)
    return gc, counts


def readout_bias_relu(z: torch.Tensor, bias: torch.Tensor | None):
    """In place on z (float32, H x B x T): z = relu(z + bias[:, None, None])
    (rqf_readout_bias_relu), the per-step hidden layer's activation; returns
    (z, mask) with the ReLU decisions as bits (uint32 words, the layout of
    readout_relu_pool)."""
    dev = _require_cuda(z)
    if z.dtype != torch.float32 or z.dim() != 3 or not z.is_contiguous():
        raise ValueError("z must be a contiguous float32 (H, B, T) tensor")
    H, B, T = (int(d) for d in z.shape)
    bb = bias.detach().to(torch.float32).contiguous() if bias is not None else None
    mask = torch.empty((H * B * ((T + 31) // 32),), dtype=torch.int32, device=dev)
    lib = _abi.load()
    with _timing.launch("rqf_readout_bias_relu", H * B * T, 2 * _nbytes(z)):
        _abi.check(lib.rqf_readout_bias_relu(_abi.ptr(z), _abi.ptr(bb), _abi.ptr(mask), H, B, T,
                                             _abi.stream_of(z)), "rqf_readout_bias_relu")
    _done(dev)
    return z, mask


def readout_bias_relu_backward(gy: torch.Tensor, mask: torch.Tensor):
    """(g, rowsum): g = gy where the ReLU passed, else 0 (float32, H x B x T),
    and rowsum (H, B) its sums over time (rqf_readout_bias_relu_backward)."""
    gg = gy.detach().to(torch.float32).contiguous()
    dev = _require_cuda(gg, mask)
    H, B, T = (int(d) for d in gg.shape)
    g = torch.empty_like(gg)
    rowsum = torch.empty((H, B), dtype=torch.float32, device=dev)
    lib = _abi.load()
    with _timing.launch("rqf_readout_bias_relu_backward", H * B * T, 2 * _nbytes(gg)):
        _abi.check(lib.rqf_readout_bias_relu_backward(
            _abi.ptr(gg), _abi.ptr(mask), _abi.ptr(g), _abi.ptr(rowsum), H, B, T,
            _abi.stream_of(gg)), "rqf_readout_bias_relu_backward")
    _done(dev)
    return g, rowsum


# ------------------------------------------------ real-operand projections
def projection_real(W: torch.Tensor, x: torch.Tensor, conj_transpose: bool = False,
                    acc: torch.Tensor | None = None) -> torch.Tensor:
    """out = op(W) @ x (+ acc) for a real float32 x (K, ...), complex64 out
    (M, ...): the readout's input cotangent V^H g with g real
    (rqf_projection_real, half the tensor-core work of projection on a
    complex x).  N not a multiple of 4 runs torch.matmul on the GPU."""
    dev = _require_cuda(W, x, acc)
    w = _c64(W)
    xx = x.detach().to(torch.float32).contiguous()
    K = int(xx.shape[0])
    M = int(w.shape[1] if conj_transpose else w.shape[0])
    if int(w.shape[0] if conj_transpose else w.shape[1]) != K:
        raise ValueError(f"W {tuple(w.shape)} does not match x {tuple(xx.shape)}")
    tail = tuple(xx.shape[1:])
    N = xx.numel() // K if K else 0
    out_shape = (M,) + tail
    a = _c64(acc) if acc is not None else None
    if a is not None and tuple(a.shape) != out_shape:
        raise ValueError(f"acc must have shape {out_shape}, got {tuple(a.shape)}")
    if N % 4 != 0:
        opw = w.mH if conj_transpose else w
        out = (opw @ xx.reshape(K, N).to(torch.complex64)).reshape(out_shape)
        return out if a is None else out.add_(a)
    lib = _abi.load()
    out = torch.empty(out_shape, dtype=torch.complex64, device=dev)
    ws = _scratch(lib.rqf_projection_workspace_bytes(M, K), dev)
    with _timing.launch("rqf_projection_real", M * N, _nbytes(xx, out, a), 4 * M * K * N):
        _abi.check(lib.rqf_projection_real(
            _abi.ptr(w), _abi.ptr(xx), _abi.ptr(a), _abi.ptr(out), M, K, N, int(bool(conj_transpose)),
            _abi.ptr(ws), _abi.stream_of(out)), "rqf_projection_real")
    _done(dev)
    return out


def projection_weight_grad_real(gz: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """gW = gz @ x^H for a real float32 gz (M, ...) and complex x (K, ...):
    the readout's weight cotangent with its real cotangent g
    (rqf_projection_weight_grad_real: the reduction runs over the samples,
    half the k-blocks of the complex form).  N not a multiple of 4 runs
    torch.matmul on the GPU."""
    dev = _require_cuda(gz, x)
    g = gz.detach().to(torch.float32).contiguous()
    xx = _c64(x)
    M, K = int(g.shape[0]), int(xx.shape[0])
    if tuple(g.shape[1:]) != tuple(xx.shape[1:]):
        raise ValueError(f"gz {tuple(g.shape)} and x {tuple(xx.shape)} differ in trailing dims")
    N = g.numel() // M if M else 0
    if N % 4 != 0:
        return g.reshape(M, N).to(torch.complex64) @ xx.reshape(K, N).mH
    lib = _abi.load()
    gw = torch.empty((M, K), dtype=torch.complex64, device=dev)
    ws = _scratch(lib.rqf_projection_weight_grad_real_workspace_bytes(M, K, N), dev)
    with _timing.launch("rqf_projection_weight_grad_real", M * N, _nbytes(g, xx, gw),
                        4 * M * K * N):
        _abi.check(lib.rqf_projection_weight_grad_real(
            _abi.ptr(g), _abi.ptr(xx), _abi.ptr(gw), M, K, N, _abi.ptr(ws),
            _abi.stream_of(g)), "rqf_projection_weight_grad_real")
    _done(dev)
    return gw


class _SplitProjection(torch.autograd.Function):
    """The selective controller's projection (rqf_models/backbones/rqf/
    selective.py:_SplitProjection :78-97): logits = weights @ v split into
    the gamma / warp / write heads, with v = [Re s; Im s] (2I, N) and
    weights (M, 2I) real.  On the split-TF32 tensor-core GEMMs in their
    complex-as-real forms, with s = v[:I] + i v[I:] and Wr, Wi the two
    column halves of weights:
      logits = Re((Wr - i Wi) s)          (rqf_projection_real_out)
      grad v = [Re u; Im u],  u = (Wr^T + i Wi^T) grad     (rqf_projection_real)
      grad weights = [Re P, -Im P],  P = grad s^H          (rqf_projection_weight_grad_real)
    The reference runs the three as fp32 cuBLAS GEMMs (SIMT on B200)."""

    @staticmethod
    def forward(ctx, v, weights, sizes):
        I = v.shape[0] // 2
        s = torch.complex(v[:I], v[I:]).contiguous()
        wr, wi = weights[:, :I], weights[:, I:]
        ctx.save_for_backward(s, weights)
        ctx.sizes = sizes
        ctx.set_materialize_grads(False)
        out = projection_real_out(torch.complex(wr, -wi), s)
        return out.split(sizes)

    @staticmethod
    @once_differentiable
    def backward(ctx, *grads):
        s, weights = ctx.saved_tensors
        I, N = s.shape
        grad = torch.cat([g if g is not None else s.real.new_zeros((n, N))
                          for g, n in zip(grads, ctx.sizes) if n])
        need = ctx.needs_input_grad
        gv = gw = None
        if need[0]:
            u = projection_real(torch.complex(weights[:, :I].t(), weights[:, I:].t()), grad)
            gv = torch.cat((u.real, u.imag))
        if need[1]:
            P = projection_weight_grad_real(grad, s)
            gw = torch.cat((P.real, -P.imag), dim=1)
        return gv, gw, None


def projection_real_out(W: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """Re(W @ x) as float32 (M, ...) for complex W (M, K) and x (K, ...): the
    readout hidden layer's pre-activation W1 [Re h; Im h] with W = W1[:, :F] -
    i W1[:, F:] (rqf_projection_real_out, half the tensor-core work of the
    complex projection).  N not a multiple of 4 runs torch.matmul on the GPU."""
    dev = _require_cuda(W, x)
    w = _c64(W)
    xx = _c64(x)
    M, K = int(w.shape[0]), int(xx.shape[0])
    if int(w.shape[1]) != K:
        raise ValueError(f"W {tuple(w.shape)} does not match x {tuple(xx.shape)}")
    tail = tuple(xx.shape[1:])
    N = xx.numel() // K if K else 0
    if N % 4 != 0:
        return (w @ xx.reshape(K, N)).real.reshape((M,) + tail).contiguous()
    lib = _abi.load()
    out = torch.empty((M,) + tail, dtype=torch.float32, device=dev)
    ws = _scratch(lib.rqf_projection_real_out_workspace_bytes(M, K), dev)
    with _timing.launch("rqf_projection_real_out", M * N, _nbytes(xx, out), 4 * M * K * N):
        _abi.check(lib.rqf_projection_real_out(
            _abi.ptr(w), _abi.ptr(xx), _abi.ptr(out), M, K, N, _abi.ptr(ws),
            _abi.stream_of(out)), "rqf_projection_real_out")
    _done(dev)
    return out


# ------------------------------------------------ two-tap coefficient producer
class TwoTapCoefficients(torch.autograd.Function):
    """(c1, tap0, tap1) complex64 of log-space leaves (log_theta, log_gamma)
    of any shape (filter.py:510-664, ZOH, tau mode, rho = 1): one forward and
    one backward launch (rqf_two_tap_coefficients[_backward], double inside)
    instead of the ~90 small torch kernels of the same expressions."""

    @staticmethod
    def forward(ctx, log_theta, log_gamma, dt, tau):
        dev = _require_cuda(log_theta, log_gamma)
        lt = log_theta.detach().to(torch.float32).contiguous()
        lg = log_gamma.detach().to(torch.float32).contiguous()
        if lt.shape != lg.shape:
            raise ValueError(f"log_theta {tuple(lt.shape)} and log_gamma {tuple(lg.shape)} differ")
        outs = [torch.empty(lt.shape, dtype=torch.complex64, device=dev) for _ in range(3)]
        lib = _abi.load()
        with _timing.launch("rqf_two_tap_coefficients", lt.numel(), 0):
            _abi.check(lib.rqf_two_tap_coefficients(
                _abi.ptr(lt), _abi.ptr(lg), *(_abi.ptr(o) for o in outs), lt.numel(), float(dt),
                float(tau), _abi.stream_of(lt)), "rqf_two_tap_coefficients")
        _done(dev)
        ctx.save_for_backward(lt, lg)
        ctx.dt, ctx.tau = float(dt), float(tau)
        return tuple(outs)

    @staticmethod
    @once_differentiable
    def backward(ctx, g1, g0, gm):
        lt, lg = ctx.saved_tensors
        gs = [None if g is None else _c64(g) for g in (g1, g0, gm)]
        glt, glg = torch.empty_like(lt), torch.empty_like(lg)
        lib = _abi.load()
        _abi.check(lib.rqf_two_tap_coefficients_backward(
            _abi.ptr(lt), _abi.ptr(lg), *(_abi.ptr(g) for g in gs), _abi.ptr(glt), _abi.ptr(glg),
            lt.numel(), ctx.dt, ctx.tau, _abi.stream_of(lt)), "rqf_two_tap_coefficients_backward")
        _done(lt.device)
        return glt, glg, None, None


# ------------------------------------------- RQF filter-bank coefficients
_DISCRETIZATIONS = {"euler": 0, "zoh": 1, "foh": 2}


class FilterTwoTapCoefficients(torch.autograd.Function):
    """(C1, tap0, tap1) complex64 of an RQF filter bank's leaves, every
    two-tap branch of filter.py:510-664 (rqf_filter_two_tap_coefficients and
    its backward: one launch each, double inside, derivatives carried through
    every branch).  Gradients reach the theta / gamma leaves, log_tau and a
    prospective_tau tensor when they need one; the sigmoid bounds are
    constants (buffers in the reference)."""

    @staticmethod
    def forward(ctx, theta_leaf, gamma_leaf, log_tau, tau_p, min_g, max_g, min_f, max_f, disc,
                prospective, gamma_mode, sigmoid, clamp, dt):
        dev = _require_cuda(theta_leaf, gamma_leaf, log_tau, tau_p, min_g, max_g, min_f, max_f)
        n = theta_leaf.numel()

        def f32(t):
            if t is None:
                return None
            t = t.detach().to(torch.float32).contiguous()
            if t.numel() != n:
                raise ValueError(f"filter-bank tensor of {t.numel()} elements, expected {n}")
            return t

        ts = [f32(t) for t in (theta_leaf, gamma_leaf, log_tau, min_g, max_g, min_f, max_f,
                               tau_p)]
        leaves = _abi.CoeffLeaves(*(_abi.ptr(t) for t in ts))
        opts = _abi.CoeffOptions(int(disc), int(prospective), int(gamma_mode), int(sigmoid),
                                 int(clamp), float(dt), 0.0)
        outs = [torch.empty(theta_leaf.shape, dtype=torch.complex64, device=dev)
                for _ in range(3)]
        lib = _abi.load()
        with _timing.launch("rqf_filter_two_tap_coefficients", n, 0):
            _abi.check(lib.rqf_filter_two_tap_coefficients(
                ctypes.byref(leaves), ctypes.byref(opts), *(_abi.ptr(o) for o in outs), n,
                _abi.stream_of(outs[0])), "rqf_filter_two_tap_coefficients")
        _done(dev)
        ctx.save_for_backward(*[t for t in ts])
        ctx.has = [t is not None for t in ts]
        ctx.opts = (int(disc), int(prospective), int(gamma_mode), int(sigmoid), int(clamp),
                    float(dt))
        ctx.shapes = [None if t is None else t.shape for t in (theta_leaf, gamma_leaf, log_tau,
                                                                tau_p)]
        return tuple(outs)

    @staticmethod
    @once_differentiable
    def backward(ctx, g1, g0, gm):
        ts = list(ctx.saved_tensors)
        n = ts[0].numel()
        leaves = _abi.CoeffLeaves(*(_abi.ptr(t) for t in ts))
        opts = _abi.CoeffOptions(*ctx.opts[:5], ctx.opts[5], 0.0)
        need = ctx.needs_input_grad
        gs = [None if g is None else _c64(g) for g in (g1, g0, gm)]
        # outputs: theta leaf, gamma leaf, log_tau, tau_p
        want = [need[0], need[1], need[2] and ts[2] is not None, need[3] and ts[7] is not None]
        grads = [torch.empty(n, dtype=torch.float32, device=ts[0].device) if w else None
                 for w in want]
        lib = _abi.load()
        _abi.check(lib.rqf_filter_two_tap_coefficients_backward(
            ctypes.byref(leaves), ctypes.byref(opts), *(_abi.ptr(g) for g in gs),
            *(_abi.ptr(g) for g in grads), n, _abi.stream_of(ts[0])),
            "rqf_filter_two_tap_coefficients_backward")
        _done(ts[0].device)
        out = [None if g is None else g.view(shape)
               for g, shape in zip(grads, ctx.shapes)]
        return (*out, None, None, None, None, None, None, None, None, None, None)


def filter_two_tap_coefficients(rqf, prospective: bool = True, mode: str = "tau",
                                prospective_tau=None):
    """Drop-in for RQF.compute_two_tap_coefficients (filter.py:510-664) of an
    RQF module whose leaves are fp32 CUDA tensors: the same (C1, tap0, tap1),
    the same errors for the forms without a two-tap update, Euler's taps real
    as the reference returns them."""
    if mode not in ("tau", "gamma"):
        raise ValueError(f"mode must be one of ('tau', 'gamma'), got {mode!r}")
    disc = rqf.discretization
    if disc == "bilinear":
        raise NotImplementedError(
            "Two-tap update is not defined for bilinear discretization. "
            "Use 'euler', 'zoh', or 'foh'.")
    if disc in ("euler", "zoh") and not prospective:
        raise NotImplementedError(
            f"Non-prospective {'Euler' if disc == 'euler' else 'ZOH'} uses the single-tap "
            "recurrence; call compute_coefficients() instead.")
    log_tau = rqf.log_tau
    if rqf.param_space == "log":
        theta_leaf, gamma_leaf, bounds, sigmoid = rqf.log_theta, rqf.log_gamma, (None,) * 4, 0
    else:
        theta_leaf, gamma_leaf, sigmoid = rqf.freq_param, rqf.gamma_param, 1
        bounds = (rqf._min_gamma, rqf._max_gamma, rqf._min_freq, rqf._max_freq)
    tau_p = None
    if prospective_tau is not None:
        tau_p = torch.as_tensor(prospective_tau, dtype=log_tau.dtype, device=log_tau.device)
        tau_p = tau_p.expand(log_tau.shape)
    c1, t0, t1 = FilterTwoTapCoefficients.apply(
        theta_leaf, gamma_leaf, log_tau, tau_p, *bounds, _DISCRETIZATIONS[disc],
        bool(prospective), mode == "gamma", sigmoid, bool(rqf.clamp_gamma), float(rqf.dt))
    if disc == "euler":
        return c1, t0.real, t1.real
    return c1, t0, t1
