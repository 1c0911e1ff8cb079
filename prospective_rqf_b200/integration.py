"""Route the reference's scan dispatch to this backend.

``install()`` rebinds the module-level callables that the reference's own
dispatch resolves at call time, so its selection logic (``ORGANICS_RQF_FBT``,
``ORGANICS_SCAN_BACKEND``, the FBT eligibility checks of
rqf_models/backbones/rqf/pure.py:194-210 / :500-508, the CUDA/Triton gates of
rqf_models/ops/scan.py:359-372) stays exactly as it is; only the kernels
behind it change.  ``uninstall()`` restores the originals.

Call sites served (reference paths):
  rqf_models/ops/scan.py:367, :509            -> _triton_chunked_scan
  rqf_models/ops/scan.py:361                   -> B-matrix scan (library GEMM drive + scan)
  rqf_models/backbones/s5/layer.py:254        -> parallel_scan with a B matrix on CUDA
  rqf_models/ops/scan.py:430-432               -> |scan| epilogue (sequential_scan_abs)
  rqf_models/backbones/rqf/block.py:926-934   -> _triton_chunked_scan_prospective
  rqf_models/backbones/rqf/block.py:737-764   -> fused multi-oscillator scans
  rqf_models/backbones/rqf/pure.py:234-238    -> fbt_prospective_scan / fbt_recompute_scan
  rqf_models/ops/fbt_scan_kernel.py:1005       -> fbt_layer0_real_scan (no caller in the reference)
  rqf_models/backbones/rqf/block.py:882, :904 -> TBPTT(1) fused surrogate on CUDA
  rqf_models/ops/selective_scan.py:119, :133   -> selective_forward / selective_backward
  rqf_models/ops/selective_scan.py:107         -> _SelectiveLayerScan (its drive GEMMs on the
                                                  tensor cores)
  rqf_models/backbones/rqf/selective.py:78     -> the controller projection _SplitProjection
                                                  (fp32 CUDA: tensor-core GEMMs)
  rqf_models/backbones/rqf/filter.py:510       -> RQF.compute_two_tap_coefficients on fp32
                                                  CUDA leaves (every caller: pure.py:225,
                                                  block.py's prospective paths, selective.py)
"""

from __future__ import annotations

import importlib

import torch

from . import ops

_SAVED: list[tuple[object, str, object]] = []

_BINDINGS = [
    ("rqf_models.ops.chunked_scan_kernel", "_triton_chunked_scan", ops._triton_chunked_scan),
    ("rqf_models.ops.chunked_scan_kernel", "_triton_chunked_scan_prospective",
     ops._triton_chunked_scan_prospective),
    ("rqf_models.ops.scan", "_triton_chunked_scan", ops._triton_chunked_scan),
    ("rqf_models.ops.scan", "_triton_sequential_scan_b_matrix",
     ops._triton_sequential_scan_b_matrix),
    ("rqf_models.ops.scan", "_sequential_scan_forward_abs_raw_block_f",
     ops._sequential_scan_forward_abs_raw_block_f),
    ("rqf_models.ops.scan", "_sequential_scan_real_forward_abs_raw_block_f",
     ops._sequential_scan_real_forward_abs_raw_block_f),
    ("rqf_models.ops.fbt_scan_kernel", "fbt_prospective_scan", ops.fbt_prospective_scan),
    ("rqf_models.ops.fbt_scan_kernel", "fbt_recompute_scan", ops.fbt_recompute_scan),
    ("rqf_models.ops.fbt_scan_kernel", "fbt_layer0_real_scan", ops.fbt_layer0_real_scan),
    ("rqf_models.backbones.rqf.block", "_triton_chunked_scan_prospective",
     ops._triton_chunked_scan_prospective),
    ("rqf_models.backbones.rqf.pure", "fbt_prospective_scan", ops.fbt_prospective_scan),
    ("rqf_models.backbones.rqf.pure", "fbt_recompute_scan", ops.fbt_recompute_scan),
    ("rqf_models.backbones.rqf.block", "_triton_sequential_scan_multi_osc",
     ops._triton_sequential_scan_multi_osc),
    ("rqf_models.backbones.rqf.block", "_triton_sequential_scan_multi_osc_real",
     ops._triton_sequential_scan_multi_osc_real),
    ("rqf_models.backbones.rqf.block", "_triton_parallel_scan_multi_osc",
     ops._triton_parallel_scan_multi_osc),
    ("rqf_models.backbones.rqf.block", "_sequential_scan_multi_osc_forward_abs_raw",
     ops._sequential_scan_multi_osc_forward_abs_raw),
    ("rqf_models.backbones.rqf.block", "_sequential_scan_multi_osc_real_forward_abs_raw",
     ops._sequential_scan_multi_osc_real_forward_abs_raw),
    ("rqf_models.ops.selective_scan_kernel", "selective_forward", ops.selective_forward),
    ("rqf_models.ops.selective_scan_kernel", "selective_backward", ops.selective_backward),
    ("rqf_models.ops.selective_scan", "_SelectiveLayerScan", ops._SelectiveLayerScan),
]


def _tbptt_two_tap(orig):
    def _scan_two_tap_with_grad_mode(self, u, C1, tap0, tap1, *, delayed_u=None):
        if (self._use_tbptt1_scan_grad() and u.is_cuda and tap0.dim() == 1
                and tap1.dim() == 1):
            return ops.tbptt1_two_tap_scan(u, C1, tap0, tap1, delayed_u=delayed_u, layout="btf")
        return orig(self, u, C1, tap0, tap1, delayed_u=delayed_u)

    _scan_two_tap_with_grad_mode.__wrapped__ = orig
    return _scan_two_tap_with_grad_mode


def _tbptt_single_tap(orig):
    def _scan_with_grad_mode(self, u, C1, C2):
        if self._use_tbptt1_scan_grad() and u.is_cuda and C1.dim() == 1 and C2.dim() == 1:
            return ops.tbptt1_scan(u, C1, C2)
        return orig(self, u, C1, C2)

    _scan_with_grad_mode.__wrapped__ = orig
    return _scan_with_grad_mode


def _cuda_parallel_scan(orig):
    """parallel_scan as bound in a caller module: CUDA inputs take this
    backend (with or without a B matrix; the reference's CUDA branch sends a
    B matrix to its PyTorch Blelloch scan, scan.py:503-529), others keep the
    reference's own path."""
    def parallel_scan(C1, C2, u, B=None):
        if u.is_cuda:
            return ops.parallel_scan(C1, C2, u, B)
        return orig(C1, C2, u, B)

    parallel_scan.__wrapped__ = orig
    return parallel_scan


def _filter_coefficients(orig):
    """RQF.compute_two_tap_coefficients: fp32 CUDA leaves take the fused
    producer (ops.filter_two_tap_coefficients); other dtypes and devices keep
    the reference's own torch expressions."""
    def compute_two_tap_coefficients(self, prospective=True, mode="tau", prospective_tau=None):
        leaves = [self.log_tau] + ([self.log_theta, self.log_gamma] if self.param_space == "log"
                                   else [self.freq_param, self.gamma_param])
        if all(t.is_cuda and t.dtype == torch.float32 for t in leaves):
            return ops.filter_two_tap_coefficients(self, prospective, mode, prospective_tau)
        return orig(self, prospective, mode, prospective_tau)

    compute_two_tap_coefficients.__wrapped__ = orig
    return compute_two_tap_coefficients


def _split_projection(orig):
    """selective.py:_SplitProjection: fp32 CUDA operands take the tensor-core
    form (ops._SplitProjection); others keep the reference's own Function."""
    class _SplitProjection:
        @staticmethod
        def apply(v, weights, sizes):
            if (v.is_cuda and v.dtype == torch.float32 and weights.dtype == torch.float32
                    and v.dim() == 2 and v.shape[0] % 2 == 0):
                return ops._SplitProjection.apply(v, weights, sizes)
            return orig.apply(v, weights, sizes)

    _SplitProjection.__wrapped__ = orig
    return _SplitProjection


# (module, attribute, wrapper of the original)
_WRAPPED = [
    ("rqf_models.backbones.s5.layer", "parallel_scan", _cuda_parallel_scan),
    ("rqf_models.backbones.rqf.selective", "_SplitProjection", _split_projection),
]


def install() -> list[str]:
    """Rebind the reference callables; returns the names that were patched."""
    if _SAVED:
        return [f"{getattr(m, '__name__', m)}.{n}" for m, n, _ in _SAVED]
    patched = []
    for mod_name, attr, fn in _BINDINGS:
        mod = importlib.import_module(mod_name)
        if hasattr(mod, attr):
            _SAVED.append((mod, attr, getattr(mod, attr)))
            setattr(mod, attr, fn)
            patched.append(f"{mod_name}.{attr}")
    for mod_name, attr, wrap in _WRAPPED:
        try:
            mod = importlib.import_module(mod_name)
        except ImportError:
            continue
        if hasattr(mod, attr):
            orig = getattr(mod, attr)
            _SAVED.append((mod, attr, orig))
            setattr(mod, attr, wrap(orig))
            patched.append(f"{mod_name}.{attr}")
    rqf_cls = importlib.import_module("rqf_models.backbones.rqf.filter").RQF
    orig = rqf_cls.compute_two_tap_coefficients
    _SAVED.append((rqf_cls, "compute_two_tap_coefficients", orig))
    rqf_cls.compute_two_tap_coefficients = _filter_coefficients(orig)
    patched.append("rqf_models.backbones.rqf.filter.RQF.compute_two_tap_coefficients")
    block = importlib.import_module("rqf_models.backbones.rqf.block")
    base = block.BaseRQFBlock
    for attr, wrap in (("_scan_two_tap_with_grad_mode", _tbptt_two_tap),
                       ("_scan_with_grad_mode", _tbptt_single_tap)):
        orig = getattr(base, attr)
        _SAVED.append((base, attr, orig))
        setattr(base, attr, wrap(orig))
        patched.append(f"rqf_models.backbones.rqf.block.BaseRQFBlock.{attr}")
    return patched


def uninstall() -> None:
    while _SAVED:
        obj, attr, orig = _SAVED.pop()
        setattr(obj, attr, orig)
