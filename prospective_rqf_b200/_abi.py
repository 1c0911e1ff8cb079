"""ctypes binding of librqf_b200.so (declarations: include/rqf_b200.h).

This is the product's only route to the GPU kernels.  Loading fails loudly
when the library is missing; there is no CPU fallback anywhere in the package.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "librqf_b200.so"

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t
_f32 = ctypes.c_float
_f64 = ctypes.c_double


class SelectiveOptions(ctypes.Structure):
    """rqf_selective_options (include/rqf_b200.h)."""

    _fields_ = [("has_gamma", _int), ("has_warp", _int), ("has_write", _int),
                ("log_shift", _int), ("gamma_scale", _f32), ("warp_scale", _f32),
                ("prospective", _int), ("gamma_horizon", _int), ("write_sigmoid", _int),
                ("write_max", _f32), ("write_bias", _f32), ("bound_warp", _int)]


class SelectiveInputs(ctypes.Structure):
    """rqf_selective_inputs (include/rqf_b200.h)."""

    _fields_ = [("gamma_logits", _p), ("warp_logits", _p), ("write_logits", _p), ("bias", _p),
                ("theta", _p), ("groups", _p), ("minimum", _p), ("span", _p), ("step", _p),
                ("horizon", _p), ("theta_minimum", _p), ("theta_maximum", _p),
                ("num_groups", _i64)]


class CoeffLeaves(ctypes.Structure):
    """rqf_coeff_leaves (include/rqf_b200.h)."""

    _fields_ = [("theta_leaf", _p), ("gamma_leaf", _p), ("log_tau", _p), ("min_gamma", _p),
                ("max_gamma", _p), ("min_freq", _p), ("max_freq", _p),
                ("prospective_tau", _p)]


class CoeffOptions(ctypes.Structure):
    """rqf_coeff_options (include/rqf_b200.h)."""

    _fields_ = [("discretization", _int), ("prospective", _int), ("gamma_mode", _int),
                ("param_space", _int), ("clamp_gamma", _int), ("dt", _f64), ("tau", _f64)]


_pin = ctypes.POINTER(SelectiveInputs)
_pop = ctypes.POINTER(SelectiveOptions)
_pcl = ctypes.POINTER(CoeffLeaves)
_pco = ctypes.POINTER(CoeffOptions)

# name -> (restype, argtypes); mirrors include/rqf_b200.h exactly.
SIGNATURES: dict[str, tuple] = {
    "rqf_abi_version": (_int, []),
    "rqf_status_string": (ctypes.c_char_p, [_int]),
    "rqf_read_device_error": (_int, [ctypes.POINTER(_int), _int, _p]),
    "rqf_selftest_lookback_timeout": (_int, [_p, _p]),
    "rqf_btf_num_tiles": (_i64, [_i64]),
    "rqf_btf_carry_count": (_i64, [_i64, _i64, _i64]),
    "rqf_btf_scratch_bytes": (_sz, [_i64, _i64, _i64]),
    "rqf_fbt_num_tiles": (_i64, [_i64]),
    "rqf_fbt_carry_count": (_i64, [_i64, _i64, _i64]),
    "rqf_fbt_scratch_bytes": (_sz, [_i64, _i64, _i64]),
    "rqf_chunked_scan_forward": (_int, [_p, _p, _p, _int, _p, _p, _p, _i64, _i64, _i64, _int,
                                        _p]),
    "rqf_chunked_scan_abs_forward": (_int, [_p, _p, _p, _int, _p, _p, _i64, _i64, _i64, _int,
                                            _p]),
    "rqf_multi_osc_forward": (_int, [_p, _p, _p, _p, _int, _p, _int, _p, _p, _i64, _i64, _i64,
                                     _i64, _p]),
    "rqf_multi_osc_backward": (_int, [_p, _p, _p, _p, _int, _p, _p, _p, _p, _p, _p, _p, _i64,
                                      _i64, _i64, _i64, _p]),
    "rqf_multi_osc_carry_count": (_i64, [_i64, _i64, _i64, _i64]),
    "rqf_multi_osc_scratch_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "rqf_chunked_scan_backward": (
        _int, [_p, _p, _p, _int, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "rqf_chunked_prospective_forward": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "rqf_chunked_prospective_backward": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "rqf_fbt_prospective_forward": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "rqf_fbt_block_forward": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "rqf_fbt_prospective_backward": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "rqf_fbt_prospective_backward_noalloc": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "rqf_selective_num_tiles": (_i64, [_i64]),
    "rqf_selective_carry_count": (_i64, [_i64, _i64, _i64]),
    "rqf_selective_scratch_bytes": (_sz, [_i64, _i64, _i64, _int]),
    "rqf_selective_forward": (_int, [_p, _pin, _pop, _p, _p, _p, _i64, _i64, _i64, _p]),
    "rqf_selective_backward": (
        _int, [_p, _pin, _pop, _p, _p, _p, _int, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64,
               _i64, _p]),
    "rqf_selective_forward_bf16": (_int, [_p, _pin, _pop, _p, _p, _p, _i64, _i64, _i64, _p]),
    "rqf_selective_backward_bf16": (
        _int, [_p, _pin, _pop, _p, _p, _p, _int, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64,
               _i64, _p]),
    "rqf_tbptt1_two_tap_backward": (
        _int, [_int, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _int,
               _p]),
    "rqf_projection_workspace_bytes": (_sz, [_i64, _i64]),
    "rqf_projection_timeout_site": (_int, [_int]),
    "rqf_projection": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _p]),
    "rqf_projection_block_scan_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "rqf_projection_block_scan": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _p]),
    "rqf_fbt_rank1_supported": (_int, [_i64, _i64, _i64]),
    "rqf_fbt_rank1_scratch_bytes": (_sz, [_i64, _i64, _i64]),
    "rqf_fbt_rank1_forward": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "rqf_fbt_rank1_backward": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int,
               _int, _p]),
    "rqf_fbt_rank1_tbptt_backward": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
               _int, _int, _p]),
    "rqf_fbt_tbptt1_backward_wsum": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "rqf_projection_block_scan_backward_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "rqf_projection_block_scan_backward": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
               _int, _p]),
    "rqf_projection_weight_grad_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "rqf_projection_weight_grad": (_int, [_p, _p, _p, _i64, _i64, _i64, _p, _p]),
    "rqf_lowrank_drive": (_int, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _int, _p]),
    "rqf_rowdot_workspace_bytes": (_sz, [_i64, _i64, _int, _int]),
    "rqf_rowdot": (_int, [_p, _p, _p, _p, _i64, _i64, _int, _int, _p]),
    "rqf_projection_real": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _p]),
    "rqf_projection_weight_grad_real_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "rqf_projection_weight_grad_real": (_int, [_p, _p, _p, _i64, _i64, _i64, _p, _p]),
    "rqf_projection_real_out_workspace_bytes": (_sz, [_i64, _i64]),
    "rqf_projection_real_out": (_int, [_p, _p, _p, _i64, _i64, _i64, _p, _p]),
    "rqf_filter_two_tap_coefficients": (_int, [_pcl, _pco, _p, _p, _p, _i64, _p]),
    "rqf_filter_two_tap_coefficients_backward": (
        _int, [_pcl, _pco, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "rqf_two_tap_coefficients": (_int, [_p, _p, _p, _p, _p, _i64, _f64, _f64, _p]),
    "rqf_two_tap_coefficients_backward": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _i64, _f64, _f64, _p]),
    "rqf_readout_relu_pool": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _p]),
    "rqf_readout_relu_pool_backward": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _p]),
    "rqf_readout_bias_relu": (_int, [_p, _p, _p, _i64, _i64, _i64, _p]),
    "rqf_readout_bias_relu_backward": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _p]),
    "rqf_per_step_cross_entropy_scratch_bytes": (_sz, [_i64, _i64]),
    "rqf_per_step_cross_entropy": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _f32, _p]),
    "rqf_per_step_cross_entropy_backward": (
        _int, [_p, _p, _p, _p, _i64, _i64, _i64, _f32, _p]),
}

_LIB = None


class RQFError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def load() -> ctypes.CDLL:
    """Load librqf_b200.so (raises if it was not built)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with prospective_rqf_b200._build.build() "
                "(the B200 backend has no CPU fallback)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def status_string(code: int) -> str:
    return load().rqf_status_string(int(code)).decode()


def check(code: int, what: str) -> None:
    if code != 0:
        raise RQFError(f"rqf_b200 {what} failed: {status_string(code)} (status {code})")


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def read_device_error(device=None, clear: bool = True) -> int:
    """Return (and by default clear) the device error word; synchronises."""
    lib = load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    code = _int(0)
    with torch.cuda.device(dev):
        st = lib.rqf_read_device_error(ctypes.byref(code), int(clear),
                                       ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    check(st, "rqf_read_device_error")
    return int(code.value)


def check_device_errors(device=None) -> None:
    """Raise if any kernel latched an error (e.g. a bounded look-back wait ran out)."""
    code = read_device_error(device, clear=True)
    if code != 0:
        raise RQFError(f"rqf_b200 device error: {status_string(code)} (status {code})")
