"""B200-native (sm_100a) backend for the RQF complex linear-recurrence scan family.

Drop-in replacements for the scan entry points of rqf_models.ops
(Sequel-Institute/prospective-rqf), computed by hand-written CUDA kernels in
librqf_b200.so behind the C ABI of include/rqf_b200.h.

    import prospective_rqf_b200 as rqf
    y = rqf.fbt_recompute_scan(C1, tap0, tap1, z)      # (F,B,T) complex64, CUDA
    rqf.install()                                       # route rqf_models to it
"""

from . import _abi
from ._abi import RQFError, check_device_errors, read_device_error
from .integration import install, uninstall
from .ops import (
    _triton_chunked_scan,
    _triton_chunked_scan_prospective,
    fbt_prospective_scan,
    fbt_layer0_real_scan,
    fbt_recompute_scan,
    parallel_scan,
    selective_backward,
    selective_forward,
    selective_layer_scan,
    sequential_scan,
    sequential_scan_abs,
    tbptt1_scan,
    tbptt1_two_tap_scan,
)

__all__ = [
    "RQFError",
    "check_device_errors",
    "read_device_error",
    "install",
    "uninstall",
    "_triton_chunked_scan",
    "_triton_chunked_scan_prospective",
    "fbt_prospective_scan",
    "fbt_layer0_real_scan",
    "fbt_recompute_scan",
    "parallel_scan",
    "selective_backward",
    "selective_forward",
    "selective_layer_scan",
    "sequential_scan",
    "sequential_scan_abs",
    "tbptt1_scan",
    "tbptt1_two_tap_scan",
]


def library_path():
    return _abi.LIB_PATH
