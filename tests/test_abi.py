"""The C-ABI library: builds for sm_100a, loads without a GPU, exports every
symbol include/rqf_b200.h declares, and validates arguments on the host
before touching CUDA.  CPU only (no kernel launches)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "rqf_b200.h"


@pytest.fixture(scope="module")
def lib():
    from prospective_rqf_b200 import _abi, _build

    _build.build()
    return _abi.load()


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rqf_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("rqf_chunked_scan_forward", "rqf_chunked_scan_backward",
                     "rqf_chunked_prospective_forward", "rqf_chunked_prospective_backward",
                     "rqf_fbt_prospective_forward", "rqf_fbt_prospective_backward",
                     "rqf_tbptt1_two_tap_backward"):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_binding_covers_header(lib):
    from prospective_rqf_b200 import _abi

    assert set(declared_functions()) == set(_abi.SIGNATURES)


def _declared_arity():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for name, params in re.findall(r"\b(rqf_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_python_binding_arity_matches_header():
    from prospective_rqf_b200 import _abi

    arity = _declared_arity()
    assert set(arity) == set(_abi.SIGNATURES)
    for name, (_, args) in _abi.SIGNATURES.items():
        assert len(args) == arity[name], f"{name}: {len(args)} ctypes args vs {arity[name]}"


def test_abi_version_and_status_strings(lib):
    assert lib.rqf_abi_version() == 1
    assert lib.rqf_status_string(0) == b"ok"
    assert b"look-back" in lib.rqf_status_string(3)
    assert lib.rqf_status_string(999) == b"unknown status"


def test_size_queries(lib):
    assert lib.rqf_fbt_num_tiles(16000) == 8
    assert lib.rqf_fbt_num_tiles(2048) == 1
    assert lib.rqf_fbt_num_tiles(2049) == 2
    assert lib.rqf_fbt_num_tiles(0) == 0
    # one entry state per thread (256) of every tile, plus the marker element
    assert lib.rqf_fbt_carry_count(128, 16, 16000) == 128 * 16 * 8 * 256 + 1
    assert lib.rqf_btf_num_tiles(161) == 3  # 64-step sub-tiles
    assert lib.rqf_btf_carry_count(32, 161, 128) == 32 * 128 * 3
    s = lib.rqf_fbt_scratch_bytes(128, 16, 16000)
    assert s % 256 == 0 and s >= 256 + 128 * 16 * 8 * 40
    assert lib.rqf_btf_scratch_bytes(0, 10, 10) == 256


def test_btf_path_is_a_per_call_argument(lib):
    """The (B,T,F) kernel family is chosen per call (0 automatic, 1 streaming,
    2 tile-resident); anything else is rejected before any CUDA call."""
    assert not hasattr(lib, "rqf_btf_select_path")
    for bad in (3, -1):
        assert lib.rqf_chunked_scan_forward(None, None, None, 0, None, None, None,
                                            2, 3, 4, bad, None) == 5
        assert lib.rqf_chunked_prospective_backward(None, None, None, None, None, None, None,
                                                    None, None, None, None, 2, 3, 4, bad,
                                                    None) == 5
        assert lib.rqf_tbptt1_two_tap_backward(0, None, None, None, None, None, None, None,
                                               None, None, None, None, None, 1, 1, 1, 0, bad,
                                               None) == 5


def test_host_side_validation_needs_no_gpu(lib):
    # negative sizes -> RQF_ERR_SHAPE, null pointers -> RQF_ERR_ARGUMENT,
    # empty problems -> RQF_OK; all decided before any CUDA call.
    assert lib.rqf_fbt_prospective_forward(None, None, None, None, None, None, None,
                                           -1, 1, 1, 1, None) == 1
    assert lib.rqf_fbt_prospective_forward(None, None, None, None, None, None, None,
                                           1, 1, 1, 1, None) == 5
    assert lib.rqf_fbt_prospective_forward(None, None, None, None, None, None, None,
                                           4, 0, 10, 1, None) == 0
    assert lib.rqf_chunked_scan_forward(None, None, None, 0, None, None, None,
                                        2, 3, -4, 0, None) == 1
    assert lib.rqf_chunked_scan_forward(None, None, None, 0, None, None, None,
                                        2, 3, 4, 0, None) == 5
    assert lib.rqf_tbptt1_two_tap_backward(7, None, None, None, None, None, None, None, None,
                                           None, None, None, None, 1, 1, 1, 0, 0, None) == 5
    # fused block forward: T a multiple of 128, k > 0; empty problems are no-ops
    nul = [None] * 10
    assert lib.rqf_projection_block_scan(*nul, 64, 64, 2, 256, 1, None) == 5
    assert lib.rqf_projection_block_scan(*nul, 64, 64, 2, 200, 1, None) == 1
    assert lib.rqf_projection_block_scan(*nul, 64, 0, 2, 256, 1, None) == 1
    assert lib.rqf_projection_block_scan(*nul, 64, -1, 2, 256, 1, None) == 1
    assert lib.rqf_projection_block_scan(*nul, 0, 64, 2, 256, 1, None) == 0
    assert lib.rqf_projection_block_scan_workspace_bytes(64, 64, 2, 200) == 0
    assert lib.rqf_projection_block_scan_workspace_bytes(64, 64, 2, 256) > \
        lib.rqf_projection_workspace_bytes(64, 64)
    # misaligned pointers -> RQF_ERR_ALIGN
    buf = (ctypes.c_char * 64)()
    base = ctypes.addressof(buf)
    odd = ctypes.c_void_p(base + 1)
    ok = ctypes.c_void_p(base + (16 - base % 16) % 16)
    assert lib.rqf_fbt_prospective_forward(odd, ok, ok, ok, ok, ok, ok, 1, 1, 1, 0, None) == 2


def test_library_is_built_for_sm100a():
    from prospective_rqf_b200 import _build

    flags = " ".join(_build.NVCC_FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags
