"""Failure detection on the GPU without a fault: a cross-tile wait whose
predecessor flag is never published runs out after its bounded number of
polls, the kernel latches RQF_ERR_LOOKBACK_TIMEOUT and returns, the host
reads the status, and the context keeps working afterwards."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_lookback_wait_reports_timeout_and_context_survives():
    import prospective_rqf_b200 as rqf
    from prospective_rqf_b200 import _abi

    assert torch.cuda.is_available()
    lib = _abi.load()
    rqf.read_device_error(clear=True)
    scratch = torch.empty(256, dtype=torch.uint8, device="cuda")
    t0 = time.perf_counter()
    _abi.check(lib.rqf_selftest_lookback_timeout(_abi.ptr(scratch), _abi.stream_of(scratch)),
               "selftest")
    code = rqf.read_device_error(clear=True)  # synchronises: the wait has ended
    elapsed = time.perf_counter() - t0
    assert code == 3, lib.rqf_status_string(code)
    assert elapsed < 30.0
    with pytest.raises(rqf.RQFError, match="look-back"):
        lib.rqf_selftest_lookback_timeout(_abi.ptr(scratch), _abi.stream_of(scratch))
        rqf.check_device_errors()
    # the context is still usable: a normal scan runs and reports no error
    c = torch.full((4,), 0.9 + 0.1j, dtype=torch.complex64, device="cuda")
    y = rqf.fbt_recompute_scan(c, c, c, torch.ones(4, 2, 5000, dtype=torch.complex64,
                                                   device="cuda"))
    assert torch.isfinite(torch.view_as_real(y)).all()
    rqf.check_device_errors()
