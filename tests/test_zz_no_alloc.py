"""The allocation-free backward entry point, through the C ABI.

rqf_fbt_prospective_backward_noalloc serves callers that cannot allocate
device memory for scratch (e.g. code inside an allocator callback or a loop
that forbids cudaMalloc after start-up): it keeps its scratch in a fixed
4 MiB array inside the library.  Its results must equal those of
rqf_fbt_prospective_backward with caller-provided scratch, on two calls in a
row (the shared array keeps the previous call's contents).  Collected last
(file name) so a stop-at-first-failure run has already run every other test.
"""

import ctypes

import pytest
import torch

from _util import rel_err

pytestmark = pytest.mark.gpu

CAPACITY = 4 << 20


def _lib():
    from prospective_rqf_b200 import _abi

    return _abi.load(), _abi


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _inputs(F, B, T, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    c1 = (0.97 * torch.exp(1j * torch.rand(F, generator=g) * 3)).to(torch.complex64).cuda()
    t0 = torch.randn(F, generator=g, dtype=torch.complex64).cuda()
    t1 = torch.randn(F, generator=g, dtype=torch.complex64).cuda()
    z = torch.randn(F, B, T, generator=g, dtype=torch.complex64).cuda()
    gy = torch.randn(F, B, T, generator=g, dtype=torch.complex64).cuda()
    return c1, t0, t1, z, gy


def _forward(lib, abi, c1, t0, t1, z, fuse):
    F, B, T = z.shape
    out = torch.empty_like(z)
    carries = torch.empty(max(lib.rqf_fbt_carry_count(F, B, T), 1), dtype=torch.complex64,
                          device="cuda")
    scratch = torch.empty(lib.rqf_fbt_scratch_bytes(F, B, T), dtype=torch.uint8, device="cuda")
    abi.check(lib.rqf_fbt_prospective_forward(_p(c1), _p(t0), _p(t1), _p(z), _p(out),
                                              _p(carries), _p(scratch), F, B, T, int(fuse),
                                              _stream()), "forward")
    return carries


def _grads(F, c1, z):
    return (torch.empty_like(z), torch.empty_like(c1), torch.empty_like(c1),
            torch.empty_like(c1))


# Each checked call follows a call on another shape, with other inputs, so the
# shared array holds a different call's look-back flags, ticket and partials:
# a missing clear would show as a mismatch.  Small row counts take the
# look-back tile kernels (odd T), large ones the persistent row kernels.
CASES = [((3, 5, 5001, True), (40, 16, 6000, True)),
         ((40, 16, 6000, True), (3, 5, 5001, True)),
         ((64, 12, 4096, False), (7, 3, 2049, False))]

# The path is the same kernel with the same launch shape and fixed-order
# reductions, so the results agree to rounding-free equality in practice; the
# bound leaves room only for a different order of the final fp64 sums.
NOALLOC_TOL = 1e-6


def _noalloc(lib, abi, c1, t0, t1, z, carries, gy, fuse):
    F, B, T = z.shape
    got = _grads(F, c1, z)
    for g in got:
        g.fill_(float("nan"))
    abi.check(lib.rqf_fbt_prospective_backward_noalloc(
        _p(c1), _p(t0), _p(t1), _p(z), _p(carries), _p(gy), *(_p(g) for g in got),
        F, B, T, int(fuse), _stream()), "backward_noalloc")
    return got


@pytest.mark.parametrize("case,other", CASES)
def test_noalloc_backward_matches_scratch_backward(case, other):
    lib, abi = _lib()
    F, B, T, fuse = case
    assert lib.rqf_fbt_scratch_bytes(F, B, T) <= CAPACITY
    c1, t0, t1, z, gy = _inputs(F, B, T, seed=F + B + T)
    carries = _forward(lib, abi, c1, t0, t1, z, fuse)

    ref = _grads(F, c1, z)
    scratch = torch.empty(lib.rqf_fbt_scratch_bytes(F, B, T), dtype=torch.uint8, device="cuda")
    abi.check(lib.rqf_fbt_prospective_backward(
        _p(c1), _p(t0), _p(t1), _p(z), _p(carries), _p(gy), *(_p(g) for g in ref),
        _p(scratch), F, B, T, int(fuse), _stream()), "backward")

    oF, oB, oT, ofuse = other
    o_in = _inputs(oF, oB, oT, seed=7 * (oF + oB + oT))
    o_carries = _forward(lib, abi, *o_in[:4], ofuse)
    for call in range(2):  # two checked calls, each after a call on another shape
        _noalloc(lib, abi, *o_in[:4], o_carries, o_in[4], ofuse)
        got = _noalloc(lib, abi, c1, t0, t1, z, carries, gy, fuse)
        torch.cuda.synchronize()
        for name, a, b in zip(("grad_z", "grad_c1", "grad_tap0", "grad_tap1"), got, ref):
            err = rel_err(a.cpu().numpy(), b.cpu().numpy())
            assert err <= NOALLOC_TOL, f"call {call}: {name} differs ({err:.2e})"
    abi.check_device_errors()


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib, _ = _lib()
    F, B, T = 256, 4096, 16000  # per-row partials alone exceed 4 MiB
    assert lib.rqf_fbt_scratch_bytes(F, B, T) > CAPACITY
    st = lib.rqf_fbt_prospective_backward_noalloc(None, None, None, None, None, None, None,
                                                  None, None, None, F, B, T, 1, None)
    assert st == 6  # RQF_ERR_CAPACITY
    assert b"maximum" in lib.rqf_status_string(st)
    # Shapes whose size products would wrap around int64 fail the shape check,
    # which runs before any size is computed.
    huge = (1 << 40, 1 << 30, 1 << 40)
    assert lib.rqf_fbt_scratch_bytes(*huge) == ctypes.c_size_t(-1).value
    st = lib.rqf_fbt_prospective_backward_noalloc(None, None, None, None, None, None, None,
                                                  None, None, None, *huge, 1, None)
    assert st == 1  # RQF_ERR_SHAPE
