"""GPU parity of the split-TF32 tcgen05 projection GEMM (rqf_projection)
against an fp64 GEMM of the same inputs.

out = op(W) @ x (+ acc), complex64; op(W) = W or W^H.  Tolerance (written
here): normwise max relative error <= 5e-6 against fp64 — fp32-comparable
(a single-TF32 product would sit near 1e-3, the fp32 SIMT GEMM it replaces
near 1e-7)."""

import numpy as np
import pytest
import torch

from _util import assert_close, rel_err

pytestmark = pytest.mark.gpu

PROJ_TOL = 5e-6


@pytest.fixture(scope="module", autouse=True)
def _device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import prospective_rqf_b200 as rqf

    rqf.read_device_error(clear=True)
    yield
    rqf.check_device_errors()


def _crandn(g, *shape, scale=1.0):
    return scale * torch.randn(*shape, dtype=torch.complex64, generator=g)


def _ref(W, x, conj, acc=None):
    w = W.cpu().to(torch.complex128)
    opw = w.mH if conj else w
    K = x.shape[0]
    out = (opw @ x.cpu().to(torch.complex128).reshape(K, -1)).reshape((opw.shape[0],) + tuple(x.shape[1:]))
    if acc is not None:
        out = out + acc.cpu().to(torch.complex128)
    return out.numpy()


# (M, K, N): tile-exact, ragged M (not a multiple of 64), ragged K (not a
# multiple of 32), ragged N (not a multiple of 128), tiny, single tile, K=1.
SHAPES = [(64, 32, 256), (128, 256, 4096), (37, 50, 1000), (5, 3, 2), (256, 256, 130),
          (64, 1, 512), (100, 96, 2 * 1111)]


@pytest.mark.parametrize("M,K,N", SHAPES)
@pytest.mark.parametrize("conj", [False, True])
def test_projection_vs_fp64(M, K, N, conj):
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(M * 7919 + K * 31 + N + int(conj))
    W = _crandn(g, *((K, M) if conj else (M, K)), scale=1 / np.sqrt(2 * K))
    x = _crandn(g, K, N)
    out = ops.projection(W.cuda(), x.cuda(), conj_transpose=conj)
    assert out.shape == (M, N)
    assert_close(out.cpu().numpy().astype(np.complex128), _ref(W, x, conj), PROJ_TOL, "projection")


@pytest.mark.parametrize("conj", [False, True])
def test_projection_accumulate_and_alias(conj):
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(11 + int(conj))
    M, K, B, T = 96, 64, 3, 700
    W = _crandn(g, *((K, M) if conj else (M, K)), scale=0.1)
    x = _crandn(g, K, B, T)
    acc = _crandn(g, M, B, T)
    ref = _ref(W, x, conj, acc)
    out = ops.projection(W.cuda(), x.cuda(), conj, acc.cuda())
    assert out.shape == (M, B, T)
    assert_close(out.cpu().numpy().astype(np.complex128), ref, PROJ_TOL, "W x + acc")


def test_projection_full_layer_shape_vs_torch_fp32():
    """The config-5 layer shape (256 x 256, N = 32 x 16000): against an fp64
    GEMM on a column sample, and against torch's fp32 complex GEMM on all of it."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(5)
    F, N = 256, 32 * 16000
    W = _crandn(g, F, F, scale=1 / np.sqrt(2 * F)).cuda()
    x = torch.randn(F, N, dtype=torch.complex64, device="cuda")
    out = ops.projection(W, x)
    cols = torch.randint(0, N, (2048,), generator=g).cuda()
    ref = _ref(W, x[:, cols], False)
    assert_close(out[:, cols].cpu().numpy().astype(np.complex128), ref, PROJ_TOL, "sampled")
    e32 = rel_err((W @ x).cpu().numpy(), out.cpu().numpy())
    assert e32 < 2 * PROJ_TOL, f"vs torch fp32 GEMM: {e32:.2e}"
    out2 = ops.projection(W, x)
    assert torch.equal(out, out2)  # deterministic


def test_projection_odd_n_uses_torch_and_matches():
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(3)
    W, x = _crandn(g, 8, 16), _crandn(g, 16, 3, 5)
    out = ops.projection(W.cuda(), x.cuda())
    assert_close(out.cpu().numpy().astype(np.complex128), _ref(W, x, False), 1e-6, "odd N")
