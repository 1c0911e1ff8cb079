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


# (M, K, N): ragged M (rows past M in the last pair tile), ragged N (a
# partial last tile), several tiles per pair, and the config-5 layer shape.
INPLACE_SHAPES = [(96, 64, 3 * 700), (37, 50, 1000), (256, 256, 4 * 4096), (256, 256, 32 * 16000)]


@pytest.mark.parametrize("M,K,N", INPLACE_SHAPES)
@pytest.mark.parametrize("conj", [False, True])
def test_projection_inplace_accumulate(M, K, N, conj):
    """ops.projection(..., acc, inplace=True): the epilogue adds its tiles into
    acc with TMA reduce-adds.  The result is the out-of-place W x + acc (one
    fp32 add per element in either path), and acc is the tensor returned."""
    from prospective_rqf_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(M + K + N + int(conj))
    shape = (K, M) if conj else (M, K)
    W = torch.randn(*shape, dtype=torch.complex64, device="cuda", generator=g) / np.sqrt(2 * K)
    x = torch.randn(K, N, dtype=torch.complex64, device="cuda", generator=g)
    acc = torch.randn(M, N, dtype=torch.complex64, device="cuda", generator=g)
    want = ops.projection(W, x, conj, acc)
    buf = acc.clone()
    got = ops.projection(W, x, conj, buf, inplace=True)
    assert got is buf
    torch.cuda.synchronize()
    err = rel_err(got.cpu().numpy(), want.cpu().numpy())
    assert err <= 1e-7, f"in-place accumulate differs from W x + acc ({err:.2e})"
    if N <= 4096:
        assert_close(got.cpu().numpy().astype(np.complex128),
                     _ref(W, x, conj, acc), PROJ_TOL, "in place vs fp64")


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


# ------------------------------------------------ weight gradient gz @ x^H
def _ref_wgrad(gz, x):
    M, K = gz.shape[0], x.shape[0]
    g = gz.cpu().to(torch.complex128).reshape(M, -1)
    xx = x.cpu().to(torch.complex128).reshape(K, -1)
    return (g @ xx.mH).numpy()


WG_SHAPES = [(64, 32, 256), (37, 50, 1000), (128, 128, 4096), (5, 3, 2), (256, 256, 2 * 1111),
             (200, 130, 64)]


@pytest.mark.parametrize("M,K,N", WG_SHAPES)
def test_weight_grad_vs_fp64(M, K, N):
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(M * 131 + K * 7 + N)
    gz, x = _crandn(g, M, N), _crandn(g, K, N)
    gw = ops.projection_weight_grad(gz.cuda(), x.cuda())
    assert gw.shape == (M, K)
    ref = _ref_wgrad(gz, x)
    e32 = rel_err((gz.cuda() @ x.cuda().mH).cpu().numpy(), ref)
    assert_close(gw.cpu().numpy().astype(np.complex128), ref, max(PROJ_TOL, 3 * e32), "gz x^H")


def test_weight_grad_full_layer_shape():
    """Config-5 layer: gz, h of 256 x (32 x 16000), a reduction over 512,000
    samples.  Against fp64 (the fp32 sum over the samples sets the error
    floor, so the bound is tied to torch's own fp32 error) and deterministic."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(9)
    F, B, T = 256, 32, 16000
    gz = torch.randn(F, B, T, dtype=torch.complex64, generator=g).cuda()
    h = torch.randn(F, B, T, dtype=torch.complex64, generator=g).cuda()
    gw = ops.projection_weight_grad(gz, h)
    ref = (gz.reshape(F, -1).to(torch.complex128) @ h.reshape(F, -1).to(torch.complex128).mH)
    ref = ref.cpu().numpy()
    e32 = rel_err((gz.reshape(F, -1) @ h.reshape(F, -1).mH).cpu().numpy(), ref)
    assert_close(gw.cpu().numpy().astype(np.complex128), ref, max(2e-5, 3 * e32), "full layer")
    assert torch.equal(gw, ops.projection_weight_grad(gz, h))


def test_weight_grad_odd_n_uses_torch():
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(4)
    gz, x = _crandn(g, 6, 3, 5), _crandn(g, 4, 3, 5)
    gw = ops.projection_weight_grad(gz.cuda(), x.cuda())
    assert_close(gw.cpu().numpy().astype(np.complex128), _ref_wgrad(gz, x), 1e-6, "odd N")


# ------------------------------------------------ real left operands (readout)
@pytest.mark.parametrize("M,K,N", [(64, 32, 256), (37, 50, 1000), (256, 256, 2 * 1112), (5, 3, 4),
                                   (200, 130, 64)])
@pytest.mark.parametrize("conj", [False, True])
def test_projection_real_x_vs_fp64(M, K, N, conj):
    """rqf_projection_real (x real) against fp64, with and without acc."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(M * 31 + K + N + int(conj))
    W = _crandn(g, *((K, M) if conj else (M, K)), scale=1 / np.sqrt(2 * K))
    x = torch.randn(K, N, generator=g)
    acc = _crandn(g, M, N)
    out = ops.projection_real(W.cuda(), x.cuda(), conj_transpose=conj)
    assert out.shape == (M, N)
    ref = _ref(W, x.to(torch.complex64), conj)
    assert_close(out.cpu().numpy().astype(np.complex128), ref, PROJ_TOL, "op(W) x, x real")
    out2 = ops.projection_real(W.cuda(), x.cuda(), conj, acc.cuda())
    assert_close(out2.cpu().numpy().astype(np.complex128),
                 _ref(W, x.to(torch.complex64), conj, acc), PROJ_TOL, "op(W) x + acc, x real")


@pytest.mark.parametrize("M,K,N", [(64, 32, 256), (37, 50, 1000), (256, 256, 2 * 1112), (5, 3, 4),
                                   (200, 130, 64)])
def test_weight_grad_real_gz_vs_fp64(M, K, N):
    """rqf_projection_weight_grad_real (gz real) against fp64."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(M * 17 + K * 3 + N)
    gz, x = torch.randn(M, N, generator=g), _crandn(g, K, N)
    gw = ops.projection_weight_grad_real(gz.cuda(), x.cuda())
    assert gw.shape == (M, K)
    ref = _ref_wgrad(gz.to(torch.complex64), x)
    e32 = rel_err((gz.cuda().to(torch.complex64) @ x.cuda().mH).cpu().numpy(), ref)
    assert_close(gw.cpu().numpy().astype(np.complex128), ref, max(PROJ_TOL, 3 * e32), "gz x^H, gz real")


def test_weight_grad_real_gz_full_layer_and_deterministic():
    """The readout shape: H = F = 256, N = 32 x 16000 samples."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(12)
    F, B, T = 256, 32, 16000
    gz = torch.randn(F, B, T, generator=g).cuda()
    h = torch.randn(F, B, T, dtype=torch.complex64, generator=g).cuda()
    gw = ops.projection_weight_grad_real(gz, h)
    ref = (gz.reshape(F, -1).double().to(torch.complex128) @ h.reshape(F, -1).to(torch.complex128).mH)
    ref = ref.cpu().numpy()
    e32 = rel_err((gz.reshape(F, -1).to(torch.complex64) @ h.reshape(F, -1).mH).cpu().numpy(), ref)
    assert_close(gw.cpu().numpy().astype(np.complex128), ref, max(2e-5, 3 * e32), "full layer, gz real")
    assert torch.equal(gw, ops.projection_weight_grad_real(gz, h))


@pytest.mark.parametrize("M,K,N", [(64, 32, 256), (37, 50, 1000), (256, 256, 2 * 1112), (5, 3, 4),
                                   (300, 20, 512)])
def test_projection_real_out_vs_fp64(M, K, N):
    """rqf_projection_real_out: Re(W x) as float32 against fp64, normwise
    relative to the full complex product's scale."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(M * 13 + K + N)
    W = _crandn(g, M, K, scale=1 / np.sqrt(2 * K))
    x = _crandn(g, K, N)
    out = ops.projection_real_out(W.cuda(), x.cuda())
    assert out.shape == (M, N) and out.dtype == torch.float32
    ref = _ref(W, x, False)
    # max |out - Re(W x)| / max |W x|: the same normalisation as the complex
    # projection's test (the real part alone is ~1/sqrt(2) of that scale)
    e = np.max(np.abs(out.cpu().numpy().astype(np.float64) - ref.real)) / np.max(np.abs(ref))
    assert e <= PROJ_TOL, f"Re(W x): {e:.3e} of max |W x| > {PROJ_TOL:.1e}"
    out3 = ops.projection_real_out(W.cuda(), x.reshape(K, N // 4, 4).cuda())
    assert out3.shape == (M, N // 4, 4) and torch.equal(out3.reshape(M, N), out)


def test_real_forms_fall_back_for_unaligned_n():
    """N not a multiple of 4 (the kernels' TMA row pitch): the real-operand
    wrappers compute the same products with torch on the GPU."""
    from prospective_rqf_b200 import ops

    g = torch.Generator().manual_seed(21)
    M, K, N = 9, 7, 6
    W = _crandn(g, M, K)
    xr = torch.randn(K, N, generator=g)
    xc = _crandn(g, K, N)
    gr = torch.randn(M, N, generator=g)
    w64 = W.to(torch.complex128)
    out = ops.projection_real(W.cuda(), xr.cuda()).cpu().numpy()
    assert_close(out.astype(np.complex128), (w64 @ xr.double().to(torch.complex128)).numpy(), 1e-6,
                 "projection_real fallback")
    ro = ops.projection_real_out(W.cuda(), xc.cuda()).cpu().numpy()
    assert_close(ro.astype(np.float64), (w64 @ xc.to(torch.complex128)).real.numpy(), 1e-6,
                 "projection_real_out fallback")
    gw = ops.projection_weight_grad_real(gr.cuda(), _crandn(g, K, N).cuda())
    assert gw.shape == (M, K) and gw.dtype == torch.complex64
