"""GPU parity of the Pure RQF block forward fused into its projection GEMM
(rqf_projection_block_scan, ops.projection_block_scan): z = W h on the
split-TF32 tensor cores with the (F,B,T) two-tap scan, split-ReLU and skip add
(rqf_models/backbones/rqf/pure.py:223 and :529-535) run in the GEMM's
epilogue.

Checked against the fp64 oracle: z against an fp64 GEMM (5e-6, the
projection's own bound), out against the oracle scan of that z plus skip
(forward tolerance 1e-4), and the (F,B,T) backward run on the fused forward's
saved context against the oracle VJP (gradient tolerance 1e-3) — the saved
entry states must be the ones the backward needs.  Against the unfused path
(rqf_projection, then rqf_fbt_block_forward) z is bit-identical and out agrees
to fp32 rounding.  Shapes cover one GEMM tile per row (T = 128), context tiles
cut by T (T % 2048 != 0: the padded slots), filters that do not fill a pair
tile (rows past F), a single chain (B = 1) whose tiles all wait on one
another, and more chains than CTA pairs.
"""

import numpy as np
import pytest
import torch

from _util import FWD_TOL, GRAD_ELEM_TOL, GRAD_TOL, assert_close
from oracle import oracle

pytestmark = pytest.mark.gpu

PROJ_TOL = 5e-6
MASK_EDGE = 1e-4


@pytest.fixture(scope="module", autouse=True)
def _device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import prospective_rqf_b200 as rqf

    rqf.read_device_error(clear=True)
    yield
    rqf.check_device_errors()


def _host(t):
    return t.detach().cpu().numpy().astype(np.complex128)


def _case(F, K, B, T, seed):
    rng = np.random.default_rng(seed)
    mag = rng.uniform(0.8, 0.999, F)
    c1 = (mag * np.exp(1j * rng.uniform(0, 2 * np.pi, F))).astype(np.complex64)
    t0 = (0.5 * (rng.standard_normal(F) + 1j * rng.standard_normal(F))).astype(np.complex64)
    t1 = (0.5 * (rng.standard_normal(F) + 1j * rng.standard_normal(F))).astype(np.complex64)
    W = ((rng.standard_normal((F, K)) + 1j * rng.standard_normal((F, K))) /
         np.sqrt(2 * K)).astype(np.complex64)
    h = (rng.standard_normal((K, B, T)) + 1j * rng.standard_normal((K, B, T))).astype(np.complex64)
    return [torch.from_numpy(a).cuda() for a in (W, h, c1, t0, t1)]


# (F, K, B, T)
SHAPES = [
    (64, 64, 2, 256),      # F below one pair tile's 128 filters
    (128, 96, 3, 2176),    # two context tiles, the second cut at 128 samples
    (256, 256, 4, 4096),   # whole context tiles
    (96, 96, 1, 128),      # one GEMM tile per row, one chain per row block
    (200, 136, 5, 1920),   # ragged F and K, T below one context tile
    (128, 128, 1, 8192),   # a single chain: 64 tiles, each waiting on the last
    (128, 128, 96, 256),   # more chains than CTA pairs
    (256, 256, 40, 256),   # two row blocks, 80 chains
]


@pytest.mark.parametrize("F,K,B,T", SHAPES)
@pytest.mark.parametrize("fuse", [True, False])
@pytest.mark.parametrize("with_skip", [True, False])
def test_block_scan_vs_oracle(F, K, B, T, fuse, with_skip):
    from prospective_rqf_b200 import ops

    W, h, c1, t0, t1 = _case(F, K, B, T, F * 131 + K * 17 + B * 7 + T + 2 * fuse + with_skip)
    skip = None
    if with_skip:
        skip = h if F == K else torch.randn(F, B, T, dtype=torch.complex64, device="cuda")
    out, saved = ops.projection_block_scan(W, h, c1, t0, t1, fuse, skip)
    z = saved[3]

    z_ref = (W.cpu().to(torch.complex128) @ h.cpu().to(torch.complex128).reshape(K, -1))
    assert_close(_host(z), z_ref.reshape(F, B, T).numpy(), PROJ_TOL, "z")

    zc, c1h, t0h, t1h = _host(z), _host(c1), _host(t0), _host(t1)
    y_ref = oracle.two_tap_forward(c1h, t0h, t1h, zc, "fbt", fuse_act=fuse)
    sk = 0 if skip is None else _host(skip)
    assert_close(_host(out), y_ref + sk, FWD_TOL, "out")

    # the unfused path on the same inputs
    z2 = ops.projection(W, h)
    assert torch.equal(z, z2), "z differs from rqf_projection's"
    out2, saved2 = ops._fbt_forward(c1, t0, t1, z2, fuse, skip)
    assert_close(_host(out), _host(out2), 1e-5, "out vs unfused")

    # the backward on the fused forward's saved context
    g = torch.randn(F, B, T, dtype=torch.complex64, device="cuda",
                    generator=torch.Generator(device="cuda").manual_seed(T + F))
    gc1, gt0, gt1, gz = ops._fbt_backward(saved, g, fuse)
    mask = None
    if fuse:
        # the kernel's own decisions: act from the same forward without skip
        # (out - skip would lose activations below the skip's rounding)
        act = out if skip is None else ops.projection_block_scan(W, h, c1, t0, t1, fuse)[0]
        mask = oracle.relu_mask_from_output(_host(act))
        raw = oracle.two_tap_forward(c1h, t0h, t1h, zc, "fbt", fuse_act=False)
        assert oracle.mask_disagreement(mask, raw) < MASK_EDGE
    rz, rc1, rt0, rt1 = oracle.two_tap_backward(c1h, t0h, t1h, zc, _host(g), "fbt",
                                                fuse_act=fuse, mask=mask)
    for got, ref, name in ((gz, rz, "gz"), (gc1, rc1, "gc1"), (gt0, rt0, "gt0"),
                           (gt1, rt1, "gt1")):
        assert_close(_host(got), ref, GRAD_TOL, name)


@pytest.mark.parametrize("T", [1920, 2176, 4096])
@pytest.mark.parametrize("B", [3, 40])
def test_block_scan_saved_entries(T, B):
    """The saved context holds the raw state entering every 8-sample group
    (slot s of context tile j of row (f, b): y[f, b, 2048 j + 8 s - 1]), zero
    in the slots past T, and the every-thread marker (1, 0) after the slots,
    with few chains (B = 3) and with more than half the CTA pairs (B = 40)."""
    from prospective_rqf_b200 import _abi, ops

    F, K = 128, 64
    W, h, c1, t0, t1 = _case(F, K, B, T, 77 + T)
    _, saved = ops.projection_block_scan(W, h, c1, t0, t1, False, None)
    z, carries = saved[3], saved[4]
    lib = _abi.load()
    ntiles = int(lib.rqf_fbt_num_tiles(T))
    assert carries.numel() == int(lib.rqf_fbt_carry_count(F, B, T)) == F * B * ntiles * 256 + 1
    c = _host(carries)
    assert c[-1] == 1.0 + 0.0j
    slots = c[:-1].reshape(F, B, ntiles * 256)
    y = oracle.two_tap_forward(_host(c1), _host(t0), _host(t1), _host(z), "fbt")
    t_entry = np.arange(0, T, 8)
    want = np.zeros((F, B, T // 8), np.complex128)
    want[:, :, 1:] = y[:, :, t_entry[1:] - 1]
    assert_close(slots[:, :, : T // 8], want, FWD_TOL, "entries")
    assert np.all(slots[:, :, T // 8:] == 0)


@pytest.mark.parametrize("fuse", [True, False])
def test_block_scan_tbptt_backward(fuse):
    """The TBPTT(1) backward (rqf_tbptt1_two_tap_backward, layout 1) replays
    from the fused forward's saved entries.  g is pointwise here, so the
    oracle runs on the cotangent pre-masked by the fused forward's own
    split-ReLU decisions (checked to differ from fp64 only near 0)."""
    from prospective_rqf_b200 import ops

    F, K, B, T = 128, 128, 4, 2176
    W, h, c1, t0, t1 = _case(F, K, B, T, 5 + fuse)
    y, saved = ops.projection_block_scan(W, h, c1, t0, t1, fuse, None)
    g = torch.randn(F, B, T, dtype=torch.complex64, device="cuda",
                    generator=torch.Generator(device="cuda").manual_seed(3))
    got = ops._tbptt_backward(saved, "fbt", (F, B, T), g, fuse)
    zc, c1h, t0h, t1h, gh = (_host(a) for a in (saved[3], c1, t0, t1, g))
    g_ref = gh
    if fuse:
        mask = oracle.relu_mask_from_output(_host(y))
        raw = oracle.two_tap_forward(c1h, t0h, t1h, zc, "fbt", fuse_act=False)
        assert oracle.mask_disagreement(mask, raw) < MASK_EDGE
        g_ref = np.where(mask[..., 0], gh.real, 0.0) + 1j * np.where(mask[..., 1], gh.imag, 0.0)
    rz, rzw, rc1, rt0, rt1 = oracle.tbptt_backward(c1h, t0h, t1h, zc, g_ref, "fbt",
                                                   fuse_act=False)
    for a, r, name in zip(got, (rc1, rt0, rt1, rz, rzw), ("gc1", "gt0", "gt1", "gz", "gzw")):
        assert_close(_host(a), r, GRAD_TOL, name)


def test_block_scan_rejects():
    from prospective_rqf_b200 import _abi, ops

    W, h, c1, t0, t1 = _case(64, 64, 2, 200, 1)
    assert not ops.block_scan_eligible(W, h)
    with pytest.raises(ValueError):
        ops.projection_block_scan(W, h, c1, t0, t1, True)
    lib = _abi.load()
    assert lib.rqf_projection_block_scan_workspace_bytes(64, 64, 2, 200) == 0
    assert lib.rqf_projection_block_scan_workspace_bytes(64, 64, 2, 256) > 0
    W, h, c1, t0, t1 = _case(64, 64, 2, 256, 2)
    out = torch.empty_like(h)
    car = torch.empty(int(lib.rqf_fbt_carry_count(64, 2, 256)), dtype=torch.complex64,
                      device="cuda")
    ws = torch.empty(int(lib.rqf_projection_block_scan_workspace_bytes(64, 64, 2, 256)),
                     dtype=torch.uint8, device="cuda")
    p = _abi.ptr
    args = lambda x, z, o, T: (p(W), p(x), p(c1), p(t0), p(t1), None, p(z), p(o), p(car), p(ws),
                               64, 64, 2, T, 1, _abi.stream_of(h))
    # out == x, z == x: RQF_ERR_ARGUMENT (5); T % 128 != 0: RQF_ERR_SHAPE (1)
    assert lib.rqf_projection_block_scan(*args(h, out, h, 256)) == 5
    assert lib.rqf_projection_block_scan(*args(h, h, out, 256)) == 5
    assert lib.rqf_projection_block_scan(*args(h, out, torch.empty_like(h), 200)) == 1
    torch.cuda.synchronize()


def test_encoder_block_scan_matches_unfused():
    """The encoder at T = 4096 (a multiple of 128) with its blocks on the
    fused forward and backward launches and on the separate projection +
    scan: features and every parameter gradient agree to fp32 rounding."""
    from prospective_rqf_b200 import encoder

    torch.manual_seed(0)
    enc = encoder.PureRQFEncoderB200(input_dims=1, hidden_dims=128, num_layers=4,
                                     samp_frequency=16000.0, tau=0.0003125, seq_duration=1.0,
                                     skip_connection=True, final_activation=False).cuda()
    x = 0.5 * torch.randn(4, 4096, 1, device="cuda")
    res = []
    for fused in ("1", "0"):
        encoder.BLOCK_SCAN = encoder.BLOCK_SCAN_BWD = fused
        try:
            enc.zero_grad()
            h = enc(x)
            (h.abs() ** 2).mean().backward()
            res.append((h.detach().clone(),
                        {n: p.grad.detach().clone() for n, p in enc.named_parameters()}))
        finally:
            encoder.BLOCK_SCAN = encoder.BLOCK_SCAN_BWD = "auto"
    (h1, g1), (h2, g2) = res
    assert_close(_host(h1), _host(h2), 1e-5, "features")
    for n in g1:
        assert_close(g1[n].cpu().numpy().astype(np.complex128),
                     g2[n].cpu().numpy().astype(np.complex128), 1e-4, n)


# ------------------------------------------------------------ fused backward
# (F, K, k, B, T): the lower block's F filters over K inputs, the upper
# block's k filters over those F
BWD_SHAPES = [
    (64, 64, 96, 2, 256),       # F below one pair tile's 128 rows
    (128, 96, 128, 3, 2176),    # two context tiles, the second cut at 128 samples
    (256, 256, 256, 4, 4096),   # whole context tiles
    (96, 96, 64, 1, 128),       # one GEMM tile per row, one chain per row block
    (200, 136, 160, 5, 1920),   # ragged F, K and k; T below one context tile
    (128, 128, 128, 1, 8192),   # a single chain of 64 tiles, run from its end
    (128, 128, 128, 96, 256),   # more chains than CTA pairs
]


def _upper(k, F, B, T, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    W = (torch.randn(k, F, generator=g, dtype=torch.complex64) / np.sqrt(F)).cuda()
    gz = torch.randn(k, B, T, generator=g, dtype=torch.complex64).cuda()
    acc = torch.randn(F, B, T, generator=g, dtype=torch.complex64).cuda()
    return W, gz, acc


@pytest.mark.parametrize("F,K,k,B,T", BWD_SHAPES)
@pytest.mark.parametrize("fuse", [True, False])
@pytest.mark.parametrize("with_acc", [True, False])
def test_block_scan_backward_vs_oracle(F, K, k, B, T, fuse, with_acc):
    """rqf_projection_block_scan_backward: g = W^H gz_above (+ acc) against an
    fp64 GEMM (the projection's bound) and bit-identical to rqf_projection's;
    the lower block's scan VJP of that g against the fp64 oracle (gradient
    tolerance, the kernel's own split-ReLU decisions) and against the
    separate (F,B,T) backward on the same g."""
    from prospective_rqf_b200 import ops

    seed = F * 7 + K * 3 + k + B * 11 + T + 2 * fuse + with_acc
    W0, h, c1, t0, t1 = _case(F, K, B, T, seed)
    act, saved = ops.projection_block_scan(W0, h, c1, t0, t1, fuse, None)
    W, gz_above, acc = _upper(k, F, B, T, seed + 1)
    if not with_acc:
        acc = None
    g, (gc1, gt0, gt1, gz) = ops.projection_block_scan_backward(W, gz_above, acc, saved, fuse)

    g2 = ops.projection(W, gz_above, conj_transpose=True, acc=acc)
    assert torch.equal(g, g2), "g differs from rqf_projection's"
    g_ref = W.cpu().to(torch.complex128).mH @ gz_above.cpu().to(torch.complex128).reshape(k, -1)
    g_ref = g_ref.reshape(F, B, T).numpy()
    if acc is not None:
        g_ref = g_ref + _host(acc)
    assert_close(_host(g), g_ref, PROJ_TOL, "g")

    zc, c1h, t0h, t1h = _host(saved[3]), _host(c1), _host(t0), _host(t1)
    mask = None
    if fuse:
        mask = oracle.relu_mask_from_output(_host(act))
        raw = oracle.two_tap_forward(c1h, t0h, t1h, zc, "fbt", fuse_act=False)
        assert oracle.mask_disagreement(mask, raw) < MASK_EDGE
    rz, rc1, rt0, rt1 = oracle.two_tap_backward(c1h, t0h, t1h, zc, _host(g), "fbt",
                                                fuse_act=fuse, mask=mask)
    sep = ops._fbt_backward(saved, g, fuse)
    for got, ref, other, name in ((gz, rz, sep[3], "gz"), (gc1, rc1, sep[0], "gc1"),
                                  (gt0, rt0, sep[1], "gt0"), (gt1, rt1, sep[2], "gt1")):
        assert_close(_host(got), ref, GRAD_TOL, name, elem_tol=GRAD_ELEM_TOL)
        assert_close(_host(got), _host(other), 1e-5, name + " vs the separate backward")


def test_block_scan_backward_after_row_kernel_forward():
    """The lower block's context from the separate (F,B,T) forward (row
    kernels at this size) serves the fused backward as well."""
    from prospective_rqf_b200 import ops

    F, B, T = 256, 8, 2048
    W0, h, c1, t0, t1 = _case(F, F, B, T, 91)
    z = ops.projection(W0, h)
    _, saved = ops._fbt_forward(c1, t0, t1, z, True)
    W, gz_above, acc = _upper(F, F, B, T, 92)
    g, vjp = ops.projection_block_scan_backward(W, gz_above, acc, saved, True)
    sep = ops._fbt_backward(saved, g, True)
    for a, b, name in zip(vjp, sep, ("gc1", "gt0", "gt1", "gz")):
        assert_close(_host(a), _host(b), 1e-5, name)


def test_block_scan_backward_needs_entry_marker():
    """A saved context without the every-thread marker latches
    RQF_ERR_ARGUMENT (5) in the device error word; nothing faults."""
    import prospective_rqf_b200 as rqf
    from prospective_rqf_b200 import ops

    F, B, T = 128, 2, 256
    W0, h, c1, t0, t1 = _case(F, F, B, T, 93)
    _, saved = ops.projection_block_scan(W0, h, c1, t0, t1, True, None)
    carries = saved[4].clone()
    carries[-1] = 0
    W, gz_above, _ = _upper(F, F, B, T, 94)
    rqf.read_device_error(clear=True)
    ops.projection_block_scan_backward(W, gz_above, None, (*saved[:4], carries), True)
    assert rqf.read_device_error(clear=True) == 5
