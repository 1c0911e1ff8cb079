"""numpy fp64 oracle of the selective (input-dependent ZOH) RQF scan.

TEST INFRASTRUCTURE ONLY (checker for tests/ and smoke()).  Restates, with an
explicit hand-derived reverse pass instead of autograd:

  controllers + coefficients  rqf_models/ops/selective_scan.py:
                              selective_coefficients (:26-68)
  recurrence                  selective_scan.py:reference_layer_scan (:71-104)
  autograd boundary           selective_scan.py:_SelectiveLayerScan (:107-170)
                              and selective_scan_kernel.py:selective_backward
                              (:517-561) for the returned tuple

Parity of this oracle with the reference is pinned by
tests/test_oracle_golden.py against tests/golden/selective_*.npz, produced by
reference_layer_scan (fp64 autograd) in tests/golden/make_golden.py.

Layout: every per-element array is (F, B, T) (warp logits (G, B, T)); the
per-channel vectors are (F,).  Options follow the reference's 12-tuple
(selective.py:249-262): (has_gamma, has_warp, has_write, log_shift,
gamma_scale, warp_scale, prospective, gamma_horizon, write_sigmoid,
write_max, write_bias, bound_warp).
"""

from __future__ import annotations

import numpy as np


def _sig(x):
    return 0.5 * (1.0 + np.tanh(0.5 * x))


def _phi_and_dphi(a):
    """phi(a) = (e^a - 1)/a and phi'(a) = (e^a - phi)/a, accurate near 0."""
    ar, ai = a.real, a.imag
    em1 = np.expm1(ar) * np.cos(ai) - 2.0 * np.sin(0.5 * ai) ** 2 + 1j * np.exp(ar) * np.sin(ai)
    A = np.exp(a)
    small = np.abs(a) < 1e-3
    safe = np.where(small, 1.0, a)
    phi = np.where(small, 1 + a / 2 + a ** 2 / 6 + a ** 3 / 24 + a ** 4 / 120 + a ** 5 / 720,
                   em1 / safe)
    dphi = np.where(small, 0.5 + a / 3 + a ** 2 / 8 + a ** 3 / 30 + a ** 4 / 144,
                    (A - phi) / safe)
    return A, phi, dphi


def controllers(gl, dl, wl, bias, theta, groups, lo, span, step, opt, th_lo, th_hi, shape):
    """Per-element gamma, theta, gate and the link intermediates; shape is
    (F, B, T)."""
    (has_gamma, has_warp, has_write, log_shift, g_scale, w_scale, _pros, _gh, w_sig, w_max,
     w_bias, bound) = opt
    b = bias[:, None, None]
    aux = {}
    if has_gamma:
        if log_shift:
            s = np.tanh(gl)
            gamma = np.exp(b + g_scale * s)
        else:
            s = _sig(b + gl)
            gamma = lo[:, None, None] + span[:, None, None] * s
        aux["sig"] = s
    else:
        gamma = np.broadcast_to(b, shape).copy()
    th0 = np.broadcast_to(theta[:, None, None], shape).copy()
    if has_warp:
        warp = np.tanh(dl[groups])
        scale = np.exp(w_scale * warp)
        th_un = th0 * scale
        th = np.clip(th_un, th_lo[:, None, None], th_hi[:, None, None]) if bound else th_un
        aux.update(warp=warp, scale=scale, th_un=th_un)
    else:
        th = th0
    if has_write:
        gate = w_max * _sig(wl + w_bias) if w_sig else 1.0 + wl
    else:
        gate = np.ones(shape)
    h = np.broadcast_to(step[:, None, None], shape)
    return gamma, th, gate, h, aux


def options(raw) -> tuple:
    """The reference's 12-tuple from a numeric array (bools, floats)."""
    v = [float(x) for x in raw]
    b = [bool(round(x)) for x in v]
    return (b[0], b[1], b[2], b[3], v[4], v[5], b[6], b[7], b[8], v[9], v[10], b[11])


def forward(z, gl, dl, wl, bias, theta, groups, lo, span, step, horizon, th_lo, th_hi, opt):
    """Returns (raw y, coefficient dict)."""
    gamma, th, gate, h, aux = controllers(gl, dl, wl, bias, theta, groups, lo, span, step, opt,
                                          th_lo, th_hi, z.shape)
    prospective, gamma_horizon = opt[6], opt[7]
    a = -gamma * h + 1j * (1.0 - gamma) * th * h
    A, phi, dphi = _phi_and_dphi(a)
    p0 = gamma * h * phi
    n0 = np.zeros_like(p0)
    ratio = None
    if prospective:
        ratio = 1.0 / gamma if gamma_horizon else np.broadcast_to(horizon[:, None, None], a.shape)
        lag = ratio * gamma * A
        p0 = p0 + lag
        n0 = -lag
    p, n = gate * p0, gate * n0
    F, B, T = z.shape
    y = np.zeros(z.shape, np.complex128)
    prev = np.zeros((F, B), np.complex128)
    for t in range(T):
        u = p[..., t] * z[..., t]
        if t and prospective:
            u = u + n[..., t] * z[..., t - 1]
        prev = A[..., t] * prev + u
        y[..., t] = prev
    co = dict(gamma=gamma, th=th, gate=gate, h=h, a=a, A=A, phi=phi, dphi=dphi, p0=p0, n0=n0,
              p=p, n=n, ratio=ratio, aux=aux)
    return y, co


def backward(z, y, co, gy, gx, gl, dl, wl, bias, theta, groups, lo, span, step, horizon,
             th_lo, th_hi, opt, truncated, mask=None):
    """VJP of forward; gy/gx are the cotangents of raw / split-ReLU(raw) (or
    None).  Returns (dz, dzw, dG, dD_group, dW, dbias, dtheta) as the
    reference's selective_backward does (dzw is dz when not truncated).
    `mask` (bool, z.shape + (2,)) overrides the split-ReLU decisions."""
    (has_gamma, has_warp, has_write, log_shift, g_scale, w_scale, prospective, gamma_horizon,
     w_sig, w_max, _wb, bound) = opt
    F, B, T = z.shape
    e = np.zeros(z.shape, np.complex128)
    if gy is not None:
        e = e + gy
    if gx is not None:
        mr, mi = (y.real > 0, y.imag > 0) if mask is None else (mask[..., 0], mask[..., 1])
        e = e + np.where(mr, gx.real, 0.0) + 1j * np.where(mi, gx.imag, 0.0)
    A, p, n = co["A"], co["p"], co["n"]
    d = np.zeros(z.shape, np.complex128)
    nxt = np.zeros((F, B), np.complex128)
    for t in range(T - 1, -1, -1):
        if truncated:
            d[..., t] = e[..., t]
        else:
            nxt = e[..., t] + (np.conj(A[..., t + 1]) * nxt if t + 1 < T else 0.0)
            d[..., t] = nxt
    dz = np.conj(p) * d
    dzw = dz.copy()
    if prospective:
        dzw[..., :-1] += np.conj(n[..., 1:]) * d[..., 1:]
    zprev = np.concatenate([np.zeros((F, B, 1), np.complex128), z[..., :-1]], axis=-1)
    yprev = np.concatenate([np.zeros((F, B, 1), np.complex128), y[..., :-1]], axis=-1)
    dp = np.conj(z) * d        # cotangent of gated p
    dn = np.conj(zprev) * d    # cotangent of gated n
    dA = np.conj(yprev) * d
    gamma, th, gate, h = co["gamma"], co["th"], co["gate"], co["h"]
    p0, n0, a, phi, dphi = co["p0"], co["n0"], co["a"], co["phi"], co["dphi"]
    dgate = (np.conj(p0) * dp).real + (np.conj(n0) * dn).real
    dp0, dn0 = gate * dp, gate * dn
    dgam = (np.conj(h * phi) * dp0).real
    if prospective:
        q = dp0 - dn0
        ratio = co["ratio"]
        dA = dA + ratio * gamma * q
        if not gamma_horizon:
            dgam = dgam + (np.conj(ratio * A) * q).real
    da = np.conj(A) * dA + np.conj(dphi) * (gamma * h * dp0)
    dgam = dgam - h * (da.real + th * da.imag)
    dth = (1.0 - gamma) * h * da.imag
    aux = co["aux"]
    dG = None
    if has_gamma:
        s = aux["sig"]
        if log_shift:
            dbias_e = dgam * gamma
            dG = dbias_e * g_scale * (1.0 - s * s)
        else:
            dbias_e = dgam * span[:, None, None] * s * (1.0 - s)
            dG = dbias_e
    else:
        dbias_e = dgam
    dDg = None
    if has_warp:
        if bound:
            inside = (aux["th_un"] >= th_lo[:, None, None]) & (aux["th_un"] <= th_hi[:, None, None])
            dth = np.where(inside, dth, 0.0)
        dD = dth * aux["th_un"] * w_scale * (1.0 - aux["warp"] ** 2)
        dtheta_e = dth * aux["scale"]
        G = dl.shape[0]
        dDg = np.zeros((G, B, T))
        for f in range(F):
            dDg[groups[f]] += dD[f]
    else:
        dtheta_e = dth
    dW = None
    if has_write:
        dW = dgate * gate * (1.0 - gate / w_max) if w_sig else dgate
    dbias = dbias_e.sum(axis=(1, 2))
    dtheta = dtheta_e.sum(axis=(1, 2))
    # Full BPTT: z feeds both taps, so its cotangent is the total (dz and dzw
    # are the same tensor, selective_scan_kernel.py:521); TBPTT(1): dz is the
    # spatial part for x, dzw the total for the weight.
    if truncated:
        return dz, dzw, dG, dDg, dW, dbias, dtheta
    return dzw, dzw, dG, dDg, dW, dbias, dtheta
