// Two-tap coefficients of the RQF filter bank and their gradient
// (rqf_models/backbones/rqf/filter.py:RQF.compute_two_tap_coefficients
// :510-664, with the parameter reads of :402-449 and the dynamic gamma clamp
// of :594-598), one thread per filter, in double precision.
//
// Per filter, from its leaves (log space: log_theta, log_gamma; sigmoid space:
// freq_param, gamma_param with per-filter bounds) and log_tau:
//
//   tau = e^log_tau
//   log space:     gamma = e^lg,  freq = e^lt / (2 pi tau)
//   sigmoid space: gamma = gmin + (gmax - gmin) sig(gp),
//                  freq  = fmin + (fmax - fmin) sig(fp)
//   clamp_gamma:   gamma = clamp(gamma, 1 - 1/sqrt(1 + x^2), x / (1 + x)),
//                  x = 2 pi freq tau
//   rho = tau_p / tau (prospective_tau given), else 1 (tau mode) or
//         1 / gamma (gamma mode)
//   A = -gamma/tau + i 2 pi freq (1 - gamma),  a = A dt,  eta = dt / tau
//   Euler: C1 = 1 + eta (-1 + (1 - gamma)(1 + i 2 pi tau freq)),
//          tap0 = gamma eta + gamma rho,  tap1 = -gamma rho
//   ZOH:   C1 = e^a, phi = (e^a - 1)/a, tap0 = gamma eta phi + gamma rho C1,
//          tap1 = -gamma rho C1
//   FOH:   psi = (e^a - 1 - a)/a^2;  prospective: tap0 = gamma eta psi +
//          gamma rho phi, tap1 = gamma eta (phi - psi) - gamma rho phi;
//          non-prospective: tap0 = gamma eta psi, tap1 = gamma eta (phi - psi)
//
// phi and psi take the reference's 4th-order Taylor forms below |a| = 1e-4 and
// 1e-3.  The gradient carries forward-mode derivatives (Dual) through exactly
// the expressions above, one leaf at a time, so every branch — including the
// Taylor forms and the clamp, whose derivative follows the selected operand as
// torch.clamp's does — is differentiated without a hand-derived formula:
// grad p = sum over the outputs y of Re(conj(dy/dp) G_y) for complex
// cotangents G (torch's convention).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rqf {
namespace coef {

constexpr double kTwoPi = 6.283185307179586476925286766559;

// Value and derivative with respect to the seeded leaf.
struct Dual {
  double v, d;
};
__device__ __forceinline__ Dual operator+(Dual a, Dual b) { return {a.v + b.v, a.d + b.d}; }
__device__ __forceinline__ Dual operator-(Dual a, Dual b) { return {a.v - b.v, a.d - b.d}; }
__device__ __forceinline__ Dual operator-(Dual a) { return {-a.v, -a.d}; }
__device__ __forceinline__ Dual operator*(Dual a, Dual b) { return {a.v * b.v, a.d * b.v + a.v * b.d}; }
__device__ __forceinline__ Dual operator/(Dual a, Dual b) {
  return {a.v / b.v, (a.d * b.v - a.v * b.d) / (b.v * b.v)};
}
__device__ __forceinline__ Dual operator+(Dual a, double b) { return {a.v + b, a.d}; }
__device__ __forceinline__ Dual operator+(double a, Dual b) { return {a + b.v, b.d}; }
__device__ __forceinline__ Dual operator-(Dual a, double b) { return {a.v - b, a.d}; }
__device__ __forceinline__ Dual operator-(double a, Dual b) { return {a - b.v, -b.d}; }
__device__ __forceinline__ Dual operator*(Dual a, double b) { return {a.v * b, a.d * b}; }
__device__ __forceinline__ Dual operator*(double a, Dual b) { return {a * b.v, a * b.d}; }
__device__ __forceinline__ Dual operator/(Dual a, double b) { return {a.v / b, a.d / b}; }
__device__ __forceinline__ Dual operator/(double a, Dual b) { return {a / b.v, -a * b.d / (b.v * b.v)}; }

__device__ __forceinline__ double val(double x) { return x; }
__device__ __forceinline__ double val(Dual x) { return x.v; }
__device__ __forceinline__ double fexp(double x) { return exp(x); }
__device__ __forceinline__ Dual fexp(Dual x) {
  const double e = exp(x.v);
  return {e, e * x.d};
}
__device__ __forceinline__ double fsqrt(double x) { return sqrt(x); }
__device__ __forceinline__ Dual fsqrt(Dual x) {
  const double s = sqrt(x.v);
  return {s, x.d / (2.0 * s)};
}
__device__ __forceinline__ void fsincos(double x, double *s, double *c) { sincos(x, s, c); }
__device__ __forceinline__ void fsincos(Dual x, Dual *s, Dual *c) {
  double sn, cs;
  sincos(x.v, &sn, &cs);
  *s = {sn, cs * x.d};
  *c = {cs, -sn * x.d};
}
__device__ __forceinline__ double fsigmoid(double x) { return 1.0 / (1.0 + exp(-x)); }
__device__ __forceinline__ Dual fsigmoid(Dual x) {
  const double s = 1.0 / (1.0 + exp(-x.v));
  return {s, s * (1.0 - s) * x.d};
}
// A leaf read as S: the seeded leaf carries derivative 1.
template <class S>
__device__ __forceinline__ S leaf(double x, bool seeded);
template <>
__device__ __forceinline__ double leaf<double>(double x, bool) { return x; }
template <>
__device__ __forceinline__ Dual leaf<Dual>(double x, bool seeded) { return {x, seeded ? 1.0 : 0.0}; }

template <class S>
struct Cx {
  S re, im;
};
template <class S>
__device__ __forceinline__ Cx<S> operator+(Cx<S> a, Cx<S> b) { return {a.re + b.re, a.im + b.im}; }
template <class S>
__device__ __forceinline__ Cx<S> operator-(Cx<S> a, Cx<S> b) { return {a.re - b.re, a.im - b.im}; }
template <class S>
__device__ __forceinline__ Cx<S> operator*(Cx<S> a, Cx<S> b) {
  return {a.re * b.re - a.im * b.im, a.re * b.im + a.im * b.re};
}
template <class S>
__device__ __forceinline__ Cx<S> operator/(Cx<S> a, Cx<S> b) {
  const S d = b.re * b.re + b.im * b.im;
  return {(a.re * b.re + a.im * b.im) / d, (a.im * b.re - a.re * b.im) / d};
}
template <class S>
__device__ __forceinline__ Cx<S> scale(Cx<S> a, S s) { return {a.re * s, a.im * s}; }
__device__ __forceinline__ Cx<Dual> scale(Cx<Dual> a, double s) { return {a.re * s, a.im * s}; }
template <class S>
__device__ __forceinline__ Cx<S> cexp(Cx<S> a) {
  const S m = fexp(a.re);
  S sn, cs;
  fsincos(a.im, &sn, &cs);
  return {m * cs, m * sn};
}
template <class S>
__device__ __forceinline__ double cabs_v(Cx<S> a) {
  const double x = val(a.re), y = val(a.im);
  return sqrt(x * x + y * y);
}
template <class S>
__device__ __forceinline__ Cx<S> cplus(Cx<S> a, double r) { return {a.re + r, a.im}; }

enum : int { kEuler = 0, kZoh = 1, kFoh = 2 };

// Host-filled, passed by value.  Null bound / tau_p / log_tau pointers fall
// back to the scalars below (`tau`) or are unused.
struct Leaves {
  const float *theta;   // log_theta (log space) or freq_param (sigmoid space)
  const float *gamma;   // log_gamma or gamma_param
  const float *log_tau; // per filter; null: log(tau)
  const float *min_gamma, *max_gamma, *min_freq, *max_freq;  // sigmoid space
  const float *tau_p;   // prospective_tau (seconds) per filter, or null
};
struct Opts {
  int disc, prospective, gamma_mode, sigmoid, clamp;
  double dt, tau;
};

// seed: 0 theta leaf, 1 gamma leaf, 2 log_tau, 3 tau_p, -1 none.
template <class S>
__device__ __forceinline__ void eval(const Leaves &L, const Opts &o, long long i, int seed,
                                     Cx<S> *c1, Cx<S> *t0, Cx<S> *t1) {
  const S log_tau = leaf<S>(L.log_tau ? (double)L.log_tau[i] : log(o.tau), seed == 2);
  const S tau = fexp(log_tau);
  S gamma, freq;
  if (!o.sigmoid) {
    gamma = fexp(leaf<S>((double)L.gamma[i], seed == 1));
    freq = fexp(leaf<S>((double)L.theta[i], seed == 0)) / (kTwoPi * tau);
  } else {
    const double g0 = L.min_gamma[i], g1 = L.max_gamma[i];
    const double f0 = L.min_freq[i], f1 = L.max_freq[i];
    gamma = g0 + (g1 - g0) * fsigmoid(leaf<S>((double)L.gamma[i], seed == 1));
    freq = f0 + (f1 - f0) * fsigmoid(leaf<S>((double)L.theta[i], seed == 0));
  }
  if (o.clamp) {  // torch.clamp(gamma, min=lo, max=hi) = min(max(gamma, lo), hi)
    const S x = kTwoPi * freq * tau;
    const S lo = 1.0 - 1.0 / fsqrt(1.0 + x * x);
    const S hi = x / (1.0 + x);
    S r = val(gamma) < val(lo) ? lo : gamma;
    gamma = val(r) > val(hi) ? hi : r;
  }
  S rho;
  if (L.tau_p)
    rho = leaf<S>((double)L.tau_p[i], seed == 3) / tau;
  else
    rho = o.gamma_mode ? 1.0 / gamma : leaf<S>(1.0, false);
  const S eta = o.dt / tau;
  const S one_m_g = 1.0 - gamma;
  if (o.disc == kEuler) {
    const S extra = gamma * rho;
    *c1 = {1.0 + eta * (one_m_g - 1.0), eta * one_m_g * (kTwoPi * tau * freq)};
    *t0 = {gamma * eta + extra, leaf<S>(0.0, false)};
    *t1 = {-extra, leaf<S>(0.0, false)};
    return;
  }
  const Cx<S> a = {-(gamma / tau) * o.dt, kTwoPi * freq * one_m_g * o.dt};
  const Cx<S> ea = cexp(a);
  const double mag = cabs_v(a);
  Cx<S> phi;
  if (mag < 1e-4) {
    const Cx<S> a2 = a * a, a3 = a2 * a, a4 = a3 * a;
    phi = cplus(scale(a, 0.5), 1.0) + scale(a2, 1.0 / 6) + scale(a3, 1.0 / 24) +
          scale(a4, 1.0 / 120);
  } else {
    phi = cplus(ea, -1.0) / a;
  }
  *c1 = ea;
  if (o.disc == kZoh) {
    const Cx<S> extra = scale(ea, gamma * rho);
    *t0 = scale(phi, gamma * eta) + extra;
    *t1 = {-extra.re, -extra.im};
    return;
  }
  Cx<S> psi;
  if (mag < 1e-3) {
    const Cx<S> a2 = a * a, a3 = a2 * a, a4 = a3 * a;
    psi = cplus(scale(a, 1.0 / 6), 0.5) + scale(a2, 1.0 / 24) + scale(a3, 1.0 / 120) +
          scale(a4, 1.0 / 720);
  } else {
    psi = (cplus(ea, -1.0) - a) / (a * a);
  }
  const Cx<S> d0 = scale(psi, gamma * eta);           // gamma D_bar
  const Cx<S> d1 = scale(phi - psi, gamma * eta);     // gamma (B_bar - D_bar)
  if (o.prospective) {
    const Cx<S> extra = scale(phi, gamma * rho);
    *t0 = d0 + extra;
    *t1 = d1 - extra;
  } else {
    *t0 = d0;
    *t1 = d1;
  }
}

__global__ void two_tap_kernel(Leaves L, Opts o, float2 *__restrict__ c1, float2 *__restrict__ tap0,
                               float2 *__restrict__ tap1, long long n) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  Cx<double> c, t0, t1;
  eval<double>(L, o, i, -1, &c, &t0, &t1);
  c1[i] = make_float2((float)c.re, (float)c.im);
  tap0[i] = make_float2((float)t0.re, (float)t0.im);
  tap1[i] = make_float2((float)t1.re, (float)t1.im);
}

// Re(conj(dy) g): the derivative parts of a dual complex against a cotangent.
__device__ __forceinline__ double rdot(Cx<Dual> u, float2 g) { return u.re.d * g.x + u.im.d * g.y; }

// Cotangents may be null (zero); so may any gradient output (not wanted).
__global__ void two_tap_backward_kernel(Leaves L, Opts o, const float2 *__restrict__ g1,
                                        const float2 *__restrict__ g0,
                                        const float2 *__restrict__ gm, float *__restrict__ grad_theta,
                                        float *__restrict__ grad_gamma,
                                        float *__restrict__ grad_log_tau,
                                        float *__restrict__ grad_tau_p, long long n) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float2 z = make_float2(0.f, 0.f);
  const float2 G1 = g1 ? g1[i] : z, G0 = g0 ? g0[i] : z, Gm = gm ? gm[i] : z;
  float *outs[4] = {grad_theta, grad_gamma, grad_log_tau, grad_tau_p};
#pragma unroll 1
  for (int p = 0; p < 4; ++p) {
    if (!outs[p]) continue;
    Cx<Dual> c, t0, t1;
    eval<Dual>(L, o, i, p, &c, &t0, &t1);
    outs[p][i] = (float)(rdot(c, G1) + rdot(t0, G0) + rdot(t1, Gm));
  }
}

}  // namespace coef
}  // namespace rqf
