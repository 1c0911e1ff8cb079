// ZOH prospective two-tap coefficients of the log-space RQF leaves (tau mode,
// rho = 1; rqf_models/backbones/rqf/filter.py:510-664) and their gradient,
// one thread per leaf, in double precision:
//
//   gamma = e^lg, theta = e^lt, s = dt / tau,
//   a = s (-gamma + i theta (1 - gamma)),   C1 = e^a,
//   phi(a) = (e^a - 1) / a  (4th-order Taylor below |a| = 1e-4, as the
//   reference),   tap0 = gamma (s phi(a) + C1),   tap1 = -gamma C1.
//
// Backward: for real leaves p and complex cotangents G (torch's convention),
// grad p = sum over the outputs y of Re(conj(dy/dp) G_y), with
// da/dlg = s (-gamma - i theta gamma), da/dlt = i s theta (1 - gamma) and
// phi'(a) = (e^a (a - 1) + 1) / a^2 (Taylor 1/2 + a/3 + a^2/8 + a^3/30 below
// the same threshold).  The torch restatement of the same formulas runs ~30
// small kernels forward and ~60 backward for these few thousand leaves.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rqf {
namespace coef {

struct cd {
  double x, y;
};
__device__ __forceinline__ cd cadd(cd a, cd b) { return {a.x + b.x, a.y + b.y}; }
__device__ __forceinline__ cd cmul(cd a, cd b) { return {a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x}; }
__device__ __forceinline__ cd cscale(cd a, double s) { return {a.x * s, a.y * s}; }
__device__ __forceinline__ cd cdiv(cd a, cd b) {
  const double d = b.x * b.x + b.y * b.y;
  return {(a.x * b.x + a.y * b.y) / d, (a.y * b.x - a.x * b.y) / d};
}
__device__ __forceinline__ cd cexp(cd a) {
  double sn, cs;
  sincos(a.y, &sn, &cs);
  const double m = exp(a.x);
  return {m * cs, m * sn};
}
// Re(conj(u) g)
__device__ __forceinline__ double rdot(cd u, float2 g) { return u.x * g.x + u.y * g.y; }

constexpr double kSmall = 1e-4;

struct Eval {
  double gamma, theta;
  cd a, ea, phi;
};

__device__ __forceinline__ Eval eval(float lt, float lg, double s) {
  Eval e;
  e.gamma = exp((double)lg);
  e.theta = exp((double)lt);
  e.a = {-s * e.gamma, s * e.theta * (1.0 - e.gamma)};
  e.ea = cexp(e.a);
  if (sqrt(e.a.x * e.a.x + e.a.y * e.a.y) < kSmall) {
    const cd a = e.a, a2 = cmul(a, a), a3 = cmul(a2, a), a4 = cmul(a3, a);
    e.phi = cadd(cadd({1.0 + a.x / 2, a.y / 2}, cscale(a2, 1.0 / 6)),
                 cadd(cscale(a3, 1.0 / 24), cscale(a4, 1.0 / 120)));
  } else {
    e.phi = cdiv({e.ea.x - 1.0, e.ea.y}, e.a);
  }
  return e;
}

__global__ void two_tap_kernel(const float *__restrict__ lt, const float *__restrict__ lg,
                               float2 *__restrict__ c1, float2 *__restrict__ tap0,
                               float2 *__restrict__ tap1, long long n, double s) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const Eval e = eval(lt[i], lg[i], s);
  const cd t0 = cscale(cadd(cscale(e.phi, s), e.ea), e.gamma);
  c1[i] = make_float2((float)e.ea.x, (float)e.ea.y);
  tap0[i] = make_float2((float)t0.x, (float)t0.y);
  tap1[i] = make_float2((float)(-e.gamma * e.ea.x), (float)(-e.gamma * e.ea.y));
}

// Cotangents may be null (zero).
__global__ void two_tap_backward_kernel(const float *__restrict__ lt, const float *__restrict__ lg,
                                        const float2 *__restrict__ g1, const float2 *__restrict__ g0,
                                        const float2 *__restrict__ gm, float *__restrict__ grad_lt,
                                        float *__restrict__ grad_lg, long long n, double s) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const Eval e = eval(lt[i], lg[i], s);
  cd dphi;
  if (sqrt(e.a.x * e.a.x + e.a.y * e.a.y) < kSmall) {
    const cd a = e.a, a2 = cmul(a, a), a3 = cmul(a2, a);
    dphi = cadd(cadd({0.5 + a.x / 3, a.y / 3}, cscale(a2, 1.0 / 8)), cscale(a3, 1.0 / 30));
  } else {
    const cd num = cadd(cmul(e.ea, {e.a.x - 1.0, e.a.y}), {1.0, 0.0});
    dphi = cdiv(num, cmul(e.a, e.a));
  }
  const float2 z = make_float2(0.f, 0.f);
  const float2 G1 = g1 ? g1[i] : z, G0 = g0 ? g0[i] : z, Gm = gm ? gm[i] : z;
  const cd sphi_c1 = cadd(cscale(e.phi, s), e.ea);    // s phi + C1
  const cd sdphi_c1 = cadd(cscale(dphi, s), e.ea);    // s phi' + C1
  // p = lg: dgamma/dp = gamma; p = lt: 0
  const cd da_lg = {-s * e.gamma, -s * e.theta * e.gamma};
  const cd da_lt = {0.0, s * e.theta * (1.0 - e.gamma)};
  double out[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const cd da = p == 0 ? da_lg : da_lt;
    const double dg = p == 0 ? e.gamma : 0.0;
    const cd dc1 = cmul(e.ea, da);
    const cd dt0 = cadd(cscale(sphi_c1, dg), cscale(cmul(sdphi_c1, da), e.gamma));
    const cd dt1 = cadd(cscale(e.ea, -dg), cscale(cmul(e.ea, da), -e.gamma));
    out[p] = rdot(dc1, G1) + rdot(dt0, G0) + rdot(dt1, Gm);
  }
  grad_lg[i] = (float)out[0];
  grad_lt[i] = (float)out[1];
}

}  // namespace coef
}  // namespace rqf
