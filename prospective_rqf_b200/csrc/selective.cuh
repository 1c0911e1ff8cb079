// Selective (input-dependent ZOH) RQF scan in (F,B,T) layout.
//
// Per sample t of row (f, b) (rqf_models/ops/selective_scan.py:
// selective_coefficients :26-68, reference_layer_scan :71-104):
//   controllers  gamma = bias                         (no gamma control)
//                      | lo + span * sigmoid(bias + G)   (sigmoid link)
//                      | exp(bias + gscale * tanh(G))    (log-shift link)
//                theta = Theta * exp(wscale * tanh(D[group(f)])), clamped to the
//                        band when bounded
//                gate  = wmax * sigmoid(W + wbias)  |  1 + W  |  1
//   ZOH          a = (-gamma + i (1-gamma) theta) * h,  A = e^a,
//                phi = (e^a - 1)/a,  p0 = gamma h phi
//   prospective  lag = ratio * gamma * A,  p0 += lag,  n0 = -lag
//                (ratio = 1/gamma in gamma-horizon mode, else horizon[f])
//   recurrence   y[t] = A[t] y[t-1] + gate (p0 z[t] + n0 z[t-1])
//
// Work decomposition: persistent CTAs each walk whole rows tile by tile
// (1024 samples, 4 per thread) with the carry on chip.  The in-tile scan
// composes time-varying (A, u) pairs (warp shuffles + shared memory).  The
// backward replays the controllers and the forward states of a tile from its
// stored entry state, runs the reverse adjoint d[t] = e[t] + conj(A[t+1])
// d[t+1] (skipped for TBPTT(1)), and fuses the whole coefficient VJP: dz, dzw,
// the gamma / write logit cotangents, the per-channel warp cotangent (group-
// reduced afterwards in fixed order) and per-row sums for bias and theta.
// The reference recomputes the same quantities in its Triton _backward
// (selective_scan_kernel.py:250-462) with one program per row.
#pragma once

#include <cuda_bf16.h>

#include "rqf_common.cuh"

namespace rqf {

struct SelOptions {  // layout of rqf_selective_options in include/rqf_b200.h
  int has_gamma, has_warp, has_write, log_shift;
  float gamma_scale, warp_scale;
  int prospective, gamma_horizon, write_sigmoid;
  float write_max, write_bias;
  int bound_warp;
};

// Storage of the logits, their cotangents and the raw / act outputs: fp32
// (complex64 outputs), or bf16 in the bf16 storage mode (complex outputs as
// interleaved bf16 pairs).  The drive z, the output cotangents, dz / dzw and
// every value computed in the kernels stay fp32.
struct SelArgs {
  const float2 *z;
  const void *G, *D, *W;  // logits (F,B,T), (groups,B,T), (F,B,T); null when unused
  const float *bias, *theta, *lo, *span, *step, *horizon, *th_lo, *th_hi;  // (F,)
  const long long *groups;                                                  // (F,)
  void *raw, *act;     // forward outputs (nullable)
  float2 *carries;     // (rows, ntiles) entry states
  const float2 *gy, *gx;
  float2 *dz, *dzw;
  void *dG, *dW;        // logit cotangents (F,B,T), the logits' storage type
  float *dD;            // per-channel (F,B,T) warp cotangent (fp32), group-reduced later
  float *partials;      // (rows, 2): bias and theta sums
  int rows, T, batch, ntiles, num_groups;
  SelOptions o;
  int truncated;
  int vec;  // T % 4 == 0 and every per-sample tensor 16-byte aligned: 16-byte accesses
};

constexpr int kSelThreads = 256;
constexpr int kSelK = 4;
constexpr int kSelTile = kSelThreads * kSelK;  // 1024 samples

struct SelChan {
  float bias, theta, lo, span, h, horizon, th_lo, th_hi;
  int group;
};

struct SelCtl {
  float g, th, gate, sig, warp, scale;
};

struct SelCoef {
  float2 a, A, phi, p0, n0;
  float ratio;
};

// Controller links on the hardware exponential (ex2-based __expf, ~2 ulp, as
// the reference's Triton tl.exp) and the 2-ulp reciprocal.  tanh comes from
// the identity tanh(x) = 1 - 2 / (e^{2x} + 1): absolute error ~1e-7, and the
// controllers only use it additively (exponents, 1 - tanh^2).
__device__ __forceinline__ float sel_rcp(float x) { return __fdividef(1.f, x); }
__device__ __forceinline__ float sel_sigmoid(float x) { return sel_rcp(1.f + __expf(-x)); }
__device__ __forceinline__ float sel_tanh(float x) {
  const float e = __expf(2.f * x);
  return e > 1e30f ? 1.f : fmaf(-2.f, sel_rcp(e + 1.f), 1.f);
}
// e^x - 1 without cancellation: the Maclaurin series through x^8/8! below
// |x| = 0.35 (truncation < 0.35^9/9! ~ 2e-10), e^x - 1 on __expf above (where
// e^x - 1 is at least 0.3 in magnitude, so no digits cancel).
__device__ __forceinline__ float sel_expm1(float x) {
  if (fabsf(x) < 0.35f) {
    float p = fmaf(x, 1.f / 40320.f, 1.f / 5040.f);
    p = fmaf(x, p, 1.f / 720.f);
    p = fmaf(x, p, 1.f / 120.f);
    p = fmaf(x, p, 1.f / 24.f);
    p = fmaf(x, p, 1.f / 6.f);
    p = fmaf(x, p, 0.5f);
    return fmaf(x * x, p, x);
  }
  return __expf(x) - 1.f;
}

// sin and cos of the ZOH half angle.  Below pi/4 (every practical step: the
// angle is (1 - gamma) theta h / 2) the Maclaurin series of sin and cos
// through x^9 and x^10 — truncation below x^11/11! < 2e-9 — evaluated in
// Horner form on x^2; larger angles take sincosf.
__device__ __forceinline__ void sel_sincos_half(float x, float &sn, float &cs) {
  if (fabsf(x) < 0.7853982f) {
    const float x2 = x * x;
    float ps = fmaf(x2, 1.f / 362880.f, -1.f / 5040.f);
    ps = fmaf(x2, ps, 1.f / 120.f);
    ps = fmaf(x2, ps, -1.f / 6.f);
    sn = fmaf(x * x2, ps, x);
    float pc = fmaf(x2, -1.f / 3628800.f, 1.f / 40320.f);
    pc = fmaf(x2, pc, -1.f / 720.f);
    pc = fmaf(x2, pc, 1.f / 24.f);
    pc = fmaf(x2, pc, -0.5f);
    cs = fmaf(x2, pc, 1.f);
  } else {
    sincosf(x, &sn, &cs);
  }
}

__device__ __forceinline__ SelChan sel_chan(const SelArgs &a, int f) {
  SelChan c;
  c.bias = a.bias[f];
  c.theta = a.theta[f];
  c.lo = a.lo[f];
  c.span = a.span[f];
  c.h = a.step[f];
  c.horizon = a.horizon[f];
  c.th_lo = a.th_lo[f];
  c.th_hi = a.th_hi[f];
  c.group = 0;
  if (a.o.has_warp) {
    const long long g = a.groups[f];
    if (g < 0 || g >= a.num_groups) {
      latch_error(5);  // RQF_ERR_ARGUMENT: warp group out of range (read clamped to group 0)
    } else {
      c.group = (int)g;
    }
  }
  return c;
}

__device__ __forceinline__ SelCtl sel_controller(const SelOptions &o, const SelChan &c, float gl,
                                                 float dl, float wl) {
  SelCtl r;
  r.sig = 0.f;
  r.warp = 0.f;
  r.scale = 1.f;
  r.g = c.bias;
  if (o.has_gamma) {
    if (o.log_shift) {
      r.sig = sel_tanh(gl);
      r.g = __expf(c.bias + o.gamma_scale * r.sig);
    } else {
      r.sig = sel_sigmoid(c.bias + gl);
      r.g = c.lo + c.span * r.sig;
    }
  }
  r.th = c.theta;
  if (o.has_warp) {
    r.warp = sel_tanh(dl);
    r.scale = __expf(o.warp_scale * r.warp);
    r.th = c.theta * r.scale;
    if (o.bound_warp) r.th = fminf(fmaxf(r.th, c.th_lo), c.th_hi);
  }
  r.gate = 1.f;
  if (o.has_write) r.gate = o.write_sigmoid ? o.write_max * sel_sigmoid(wl + o.write_bias) : 1.f + wl;
  return r;
}

__device__ __forceinline__ SelCoef sel_coef(const SelOptions &o, const SelChan &c,
                                            const SelCtl &k) {
  SelCoef r;
  const float ar = -k.g * c.h, ai = (1.f - k.g) * k.th * c.h;
  // half-angle sincos gives sin(ai), cos(ai) and the cancellation-free
  // 1 - cos(ai) = 2 sin^2(ai/2) from one evaluation
  float hs, hc;
  sel_sincos_half(0.5f * ai, hs, hc);
  const float sn = 2.f * hs * hc, one_m_cs = 2.f * hs * hs, cs = 1.f - one_m_cs;
  const float e = __expf(ar);
  r.a = make_float2(ar, ai);
  r.A = make_float2(e * cs, e * sn);
  const float den = ar * ar + ai * ai;
  if (den < 1e-8f) {  // exprel Taylor series near 0: 1 + a/2 + a^2/6 + a^3/24
    float2 s = c_fma(r.a, make_float2(1.f / 24.f, 0.f), make_float2(1.f / 6.f, 0.f));
    s = c_fma(r.a, s, make_float2(0.5f, 0.f));
    r.phi = c_fma(r.a, s, cone());
  } else {
    // e^a - 1 without cancellation: expm1(ar) cos(ai) - (1 - cos(ai)) + i e^ar sin(ai)
    const float er = sel_expm1(ar) * cs - one_m_cs, ei = r.A.y;
    const float inv = sel_rcp(den);
    r.phi = make_float2((er * ar + ei * ai) * inv, (ei * ar - er * ai) * inv);
  }
  const float gh = k.g * c.h;
  r.p0 = make_float2(gh * r.phi.x, gh * r.phi.y);
  r.n0 = cz();
  r.ratio = 0.f;
  if (o.prospective) {
    r.ratio = o.gamma_horizon ? sel_rcp(k.g) : c.horizon;
    const float rg = r.ratio * k.g;
    const float2 lag = make_float2(rg * r.A.x, rg * r.A.y);
    r.p0 = c_add(r.p0, lag);
    r.n0 = make_float2(-lag.x, -lag.y);
  }
  return r;
}

// exprel'(a) = (e^a - phi)/a with the Taylor series sum_k (k+1)/(k+2)! a^k
// below |a|^2 < 1/64 (8 terms) and its cubic truncation below 1e-8.
__device__ __forceinline__ float2 sel_dphi(float2 a, float2 A, float2 phi) {
  const float den = a.x * a.x + a.y * a.y;
  if (den < 1e-8f) {
    float2 s = c_fma(a, make_float2(1.f / 8.f, 0.f), make_float2(1.f / 3.f, 0.f));
    return c_fma(a, s, make_float2(0.5f, 0.f));
  }
  if (den < 0.015625f) {
    const float c[8] = {1.f / 45360.f, 1.f / 5760.f, 1.f / 840.f, 1.f / 144.f,
                        1.f / 30.f,    1.f / 8.f,    1.f / 3.f,   0.5f};
    float2 s = make_float2(c[0], 0.f);
#pragma unroll
    for (int i = 1; i < 8; ++i) s = c_fma(a, s, make_float2(c[i], 0.f));
    return s;
  }
  const float2 d = make_float2(A.x - phi.x, A.y - phi.y);
  const float inv = sel_rcp(den);
  return make_float2((d.x * a.x + d.y * a.y) * inv, (d.y * a.x - d.x * a.y) * inv);
}

// Per-thread groups of K = 4 consecutive samples [t0, t0 + 4) of one row:
// 16-byte accesses when `vec` and the group lies inside the row, element-wise
// (zero fill past T) otherwise.  Complex rows stream (read or written once).
static_assert(kSelK == 4, "the vector accesses below move 4 samples per thread");
__device__ __forceinline__ void sel_ld_f(const float *row, int t0, int T, bool vec,
                                         float (&v)[kSelK]) {
  if (row && vec && t0 + kSelK <= T) {
    const float4 q = __ldg(reinterpret_cast<const float4 *>(row + t0));
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    return;
  }
#pragma unroll
  for (int k = 0; k < kSelK; ++k) v[k] = (row && t0 + k < T) ? __ldg(row + t0 + k) : 0.f;
}
__device__ __forceinline__ void sel_ld_c(const float2 *row, int t0, int T, bool vec,
                                         float2 (&v)[kSelK]) {
  if (row && vec && t0 + kSelK <= T) {
    const float4 *q = reinterpret_cast<const float4 *>(row + t0);
    const float4 a = __ldcs(q), b = __ldcs(q + 1);
    v[0] = make_float2(a.x, a.y); v[1] = make_float2(a.z, a.w);
    v[2] = make_float2(b.x, b.y); v[3] = make_float2(b.z, b.w);
    return;
  }
#pragma unroll
  for (int k = 0; k < kSelK; ++k) v[k] = (row && t0 + k < T) ? __ldcs(row + t0 + k) : cz();
}
__device__ __forceinline__ void sel_st_c(float2 *row, int t0, int T, bool vec,
                                         const float2 (&v)[kSelK]) {
  if (vec && t0 + kSelK <= T) {
    float4 *q = reinterpret_cast<float4 *>(row + t0);
    __stcs(q, make_float4(v[0].x, v[0].y, v[1].x, v[1].y));
    __stcs(q + 1, make_float4(v[2].x, v[2].y, v[3].x, v[3].y));
    return;
  }
#pragma unroll
  for (int k = 0; k < kSelK; ++k)
    if (t0 + k < T) __stcs(row + t0 + k, v[k]);
}
__device__ __forceinline__ void sel_st_f(float *row, int t0, int T, bool vec,
                                         const float (&v)[kSelK]) {
  if (vec && t0 + kSelK <= T) {
    __stcs(reinterpret_cast<float4 *>(row + t0), make_float4(v[0], v[1], v[2], v[3]));
    return;
  }
#pragma unroll
  for (int k = 0; k < kSelK; ++k)
    if (t0 + k < T) __stcs(row + t0 + k, v[k]);
}
// The same accesses in the logits' storage type (fp32 or bf16) and for the
// complex outputs (complex64 or bf16 pairs).  bf16 values are widened exactly
// and written rounded to nearest-even.
template <bool BF>
__device__ __forceinline__ const void *sel_row(const void *base, size_t off) {
  return base ? static_cast<const char *>(base) + off * (BF ? 2 : 4) : nullptr;
}
template <bool BF>
__device__ __forceinline__ void *sel_row_out(void *base, size_t off, int per_sample) {
  return static_cast<char *>(base) + off * (size_t)per_sample * (BF ? 2 : 4);
}
__device__ __forceinline__ float bf_to_f(unsigned short u) {
  return __uint_as_float((unsigned)u << 16);
}
__device__ __forceinline__ unsigned short f_to_bf(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
template <bool BF>
__device__ __forceinline__ void sel_ld_l(const void *row, int t0, int T, bool vec,
                                         float (&v)[kSelK]) {
  if constexpr (!BF) {
    sel_ld_f(static_cast<const float *>(row), t0, T, vec, v);
  } else {
    const unsigned short *r = static_cast<const unsigned short *>(row);
    if (r && vec && t0 + kSelK <= T) {
      const uint2 q = __ldg(reinterpret_cast<const uint2 *>(r + t0));
      v[0] = __uint_as_float(q.x << 16); v[1] = __uint_as_float(q.x & 0xffff0000u);
      v[2] = __uint_as_float(q.y << 16); v[3] = __uint_as_float(q.y & 0xffff0000u);
      return;
    }
#pragma unroll
    for (int k = 0; k < kSelK; ++k) v[k] = (r && t0 + k < T) ? bf_to_f(__ldg(r + t0 + k)) : 0.f;
  }
}
template <bool BF>
__device__ __forceinline__ void sel_st_l(void *row, int t0, int T, bool vec,
                                         const float (&v)[kSelK]) {
  if constexpr (!BF) {
    sel_st_f(static_cast<float *>(row), t0, T, vec, v);
  } else {
    unsigned short *r = static_cast<unsigned short *>(row);
    if (vec && t0 + kSelK <= T) {
      const uint2 q = make_uint2((unsigned)f_to_bf(v[0]) | ((unsigned)f_to_bf(v[1]) << 16),
                                 (unsigned)f_to_bf(v[2]) | ((unsigned)f_to_bf(v[3]) << 16));
      __stcs(reinterpret_cast<uint2 *>(r + t0), q);
      return;
    }
#pragma unroll
    for (int k = 0; k < kSelK; ++k)
      if (t0 + k < T) r[t0 + k] = f_to_bf(v[k]);
  }
}
template <bool BF>
__device__ __forceinline__ void sel_st_out(void *row, int t0, int T, bool vec,
                                           const float2 (&v)[kSelK]) {
  if constexpr (!BF) {
    sel_st_c(static_cast<float2 *>(row), t0, T, vec, v);
  } else {
    unsigned *r = static_cast<unsigned *>(row);  // one bf16 pair per sample
    auto pack = [](float2 c) { return (unsigned)f_to_bf(c.x) | ((unsigned)f_to_bf(c.y) << 16); };
    if (vec && t0 + kSelK <= T) {
      __stcs(reinterpret_cast<uint4 *>(r + t0),
             make_uint4(pack(v[0]), pack(v[1]), pack(v[2]), pack(v[3])));
      return;
    }
#pragma unroll
    for (int k = 0; k < kSelK; ++k)
      if (t0 + k < T) r[t0 + k] = pack(v[k]);
  }
}

// z[t0 - 1]: the previous thread's last sample, from memory for lane 0.
__device__ __forceinline__ float2 sel_prev_z(const float2 *row, int t0, int T, float2 zlast,
                                             int lane) {
  float2 zp = shfl_up2(zlast, 1);
  if (lane == 0) zp = (t0 > 0 && t0 - 1 < T) ? row[t0 - 1] : cz();
  return zp;
}

// ------------------------------------------------------------ forward
template <int NT, int K, bool BF = false>
__global__ void __launch_bounds__(NT) sel_fwd_kernel(const SelArgs a) {
  constexpr int L = NT * K;
  __shared__ float4 s_warp[2][NT / 32];  // double-buffered across consecutive tiles
  const int tid = threadIdx.x;
  const int T = a.T;
  const bool vec = a.vec != 0;
  unsigned tcount = 0;
  for (int row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int f = row / a.batch, b = row - f * a.batch;
    const SelChan c = sel_chan(a, f);
    const float2 *zrow = a.z + (size_t)row * T;
    const void *grow = a.o.has_gamma ? sel_row<BF>(a.G, (size_t)row * T) : nullptr;
    const void *wrow = a.o.has_write ? sel_row<BF>(a.W, (size_t)row * T) : nullptr;
    const void *drow =
        a.o.has_warp ? sel_row<BF>(a.D, ((size_t)c.group * a.batch + b) * T) : nullptr;
    float2 carry = cz();
    for (int j = 0; j < a.ntiles; ++j, ++tcount) {
      const int t0 = j * L + tid * K;
      float2 z[K];
      sel_ld_c(zrow, t0, T, vec, z);
      const float2 zp = sel_prev_z(zrow, t0, T, z[K - 1], tid & 31);
      float gl[K], dl[K], wl[K];
      sel_ld_l<BF>(grow, t0, T, vec, gl);
      sel_ld_l<BF>(drow, t0, T, vec, dl);
      sel_ld_l<BF>(wrow, t0, T, vec, wl);
      float2 A[K], u[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const SelCtl ct = sel_controller(a.o, c, gl[k], dl[k], wl[k]);
        const SelCoef co = sel_coef(a.o, c, ct);
        const float2 p = make_float2(ct.gate * co.p0.x, ct.gate * co.p0.y);
        const float2 n = make_float2(ct.gate * co.n0.x, ct.gate * co.n0.y);
        const bool in = t0 + k < T;
        A[k] = in ? co.A : cz();
        u[k] = in ? c_fma(n, k > 0 ? z[k - 1] : zp, c_mul(p, z[k])) : cz();
      }
      float2 g = cone(), y = cz();
#pragma unroll
      for (int k = 0; k < K; ++k) {
        y = c_fma(A[k], y, u[k]);
        g = c_mul(A[k], g);
      }
      float2 e, At;
      cta_scan_pair_entry_fwd<NT>(g, y, carry, e, At, s_warp[tcount & 1]);
      if (tid == 0) a.carries[(size_t)row * a.ntiles + j] = carry;
      carry = At;
      float2 ys[K], acts[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        e = c_fma(A[k], e, u[k]);
        ys[k] = e;
        acts[k] = c_relu(e);
      }
      if (a.raw) sel_st_out<BF>(sel_row_out<BF>(a.raw, (size_t)row * T, 2), t0, T, vec, ys);
      if (a.act) sel_st_out<BF>(sel_row_out<BF>(a.act, (size_t)row * T, 2), t0, T, vec, acts);
    }
  }
}

// ------------------------------------------------------------ backward
template <int NT, int K, bool BF = false>
__global__ void __launch_bounds__(NT, 3) sel_bwd_kernel(const SelArgs a) {
  constexpr int NW = NT / 32, L = NT * K;
  __shared__ float4 s_warp_f[NW];
  __shared__ float4 s_warp_r[NW];
  __shared__ float4 s_first[NW + 1];  // (A, gated n) of each warp's first sample
  __shared__ float2 s_efirst[NW];     // e at each warp's first sample (TBPTT(1))
  __shared__ float s_red[2][NW];
  // Per-sample controller / ZOH values of the replay, reused by the VJP so the
  // transcendentals run once per sample: [field][k][thread] (conflict-free).
  constexpr int kStash = 10;  // A.re, A.im, phi.re, phi.im, g, th, gate, sig, warp, scale
  __shared__ float s_stash[kStash][K][NT];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = a.T;
  const bool prosp = a.o.prospective != 0;
  const bool vec = a.vec != 0;
  for (int row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int f = row / a.batch, b = row - f * a.batch;
    const SelChan c = sel_chan(a, f);
    const size_t roff = (size_t)row * T;
    const void *grow = a.o.has_gamma ? sel_row<BF>(a.G, roff) : nullptr;
    const void *wrow = a.o.has_write ? sel_row<BF>(a.W, roff) : nullptr;
    const void *drow =
        a.o.has_warp ? sel_row<BF>(a.D, ((size_t)c.group * a.batch + b) * T) : nullptr;
    float2 dcarry = cz();                   // d at the first sample of the next tile
    float2 A_next = cz(), n_next = cz();    // A, gated n at that sample (0 past T)
    float acc_bias = 0.f, acc_theta = 0.f;
    for (int jr = a.ntiles - 1; jr >= 0; --jr) {
      __syncthreads();  // shared slots of the previous tile are free
      const int t0 = jr * L + tid * K;
      if (jr > 0 && tid < 64) {
        // The tile processed next (the one before in time, whole inside the
        // row) into L2, one 128-byte line per thread and tensor, so its loads
        // do not wait on HBM when it starts.
        const size_t pt = roff + (size_t)(jr - 1) * L;
        const size_t lb = (size_t)tid * 128;
        auto pf = [](const void *p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); };
        pf(reinterpret_cast<const char *>(a.z + pt) + lb);
        if (a.gy) pf(reinterpret_cast<const char *>(a.gy + pt) + lb);
        if (a.gx) pf(reinterpret_cast<const char *>(a.gx + pt) + lb);
        constexpr int kLogitLines = L * (BF ? 2 : 4) / 128;
        if (tid < kLogitLines) {
          const size_t lo = (size_t)(jr - 1) * L * (BF ? 2 : 4) + lb;
          if (grow) pf(static_cast<const char *>(grow) + lo);
          if (wrow) pf(static_cast<const char *>(wrow) + lo);
          if (drow) pf(static_cast<const char *>(drow) + lo);
        }
      }
      float2 z[K], e[K];
      sel_ld_c(a.z + roff, t0, T, vec, z);
      const float2 zp = sel_prev_z(a.z + roff, t0, T, z[K - 1], lane);
      float gl[K], dl[K], wl[K];
      sel_ld_l<BF>(grow, t0, T, vec, gl);
      sel_ld_l<BF>(drow, t0, T, vec, dl);
      sel_ld_l<BF>(wrow, t0, T, vec, wl);
      float2 gyv[K], gxv[K];
      sel_ld_c(a.gy ? a.gy + roff : nullptr, t0, T, vec, gyv);
      sel_ld_c(a.gx ? a.gx + roff : nullptr, t0, T, vec, gxv);
      // forward replay of the tile from its stored entry state
      float2 A[K], nn[K], u[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const SelCtl ct = sel_controller(a.o, c, gl[k], dl[k], wl[k]);
        const SelCoef co = sel_coef(a.o, c, ct);
        const float2 p = make_float2(ct.gate * co.p0.x, ct.gate * co.p0.y);
        const bool in = t0 + k < T;
        nn[k] = in ? make_float2(ct.gate * co.n0.x, ct.gate * co.n0.y) : cz();
        A[k] = in ? co.A : cz();
        u[k] = in ? c_fma(nn[k], k > 0 ? z[k - 1] : zp, c_mul(p, z[k])) : cz();
        s_stash[0][k][tid] = co.A.x;
        s_stash[1][k][tid] = co.A.y;
        s_stash[2][k][tid] = co.phi.x;
        s_stash[3][k][tid] = co.phi.y;
        s_stash[4][k][tid] = ct.g;
        s_stash[5][k][tid] = ct.th;
        s_stash[6][k][tid] = ct.gate;
        s_stash[7][k][tid] = ct.sig;
        s_stash[8][k][tid] = ct.warp;
        s_stash[9][k][tid] = ct.scale;
      }
      float2 g = cone(), y = cz();
#pragma unroll
      for (int k = 0; k < K; ++k) {
        y = c_fma(A[k], y, u[k]);
        g = c_mul(A[k], g);
      }
      float2 ent, At;
      cta_scan_pair_entry_fwd<NT>(g, y, a.carries[(size_t)row * a.ntiles + jr], ent, At,
                                  s_warp_f);
      float2 yprev[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        yprev[k] = ent;
        ent = c_fma(A[k], ent, u[k]);
        float2 ek = gyv[k];  // zero past T
        if (a.gx) ek = c_add(ek, c_relu_mask(gxv[k], ent));
        e[k] = ek;
      }
      // neighbours: (A, n) of the sample after each thread's last one
      float2 An = make_float2(__shfl_down_sync(0xffffffffu, A[0].x, 1),
                              __shfl_down_sync(0xffffffffu, A[0].y, 1));
      float2 Nn = make_float2(__shfl_down_sync(0xffffffffu, nn[0].x, 1),
                              __shfl_down_sync(0xffffffffu, nn[0].y, 1));
      if (lane == 0) {
        s_first[warp] = make_float4(A[0].x, A[0].y, nn[0].x, nn[0].y);
        s_efirst[warp] = e[0];
      }
      if (tid == NT - 1) s_first[NW] = make_float4(A_next.x, A_next.y, n_next.x, n_next.y);
      __syncthreads();
      if (lane == 31) {
        const float4 q = s_first[warp + 1];
        An = make_float2(q.x, q.y);
        Nn = make_float2(q.z, q.w);
      }
      // reverse adjoint over the tile
      float2 dn;  // d at the sample after this thread's last one
      float2 dcarry_next;
      if (a.truncated) {  // no temporal adjoint: d = e
        dn = shfl_down2(e[0], 1);
        if (lane == 31) dn = warp + 1 < NW ? s_efirst[warp + 1] : dcarry;
        dcarry_next = s_efirst[0];
      } else {
        float2 gr = cone(), h = cz();
        float2 An_k = An;
#pragma unroll
        for (int k = K - 1; k >= 0; --k) {
          const float2 m = c_conj(An_k);
          h = c_fma(m, h, e[k]);
          gr = c_mul(m, gr);
          An_k = A[k];
        }
        float2 Art;
        cta_scan_pair_entry_rev<NT>(gr, h, dcarry, dn, Art, s_warp_r);
        dcarry_next = Art;
      }
      // per-sample coefficient VJP, in reverse order; results gathered per
      // thread and stored as 16-byte groups after the loop
      float2 dnext = dn, A1 = An, N1 = Nn;
      float2 o_dz[K], o_dzw[K];
      float o_dG[K], o_dD[K], o_dW[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        o_dz[k] = cz();
        o_dzw[k] = cz();
        o_dG[k] = 0.f;
        o_dD[k] = 0.f;
        o_dW[k] = 0.f;
      }
#pragma unroll
      for (int k = K - 1; k >= 0; --k) {
        const int t = t0 + k;
        const float2 d = a.truncated ? e[k] : c_fma(c_conj(A1), dnext, e[k]);
        if (t < T) {
          SelCtl ct;
          ct.g = s_stash[4][k][tid];
          ct.th = s_stash[5][k][tid];
          ct.gate = s_stash[6][k][tid];
          ct.sig = s_stash[7][k][tid];
          ct.warp = s_stash[8][k][tid];
          ct.scale = s_stash[9][k][tid];
          SelCoef co;
          co.A = make_float2(s_stash[0][k][tid], s_stash[1][k][tid]);
          co.phi = make_float2(s_stash[2][k][tid], s_stash[3][k][tid]);
          co.a = make_float2(-ct.g * c.h, (1.f - ct.g) * ct.th * c.h);
          const float gh0 = ct.g * c.h;
          co.p0 = make_float2(gh0 * co.phi.x, gh0 * co.phi.y);
          co.n0 = cz();
          co.ratio = 0.f;
          if (prosp) {
            co.ratio = a.o.gamma_horizon ? sel_rcp(ct.g) : c.horizon;
            const float rg = co.ratio * ct.g;
            co.p0 = make_float2(fmaf(rg, co.A.x, co.p0.x), fmaf(rg, co.A.y, co.p0.y));
            co.n0 = make_float2(-rg * co.A.x, -rg * co.A.y);
          }
          const float2 p = make_float2(ct.gate * co.p0.x, ct.gate * co.p0.y);
          const float2 dzs = c_cfma(p, d, cz());
          const float2 dzwv = prosp ? c_cfma(N1, dnext, dzs) : dzs;
          o_dz[k] = a.truncated ? dzs : dzwv;
          o_dzw[k] = dzwv;
          const float2 zk = z[k], zpk = k > 0 ? z[k - 1] : zp;
          const float2 dp = c_cfma(zk, d, cz());
          const float2 dnv = c_cfma(zpk, d, cz());
          float2 dA = c_cfma(yprev[k], d, cz());
          const float dgate =
              co.p0.x * dp.x + co.p0.y * dp.y + co.n0.x * dnv.x + co.n0.y * dnv.y;
          const float2 dp0 = make_float2(ct.gate * dp.x, ct.gate * dp.y);
          const float2 dn0 = make_float2(ct.gate * dnv.x, ct.gate * dnv.y);
          float dgam = c.h * (co.phi.x * dp0.x + co.phi.y * dp0.y);
          if (prosp) {
            const float2 q = make_float2(dp0.x - dn0.x, dp0.y - dn0.y);
            const float rg = co.ratio * ct.g;
            dA = make_float2(fmaf(rg, q.x, dA.x), fmaf(rg, q.y, dA.y));
            if (!a.o.gamma_horizon) dgam += co.ratio * (co.A.x * q.x + co.A.y * q.y);
          }
          const float2 dphi = sel_dphi(co.a, co.A, co.phi);
          const float gh = ct.g * c.h;
          const float2 da =
              c_cfma(dphi, make_float2(gh * dp0.x, gh * dp0.y), c_cfma(co.A, dA, cz()));
          dgam -= c.h * (da.x + ct.th * da.y);
          float dth = (1.f - ct.g) * c.h * da.y;
          float dbias_e = dgam;
          if (a.o.has_gamma) {
            if (a.o.log_shift) {
              dbias_e = dgam * ct.g;
              o_dG[k] = dbias_e * a.o.gamma_scale * (1.f - ct.sig * ct.sig);
            } else {
              dbias_e = dgam * c.span * ct.sig * (1.f - ct.sig);
              o_dG[k] = dbias_e;
            }
          }
          float dtheta_e = dth;
          if (a.o.has_warp) {
            if (a.o.bound_warp) {
              const float un = c.theta * ct.scale;
              dth = (un >= c.th_lo && un <= c.th_hi) ? dth : 0.f;
            }
            o_dD[k] = dth * ct.th * a.o.warp_scale * (1.f - ct.warp * ct.warp);
            dtheta_e = dth * ct.scale;
          }
          if (a.o.has_write)
            o_dW[k] =
                a.o.write_sigmoid ? dgate * ct.gate * (1.f - ct.gate / a.o.write_max) : dgate;
          acc_bias += dbias_e;
          acc_theta += dtheta_e;
        }
        dnext = d;
        A1 = A[k];
        N1 = nn[k];
      }
      sel_st_c(a.dz + roff, t0, T, vec, o_dz);
      if (a.truncated) sel_st_c(a.dzw + roff, t0, T, vec, o_dzw);
      if (a.o.has_gamma) sel_st_l<BF>(sel_row_out<BF>(a.dG, roff, 1), t0, T, vec, o_dG);
      if (a.o.has_warp) sel_st_f(a.dD + roff, t0, T, vec, o_dD);
      if (a.o.has_write) sel_st_l<BF>(sel_row_out<BF>(a.dW, roff, 1), t0, T, vec, o_dW);
      dcarry = dcarry_next;
      {
        const float4 q = s_first[0];
        A_next = make_float2(q.x, q.y);
        n_next = make_float2(q.z, q.w);
      }
    }
    // row finished: deterministic CTA reduction of the bias / theta sums
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc_bias += __shfl_xor_sync(0xffffffffu, acc_bias, o);
      acc_theta += __shfl_xor_sync(0xffffffffu, acc_theta, o);
    }
    __syncthreads();
    if (lane == 0) {
      s_red[0][warp] = acc_bias;
      s_red[1][warp] = acc_theta;
    }
    __syncthreads();
    if (tid < 2) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) s += s_red[tid][w];
      a.partials[(size_t)row * 2 + tid] = s;
    }
  }
}

// Channels ordered by warp group (stable in f) for the group reduction:
// order[bounds[g] .. bounds[g+1]) are the channels of group g in increasing f.
// One warp per group; channels with an out-of-range group (latched as an
// argument error by the backward kernel) are left out.  One block.
__global__ void __launch_bounds__(1024)
    sel_group_order_kernel(const long long *__restrict__ groups, int F, int ngroups,
                           int *__restrict__ order, int *__restrict__ bounds) {
  __shared__ int s_count[32];
  const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int count = 0;
  if (g < ngroups)
    for (int f0 = 0; f0 < F; f0 += 32) {
      const int f = f0 + lane;
      count += __popc(__ballot_sync(0xffffffffu, f < F && groups[f] == g));
    }
  if (lane == 0 && g < 32) s_count[g] = count;
  __syncthreads();
  int base = 0;
  for (int q = 0; q < g && q < ngroups; ++q) base += s_count[q];
  if (g < ngroups) {
    if (lane == 0) {
      bounds[g] = base;
      if (g == ngroups - 1) bounds[ngroups] = base + count;
    }
    for (int f0 = 0; f0 < F; f0 += 32) {
      const int f = f0 + lane;
      const bool in = f < F && groups[f] == g;
      const unsigned m = __ballot_sync(0xffffffffu, in);
      if (in) order[base + __popc(m & ((1u << lane) - 1u))] = f;
      base += __popc(m);
    }
  }
}

// dd_group[g, b, t] = sum of dD[f, b, t] over the channels f of group g, in
// increasing f (deterministic); one thread per (b, t), eight loads in flight.
template <bool BF = false>
__global__ void __launch_bounds__(256)
    sel_group_reduce_kernel(const float *__restrict__ dD, const int *__restrict__ order,
                            const int *__restrict__ bounds, void *__restrict__ out, int ngroups,
                            int64_t BT) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= BT) return;
  for (int g = 0; g < ngroups; ++g) {
    const int b0 = bounds[g], b1 = bounds[g + 1];
    float acc = 0.f;
    int q = b0;
    for (; q + 8 <= b1; q += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldcs(dD + (int64_t)order[q + u] * BT + i);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc += v[u];
    }
    for (; q < b1; ++q) acc += __ldcs(dD + (int64_t)order[q] * BT + i);
    if constexpr (BF)
      static_cast<unsigned short *>(out)[(int64_t)g * BT + i] = f_to_bf(acc);
    else
      static_cast<float *>(out)[(int64_t)g * BT + i] = acc;
  }
}

// dbias / dtheta from the per-row sums, summed in double over the batch.
__global__ void sel_param_reduce_kernel(const float *__restrict__ partials, float *dbias,
                                        float *dtheta, int F, int batch) {
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= F) return;
  double sb = 0.0, st = 0.0;
  for (int b = 0; b < batch; ++b) {
    sb += partials[((int64_t)f * batch + b) * 2];
    st += partials[((int64_t)f * batch + b) * 2 + 1];
  }
  dbias[f] = (float)sb;
  dtheta[f] = (float)st;
}

}  // namespace rqf
