/*
 * rqf_oracle.c — CPU restatement (double precision) of the RQF diagonal
 * complex scan family, used ONLY as the parity checker by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg.  It is not part
 * of the product and nothing in prospective_rqf_b200/ links or calls it.
 *
 * Parity is pinned: tests/test_oracle_golden.py checks these functions
 * against golden vectors produced by the reference implementation itself
 * (tests/golden/make_golden.py imports rqf_models from the reference tree).
 *
 * Restated algorithms (reference paths relative to the reference project):
 *   two-tap forward   y[t] = c1*y[t-1] + tap0*x[t] + tap1*x[t-1], y[-1]=x[-1]=0
 *       rqf_models/backbones/rqf/block.py:_apply_prospective_taps (:644-682)
 *       + rqf_models/ops/scan.py:_sequential_scan_cpu (:252-287).
 *       tap1 == NULL gives the single-tap scan y = c1*y + c2*u (tap0 = c2),
 *       scan.py:sequential_scan (:290-378).
 *   two-tap backward  reverse adjoint g[t] = gbar[t] + conj(c1) g[t+1],
 *       gx = conj(tap0) g[t] + conj(tap1) g[t+1],
 *       gc1 = sum conj(y[t-1]) g, gt0 = sum conj(x[t]) g, gt1 = sum conj(x[t-1]) g
 *       rqf_models/ops/chunked_scan_kernel.py:_chunked_scan_backward_kernel
 *       (:122-209) and :489-503; with the split-ReLU mask of
 *       rqf_models/ops/fbt_scan_kernel.py:180-185 when fuse_act.
 *   TBPTT(1) backward the pointwise autograd of the one-step rebuild
 *       rqf_models/backbones/rqf/block.py:_scan_two_tap_with_grad_mode
 *       (:938-954): gz = conj(tap0) g, gzw[t] = conj(tap1) g[t+1], sums as above.
 *
 * Layouts: 0 = BTF (dims d0=B, d1=T, d2=F), 1 = FBT (dims d0=F, d1=B, d2=T).
 * Complex arrays are interleaved double (complex128).  Rows run in parallel
 * (OpenMP); per-channel sums are reduced over rows in a fixed order.
 */
#include <complex.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef double complex cplx;

typedef struct {
  int64_t R, T, ts, B, F;
  int layout;
} rows_t;

static rows_t make_rows(int layout, int64_t d0, int64_t d1, int64_t d2) {
  rows_t r;
  r.layout = layout;
  if (layout == 0) { /* BTF */
    r.B = d0;
    r.T = d1;
    r.F = d2;
    r.ts = d2;
  } else { /* FBT */
    r.F = d0;
    r.B = d1;
    r.T = d2;
    r.ts = 1;
  }
  r.R = r.B * r.F;
  return r;
}

/* row index -> (offset of t=0, channel) */
static void row_info(const rows_t *r, int64_t row, int64_t *off, int64_t *ch) {
  if (r->layout == 0) {
    const int64_t b = row / r->F, f = row % r->F;
    *off = b * r->T * r->F + f;
    *ch = f;
  } else {
    *off = row * r->T;
    *ch = row / r->B;
  }
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
}

static inline cplx relu_c(cplx v) {
  const double re = creal(v) > 0 ? creal(v) : 0.0;
  const double im = cimag(v) > 0 ? cimag(v) : 0.0;
  return re + I * im;
}

static inline cplx mask_c(cplx g, cplx y) {
  const double re = creal(y) > 0 ? creal(g) : 0.0;
  const double im = cimag(y) > 0 ? cimag(g) : 0.0;
  return re + I * im;
}

int rqfo_two_tap_forward(int layout, int64_t d0, int64_t d1, int64_t d2, const cplx *c1,
                         const cplx *tap0, const cplx *tap1, const cplx *x, cplx *y,
                         int fuse_act, int nthreads) {
  const rows_t r = make_rows(layout, d0, d1, d2);
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t row = 0; row < r.R; ++row) {
    int64_t off, ch;
    row_info(&r, row, &off, &ch);
    const cplx lam = c1[ch], a0 = tap0[ch], a1 = tap1 ? tap1[ch] : 0.0;
    cplx state = 0.0, xprev = 0.0;
    for (int64_t t = 0; t < r.T; ++t) {
      const cplx xt = x[off + t * r.ts];
      state = lam * state + a0 * xt + a1 * xprev;
      xprev = xt;
      y[off + t * r.ts] = fuse_act ? relu_c(state) : state;
    }
  }
  return 0;
}

/* g_coef arrays: complex (F,).  When fuse_act and `mask` is non-NULL, the
 * split-ReLU derivative is taken from mask (2 bytes per element: Re, Im;
 * nonzero = active) instead of the sign of the recomputed state.  relu' is
 * discontinuous at 0, so checks of an fp32 kernel at millions of elements
 * pass the kernel's own forward decisions here and test separately that the
 * decisions differ only where the state is within rounding of 0. */
int rqfo_two_tap_backward_masked(int layout, int64_t d0, int64_t d1, int64_t d2, const cplx *c1,
                                 const cplx *tap0, const cplx *tap1, const cplx *x,
                                 const cplx *gy, int fuse_act, const unsigned char *mask,
                                 cplx *gx, cplx *gc1, cplx *gt0, cplx *gt1, int nthreads);

int rqfo_two_tap_backward(int layout, int64_t d0, int64_t d1, int64_t d2, const cplx *c1,
                          const cplx *tap0, const cplx *tap1, const cplx *x, const cplx *gy,
                          int fuse_act, cplx *gx, cplx *gc1, cplx *gt0, cplx *gt1,
                          int nthreads) {
  return rqfo_two_tap_backward_masked(layout, d0, d1, d2, c1, tap0, tap1, x, gy, fuse_act, NULL,
                                      gx, gc1, gt0, gt1, nthreads);
}

int rqfo_two_tap_backward_masked(int layout, int64_t d0, int64_t d1, int64_t d2, const cplx *c1,
                                 const cplx *tap0, const cplx *tap1, const cplx *x,
                                 const cplx *gy, int fuse_act, const unsigned char *mask,
                                 cplx *gx, cplx *gc1, cplx *gt0, cplx *gt1, int nthreads) {
  const rows_t r = make_rows(layout, d0, d1, d2);
  set_threads(nthreads);
  cplx *part = (cplx *)calloc((size_t)(r.R > 0 ? r.R : 1) * 3, sizeof(cplx));
  if (!part) return 1;
  int failed = 0;
#pragma omp parallel
  {
    cplx *ybuf = (cplx *)malloc((size_t)(r.T + 1) * sizeof(cplx));
    if (!ybuf) {
#pragma omp atomic write
      failed = 1;
    }
#pragma omp for schedule(dynamic, 4)
    for (int64_t row = 0; row < r.R; ++row) {
      if (!ybuf) continue;
      int64_t off, ch;
      row_info(&r, row, &off, &ch);
      const cplx lam = c1[ch], a0 = tap0[ch], a1 = tap1 ? tap1[ch] : 0.0;
      /* forward recompute: ybuf[t+1] = y[t], ybuf[0] = y[-1] = 0 */
      cplx state = 0.0, xprev = 0.0;
      ybuf[0] = 0.0;
      for (int64_t t = 0; t < r.T; ++t) {
        const cplx xt = x[off + t * r.ts];
        state = lam * state + a0 * xt + a1 * xprev;
        xprev = xt;
        ybuf[t + 1] = state;
      }
      cplx gnext = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
      for (int64_t t = r.T - 1; t >= 0; --t) {
        const cplx gt = gy[off + t * r.ts];
        cplx gbar = gt;
        if (fuse_act) {
          if (mask) {
            const unsigned char *m = mask + 2 * (off + t * r.ts);
            gbar = (m[0] ? creal(gt) : 0.0) + I * (m[1] ? cimag(gt) : 0.0);
          } else {
            gbar = mask_c(gt, ybuf[t + 1]);
          }
        }
        const cplx g = gbar + conj(lam) * gnext;
        const cplx xt = x[off + t * r.ts];
        const cplx xp = t > 0 ? x[off + (t - 1) * r.ts] : 0.0;
        gx[off + t * r.ts] = conj(a0) * g + conj(a1) * gnext;
        s1 += conj(ybuf[t]) * g;
        s2 += conj(xt) * g;
        s3 += conj(xp) * g;
        gnext = g;
      }
      part[row * 3 + 0] = s1;
      part[row * 3 + 1] = s2;
      part[row * 3 + 2] = s3;
    }
    free(ybuf);
  }
  if (failed) {
    free(part);
    return 1;
  }
  for (int64_t f = 0; f < r.F; ++f) {
    gc1[f] = 0.0;
    gt0[f] = 0.0;
    if (gt1) gt1[f] = 0.0;
  }
  for (int64_t row = 0; row < r.R; ++row) {
    int64_t off, ch;
    row_info(&r, row, &off, &ch);
    gc1[ch] += part[row * 3 + 0];
    gt0[ch] += part[row * 3 + 1];
    if (gt1) gt1[ch] += part[row * 3 + 2];
  }
  free(part);
  return 0;
}

int rqfo_tbptt_backward(int layout, int64_t d0, int64_t d1, int64_t d2, const cplx *c1,
                        const cplx *tap0, const cplx *tap1, const cplx *x, const cplx *gy,
                        int fuse_act, cplx *gz, cplx *gzw, cplx *gc1, cplx *gt0, cplx *gt1,
                        int nthreads) {
  const rows_t r = make_rows(layout, d0, d1, d2);
  set_threads(nthreads);
  cplx *part = (cplx *)calloc((size_t)(r.R > 0 ? r.R : 1) * 3, sizeof(cplx));
  if (!part) return 1;
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t row = 0; row < r.R; ++row) {
    int64_t off, ch;
    row_info(&r, row, &off, &ch);
    const cplx lam = c1[ch], a0 = tap0[ch], a1 = tap1[ch];
    cplx state = 0.0, xprev = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    cplx gprev = 0.0; /* masked g at t-1, for gzw[t-1] */
    for (int64_t t = 0; t < r.T; ++t) {
      const cplx xt = x[off + t * r.ts];
      const cplx yprev = state;
      state = lam * state + a0 * xt + a1 * xprev;
      const cplx graw = gy[off + t * r.ts];
      const cplx g = fuse_act ? mask_c(graw, state) : graw;
      gz[off + t * r.ts] = conj(a0) * g;
      if (t > 0) gzw[off + (t - 1) * r.ts] = conj(a1) * g;
      s1 += conj(yprev) * g;
      s2 += conj(xt) * g;
      s3 += conj(xprev) * g;
      xprev = xt;
      gprev = g;
    }
    (void)gprev;
    if (r.T > 0) gzw[off + (r.T - 1) * r.ts] = 0.0;
    part[row * 3 + 0] = s1;
    part[row * 3 + 1] = s2;
    part[row * 3 + 2] = s3;
  }
  for (int64_t f = 0; f < r.F; ++f) gc1[f] = gt0[f] = gt1[f] = 0.0;
  for (int64_t row = 0; row < r.R; ++row) {
    int64_t off, ch;
    row_info(&r, row, &off, &ch);
    gc1[ch] += part[row * 3 + 0];
    gt0[ch] += part[row * 3 + 1];
    gt1[ch] += part[row * 3 + 2];
  }
  free(part);
  return 0;
}

int rqfo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
