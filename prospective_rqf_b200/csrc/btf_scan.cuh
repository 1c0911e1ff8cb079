// Diagonal scans in (batch, time, filters) layout — filters innermost.
//
// Serves rqf_models/ops/chunked_scan_kernel.py:_triton_chunked_scan (:340)
// and _triton_chunked_scan_prospective (:506) without their (B,T,F) <-> (B,F,T)
// permutes (chunked_scan_kernel.py:212-214, :249, :272-275, :302):
//   PLAIN    y[t] = c1*y[t-1] + c2*u[t]                 (u complex)
//   REAL     same with u real (scan.py:366 promotes; the values are identical)
//   TWO_TAP  y[t] = c1*y[t-1] + tap0*x[t] + tap1*x[t-1]
//
// Work decomposition: one CTA = 32 adjacent channels (lanes, so every load
// and store of a time step is one coalesced 256-byte row segment) x NW warps,
// warp w owning K consecutive time steps.  Each lane runs its channel's
// recurrence serially over its K steps, warps are composed in shared memory,
// and tiles of NW*K steps are chained by a per-channel decoupled look-back.
// Backward recomputes y from the per-tile carries and fuses the adjoint with
// grad_u / grad_x and the coefficient-gradient partial sums.
#pragma once

#include "rqf_common.cuh"

namespace rqf {

enum BtfDrive { kPlain = 0, kReal = 1, kTwoTap = 2 };

struct BtfArgs {
  const float2 *c1;
  const float2 *c2;    // c2 (PLAIN/REAL) or tap0 (TWO_TAP)
  const float2 *tap1;  // TWO_TAP only
  const void *x;       // (B,T,F) complex, or float for REAL
  const float2 *gout;  // (B,T,F) cotangent (backward)
  void *out;           // forward: y; backward: grad_x (float for REAL)
  float2 *out2;        // TBPTT backward: grad_zw
  float2 *carries;     // (B*F, ntiles), row = b*F + f
  float2 *partials;    // (B*F, ntiles, 3)
  u64 *flags;          // (B*F, ntiles, 2)
  unsigned *ticket;
  int64_t B, T, F;
  int nfb;     // channel blocks of 32
  int ntiles;  // tiles along time
  int log2L;
};

constexpr int kBtfWarps = 8;
constexpr int kBtfK = 16;
constexpr int kBtfTile = kBtfWarps * kBtfK;  // 128 time steps x 32 channels
constexpr int kBtfLog2Tile = 7;

template <int DRIVE>
__device__ __forceinline__ float2 btf_load_x(const void *x, int64_t idx) {
  if constexpr (DRIVE == kReal) {
    return make_float2(__ldcs(static_cast<const float *>(x) + idx), 0.f);
  } else {
    return __ldcs(static_cast<const float2 *>(x) + idx);
  }
}

template <int NW, int K, int DRIVE>
__global__ void __launch_bounds__(NW * 32) btf_fwd_kernel(const BtfArgs a) {
  constexpr int L = NW * K;
  __shared__ float4 s_agg[NW][32];
  __shared__ float2 s_C[32];
  __shared__ unsigned s_ticket;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_ticket = atomicAdd(a.ticket, 1u);
  __syncthreads();
  const unsigned tk = s_ticket;
  const int64_t grp = tk / (unsigned)a.ntiles;
  const int j = (int)(tk - (unsigned)(grp * a.ntiles));
  const int64_t bi = grp / a.nfb;
  const int64_t f = (grp - bi * a.nfb) * 32 + lane;
  const bool fv = f < a.F;
  const float2 lam = fv ? a.c1[f] : cz();
  const float2 c2 = fv ? a.c2[f] : cz();
  const float2 t1 = (DRIVE == kTwoTap && fv) ? a.tap1[f] : cz();
  const int64_t base = bi * a.T * a.F + f;  // element (bi, t, f) = base + t*F
  const int64_t tw = (int64_t)j * L + (int64_t)warp * K;

  float2 x[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int64_t t = tw + k;
    x[k] = (fv && t < a.T) ? btf_load_x<DRIVE>(a.x, base + t * a.F) : cz();
  }
  float2 b[K];
  if constexpr (DRIVE == kTwoTap) {
    const float2 xp = (fv && tw > 0 && tw - 1 < a.T) ? btf_load_x<DRIVE>(a.x, base + (tw - 1) * a.F)
                                                     : cz();
    b[0] = c_fma(t1, xp, c_mul(c2, x[0]));
#pragma unroll
    for (int k = 1; k < K; ++k) b[k] = c_fma(t1, x[k - 1], c_mul(c2, x[k]));
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) b[k] = c_mul(c2, x[k]);
  }
  float2 y = cz();
#pragma unroll
  for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
  const float2 gK = c_pow2k(lam, (K == 8) ? 3 : (K == 16) ? 4 : 2);
  s_agg[warp][lane] = make_float4(gK.x, gK.y, y.x, y.y);
  __syncthreads();
  float2 Gw = cone(), Xw = cz(), Xall = cz();
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const float4 q = s_agg[w][lane];
    const float2 gw = make_float2(q.x, q.y), aw = make_float2(q.z, q.w);
    if (w == warp) Xw = Xall;
    if (w < warp) Gw = c_mul(gw, Gw);
    Xall = c_fma(gw, Xall, aw);
  }
  if (warp == 0) {
    float2 C = cz();
    if (fv) {
      const int64_t row = bi * a.F + f;
      u64 *fl = a.flags + row * (int64_t)a.ntiles * 2;
      const bool has_next = j + 1 < a.ntiles;
      if (j == 0) {
        if (has_next) flag_publish2(fl, Xall, kInclusive);
      } else {
        if (has_next) flag_publish2(fl + 2 * j, Xall, kAggregate);
        const float2 M = c_pow2k(lam, a.log2L);
        C = lookback_const(fl, j, M);
        if (has_next) flag_publish2(fl + 2 * j, c_fma(M, C, Xall), kInclusive);
      }
      a.carries[row * a.ntiles + j] = C;
    }
    s_C[lane] = C;
  }
  __syncthreads();
  float2 e = c_fma(Gw, s_C[lane], Xw);
  float2 *yout = static_cast<float2 *>(a.out);
#pragma unroll
  for (int k = 0; k < K; ++k) {
    e = c_fma(lam, e, b[k]);
    const int64_t t = tw + k;
    if (fv && t < a.T) __stcs(yout + base + t * a.F, e);
  }
}

template <int NW, int K, int DRIVE>
__global__ void __launch_bounds__(NW * 32) btf_bwd_kernel(const BtfArgs a) {
  constexpr int L = NW * K;
  __shared__ float4 s_agg[NW][32];
  __shared__ float4 s_rev[NW][32];
  __shared__ float2 s_red[3][NW][32];
  __shared__ float2 s_D[32];
  __shared__ unsigned s_ticket;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_ticket = atomicAdd(a.ticket, 1u);
  __syncthreads();
  const unsigned tk = s_ticket;
  const int64_t grp = tk / (unsigned)a.ntiles;
  const int p = (int)(tk - (unsigned)(grp * a.ntiles));
  const int j = a.ntiles - 1 - p;
  const int64_t bi = grp / a.nfb;
  const int64_t f = (grp - bi * a.nfb) * 32 + lane;
  const bool fv = f < a.F;
  const int64_t row = bi * a.F + f;
  const float2 lam = fv ? a.c1[f] : cz();
  const float2 c2 = fv ? a.c2[f] : cz();
  const float2 t1 = (DRIVE == kTwoTap && fv) ? a.tap1[f] : cz();
  const float2 C = fv ? a.carries[row * a.ntiles + j] : cz();
  const int64_t base = bi * a.T * a.F + f;
  const int64_t tw = (int64_t)j * L + (int64_t)warp * K;

  float2 x[K], go[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int64_t t = tw + k;
    const bool in = fv && t < a.T;
    x[k] = in ? btf_load_x<DRIVE>(a.x, base + t * a.F) : cz();
    go[k] = in ? __ldcs(a.gout + base + t * a.F) : cz();
  }
  float2 xp = cz();
  float2 b[K];
  if constexpr (DRIVE == kTwoTap) {
    xp = (fv && tw > 0 && tw - 1 < a.T) ? btf_load_x<DRIVE>(a.x, base + (tw - 1) * a.F) : cz();
    b[0] = c_fma(t1, xp, c_mul(c2, x[0]));
#pragma unroll
    for (int k = 1; k < K; ++k) b[k] = c_fma(t1, x[k - 1], c_mul(c2, x[k]));
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) b[k] = c_mul(c2, x[k]);
  }
  // forward recompute from the stored tile carry
  float2 y = cz();
#pragma unroll
  for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
  const float2 gK = c_pow2k(lam, (K == 8) ? 3 : (K == 16) ? 4 : 2);
  // reverse local aggregate of the adjoint
  const float2 mu = c_conj(lam);
  float2 h = cz();
#pragma unroll
  for (int k = K - 1; k >= 0; --k) h = c_fma(mu, h, go[k]);
  const float2 muK = c_conj(gK);
  s_agg[warp][lane] = make_float4(gK.x, gK.y, y.x, y.y);
  s_rev[warp][lane] = make_float4(muK.x, muK.y, h.x, h.y);
  __syncthreads();
  float2 Gw = cone(), Xw = cz(), Xall = cz();
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const float4 q = s_agg[w][lane];
    const float2 gw = make_float2(q.x, q.y), aw = make_float2(q.z, q.w);
    if (w == warp) Xw = Xall;
    if (w < warp) Gw = c_mul(gw, Gw);
    Xall = c_fma(gw, Xall, aw);
  }
  float2 Grw = cone(), Xrw = cz(), Xrall = cz();
#pragma unroll
  for (int w = NW - 1; w >= 0; --w) {
    const float4 q = s_rev[w][lane];
    const float2 gw = make_float2(q.x, q.y), aw = make_float2(q.z, q.w);
    if (w == warp) Xrw = Xrall;
    if (w > warp) Grw = c_mul(gw, Grw);
    Xrall = c_fma(gw, Xrall, aw);
  }
  if (warp == 0) {
    float2 D = cz();
    if (fv) {
      u64 *fl = a.flags + row * (int64_t)a.ntiles * 2;
      const bool has_next = p + 1 < a.ntiles;
      if (p == 0) {
        if (has_next) flag_publish2(fl, Xrall, kInclusive);
      } else {
        if (has_next) flag_publish2(fl + 2 * p, Xrall, kAggregate);
        const float2 M = c_pow2k(mu, a.log2L);
        D = lookback_const(fl, p, M);
        if (has_next) flag_publish2(fl + 2 * p, c_fma(M, D, Xrall), kInclusive);
      }
    }
    s_D[lane] = D;
  }
  __syncthreads();
  float2 e = c_fma(Gw, C, Xw);
  float2 yprev[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    yprev[k] = e;
    e = c_fma(lam, e, b[k]);
  }
  float2 gnext = c_fma(Grw, s_D[lane], Xrw);
  float2 acc_c1 = cz(), acc_1 = cz(), acc_2 = cz();
#pragma unroll
  for (int k = K - 1; k >= 0; --k) {
    const float2 g = c_fma(mu, gnext, go[k]);
    const int64_t t = tw + k;
    const bool in = fv && t < a.T;
    if constexpr (DRIVE == kReal) {
      // grad of the real input: Re(conj(c2) g)
      if (in) __stcs(static_cast<float *>(a.out) + base + t * a.F, c2.x * g.x + c2.y * g.y);
      acc_1 = make_float2(fmaf(x[k].x, g.x, acc_1.x), fmaf(x[k].x, g.y, acc_1.y));
    } else if constexpr (DRIVE == kPlain) {
      if (in) __stcs(static_cast<float2 *>(a.out) + base + t * a.F, c_cfma(c2, g, cz()));
      acc_1 = c_cfma(x[k], g, acc_1);
    } else {
      if (in)
        __stcs(static_cast<float2 *>(a.out) + base + t * a.F,
               c_cfma(t1, gnext, c_cfma(c2, g, cz())));
      acc_1 = c_cfma(x[k], g, acc_1);
      acc_2 = c_cfma(k > 0 ? x[k - 1] : xp, g, acc_2);
    }
    acc_c1 = c_cfma(yprev[k], g, acc_c1);
    gnext = g;
  }
  s_red[0][warp][lane] = acc_c1;
  s_red[1][warp][lane] = acc_1;
  s_red[2][warp][lane] = acc_2;
  __syncthreads();
  if (warp < 3 && fv) {
    float2 s = cz();
#pragma unroll
    for (int w = 0; w < NW; ++w) s = c_add(s, s_red[warp][w][lane]);
    a.partials[(row * a.ntiles + j) * 3 + warp] = s;
  }
}

// TBPTT(1) surrogate backward in (B,T,F) layout (no temporal adjoint).  One
// CTA per (batch, channel block, tile) in blockIdx order.
template <int NW, int K, bool FUSE_ACT>
__global__ void __launch_bounds__(NW * 32) btf_tbptt_bwd_kernel(const BtfArgs a) {
  constexpr int L = NW * K;
  __shared__ float4 s_agg[NW][32];
  __shared__ float2 s_first[NW + 1][32];
  __shared__ float2 s_red[3][NW][32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t grp = blockIdx.x / (unsigned)a.ntiles;
  const int j = (int)(blockIdx.x - (unsigned)(grp * a.ntiles));
  const int64_t bi = grp / a.nfb;
  const int64_t f = (grp - bi * a.nfb) * 32 + lane;
  const bool fv = f < a.F;
  const int64_t row = bi * a.F + f;
  const float2 lam = fv ? a.c1[f] : cz();
  const float2 t0 = fv ? a.c2[f] : cz();
  const float2 t1 = fv ? a.tap1[f] : cz();
  const float2 C = fv ? a.carries[row * a.ntiles + j] : cz();
  const int64_t base = bi * a.T * a.F + f;
  const int64_t tw = (int64_t)j * L + (int64_t)warp * K;
  const float2 *xs = static_cast<const float2 *>(a.x);

  float2 x[K], go[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int64_t t = tw + k;
    const bool in = fv && t < a.T;
    x[k] = in ? __ldcs(xs + base + t * a.F) : cz();
    go[k] = in ? __ldcs(a.gout + base + t * a.F) : cz();
  }
  const float2 xp = (fv && tw > 0 && tw - 1 < a.T) ? xs[base + (tw - 1) * a.F] : cz();
  float2 b[K];
  b[0] = c_fma(t1, xp, c_mul(t0, x[0]));
#pragma unroll
  for (int k = 1; k < K; ++k) b[k] = c_fma(t1, x[k - 1], c_mul(t0, x[k]));
  float2 y = cz();
#pragma unroll
  for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
  const float2 gK = c_pow2k(lam, (K == 8) ? 3 : (K == 16) ? 4 : 2);
  s_agg[warp][lane] = make_float4(gK.x, gK.y, y.x, y.y);
  __syncthreads();
  float2 Gw = cone(), Xw = cz(), Xall = cz();
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const float4 q = s_agg[w][lane];
    const float2 gw = make_float2(q.x, q.y), aw = make_float2(q.z, q.w);
    if (w == warp) Xw = Xall;
    if (w < warp) Gw = c_mul(gw, Gw);
    Xall = c_fma(gw, Xall, aw);
  }
  float2 e = c_fma(Gw, C, Xw);
  float2 yprev[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    yprev[k] = e;
    e = c_fma(lam, e, b[k]);
    if (FUSE_ACT) go[k] = c_relu_mask(go[k], e);
  }
  s_first[warp][lane] = go[0];
  if (warp == NW - 1) {
    const int64_t tn = (int64_t)(j + 1) * L;
    float2 g_next = cz();
    if (fv && tn < a.T) {
      g_next = a.gout[base + tn * a.F];
      if (FUSE_ACT) {
        const float2 yn = c_fma(lam, e, c_fma(t1, x[K - 1], c_mul(t0, xs[base + tn * a.F])));
        g_next = c_relu_mask(g_next, yn);
      }
    }
    s_first[NW][lane] = g_next;
  }
  __syncthreads();
  const float2 gn = s_first[warp + 1][lane];
  float2 acc_c1 = cz(), acc_t0 = cz(), acc_t1 = cz();
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float2 g = go[k];
    const float2 g1 = (k + 1 < K) ? go[k + 1] : gn;
    const int64_t t = tw + k;
    if (fv && t < a.T) {
      __stcs(static_cast<float2 *>(a.out) + base + t * a.F, c_cfma(t0, g, cz()));
      __stcs(a.out2 + base + t * a.F, c_cfma(t1, g1, cz()));
    }
    acc_c1 = c_cfma(yprev[k], g, acc_c1);
    acc_t0 = c_cfma(x[k], g, acc_t0);
    acc_t1 = c_cfma(k > 0 ? x[k - 1] : xp, g, acc_t1);
  }
  s_red[0][warp][lane] = acc_c1;
  s_red[1][warp][lane] = acc_t0;
  s_red[2][warp][lane] = acc_t1;
  __syncthreads();
  if (warp < 3 && fv) {
    float2 s = cz();
#pragma unroll
    for (int w = 0; w < NW; ++w) s = c_add(s, s_red[warp][w][lane]);
    a.partials[(row * a.ntiles + j) * 3 + warp] = s;
  }
}

}  // namespace rqf
