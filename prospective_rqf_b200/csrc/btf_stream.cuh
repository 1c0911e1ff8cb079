// Diagonal scans in (batch, time, filters) layout — filters innermost.
//
// Serves rqf_models/ops/chunked_scan_kernel.py:_triton_chunked_scan (:340)
// and _triton_chunked_scan_prospective (:506) without their (B,T,F) <-> (B,F,T)
// permutes (chunked_scan_kernel.py:212-214, :249, :272-275, :302):
//   PLAIN    y[t] = c1*y[t-1] + c2*u[t]                 (u complex)
//   REAL     same with u real (scan.py:366 promotes; the values are identical)
//   TWO_TAP  y[t] = c1*y[t-1] + tap0*x[t] + tap1*x[t-1]
//
// Streaming variant (namespace rqf::btfs), used when there are few chains
// (batch x 32-channel blocks): long tiles keep the look-back hops per step
// low, and the second pass re-reads a tile from L2 instead of holding it in
// shared memory (rqf::btf_*_kernel in btf_scan.cuh hold it).
//
// Work decomposition.  A "chain" is one batch index and a block of 32 adjacent
// channels (lanes, so every load and store of a time step is one coalesced
// 256-byte row segment).  A sub-tile is NW warps x K consecutive time steps
// (128 steps): each lane runs its channel's recurrence serially over its K
// steps and the warps are composed in shared memory.  A CTA owns a tile of S
// consecutive sub-tiles: pass 1 streams them to form the tile's aggregate, a
// per-channel decoupled look-back chains the tiles of a chain, and pass 2
// re-streams the sub-tiles (from L2: the tile was just read) with their
// entry states to produce the outputs.  S (1..8) is chosen per call from the
// number of chains.  Tickets run tile-major across chains, so resident CTAs
// work on different chains instead of queueing behind one.
// The forward saves the state entering every sub-tile; the backward starts
// each sub-tile from it, and fuses the adjoint with
// grad_u / grad_x and the coefficient-gradient partial sums (one partial per
// tile, reduced in fixed order afterwards).
#pragma once

#include "rqf_common.cuh"

namespace rqf {
namespace btfs {


struct BtfArgs {
  const float2 *c1;
  const float2 *c2;    // c2 (PLAIN/REAL) or tap0 (TWO_TAP)
  const float2 *tap1;  // TWO_TAP only
  const void *x;       // (B,T,F) complex, or float for REAL
  const float2 *gout;  // (B,T,F) cotangent (backward)
  void *out;           // forward: y; backward: grad_x (float for REAL)
  float2 *out2;        // TBPTT backward: grad_zw
  float2 *carries;     // (B*F, csub), row = b*F + f: the state entering each 128-step sub-tile
  int csub;            // saved states per row (at least the sub-tiles that start before T)
  float2 *partials;    // (B*F, ntiles, 3)
  u64 *flags;          // (B*F, ntiles, 2)
  unsigned *ticket;
  int64_t B, T, F;
  int nfb;      // channel blocks of 32
  int ngroups;  // chains: B * nfb
  int ntiles;   // tiles along time
  int log2L;    // log2 of the tile length (S sub-tiles)
};

constexpr int kBtfSub = 128;     // time steps of a sub-tile
constexpr int kBtfLog2Sub = 7;
constexpr int kBtfMaxS = 8;      // sub-tiles per tile, at most

// Load policies.  A tile read twice (S > 1) is read in pass 1 with the default
// policy so that it stays in L2, and in pass 2 (its last use) as streaming
// (evict-first); a tile read once streams.
template <typename V>
__device__ __forceinline__ V btf_ld(const V *p, bool last_use) {
  return last_use ? __ldcs(p) : __ldcg(p);
}
template <int DRIVE>
__device__ __forceinline__ float2 btf_load_x(const void *x, int64_t idx, bool last_use) {
  if constexpr (DRIVE == kReal) {
    return make_float2(btf_ld(static_cast<const float *>(x) + idx, last_use), 0.f);
  } else {
    return btf_ld(static_cast<const float2 *>(x) + idx, last_use);
  }
}

__host__ __device__ constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v / 2); }

// Drive b[k] = c2 x[k] (+ tap1 x[k-1]) of a warp's K steps starting at tw;
// LAST: this is the tile's last read (see the load policies above).
template <int K, int DRIVE, bool LAST>
__device__ __forceinline__ void btf_drive(const BtfArgs &a, int64_t base, int64_t tw, bool fv,
                                          float2 c2, float2 t1, float2 (&x)[K], float2 &xp,
                                          float2 (&b)[K]) {
  if (fv && tw + K <= a.T) {  // the whole segment in range: no per-step tests
    int64_t idx = base + tw * a.F;
#pragma unroll
    for (int k = 0; k < K; ++k, idx += a.F) x[k] = btf_load_x<DRIVE>(a.x, idx, LAST);
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t t = tw + k;
      const bool in = fv && t < a.T;
      x[k] = in ? btf_load_x<DRIVE>(a.x, base + t * a.F, LAST) : cz();
    }
  }
  xp = cz();
  if constexpr (DRIVE == kTwoTap) {
    xp = (fv && tw > 0 && tw - 1 < a.T) ? btf_load_x<DRIVE>(a.x, base + (tw - 1) * a.F, false)
                                        : cz();
    b[0] = c_fma(t1, xp, c_mul(c2, x[0]));
#pragma unroll
    for (int k = 1; k < K; ++k) b[k] = c_fma(t1, x[k - 1], c_mul(c2, x[k]));
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) b[k] = c_mul(c2, x[k]);
  }
}

// The cotangent of a warp's K steps starting at tw (zero past T).
template <int K>
__device__ __forceinline__ void btf_load_go(const BtfArgs &a, int64_t base, int64_t tw, bool fv,
                                            bool last_use, float2 (&go)[K]) {
  if (fv && tw + K <= a.T) {
    int64_t idx = base + tw * a.F;
#pragma unroll
    for (int k = 0; k < K; ++k, idx += a.F) go[k] = btf_ld(a.gout + idx, last_use);
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t t = tw + k;
      go[k] = (fv && t < a.T) ? btf_ld(a.gout + base + t * a.F, last_use) : cz();
    }
  }
}

// Into L2: the warp's K steps starting at tw of its chain in x (ESZ bytes per
// element), one 128-byte line per lane (a step of 32 complex channels is two
// lines, of 32 real ones one), so that the loads issued for them after the
// next sub-tile barrier find them in L2.  base0: element (bi, 0, first
// channel of the chain), fb0 that channel; only lines holding channels below
// F are touched.
template <int K, int ESZ>
__device__ __forceinline__ void btf_prefetch(const void *x, int64_t base0, int64_t tw,
                                             const BtfArgs &a, int fb0, int lane) {
  constexpr int kLines = (32 * ESZ) / 128;  // lines per step: 2 or 1
  const int step = lane / kLines, part = lane - step * kLines;
  const int64_t t = tw + step;
  if (step < K && t < a.T && fb0 + part * (128 / ESZ) < a.F)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(static_cast<const char *>(x) +
                                                 (base0 + t * a.F) * ESZ + part * 128));
}

// ------------------------------------------------------------ forward
// ABS: write |y| (float) instead of y (rqf::btf_store_y); a null carries
// pointer skips the saved entry states.
template <int NW, int K, int S, int DRIVE, bool ABS = false>
__global__ void __launch_bounds__(NW * 32) btf_fwd_kernel(const BtfArgs a) {
  constexpr int L = NW * K;  // sub-tile
  static_assert(L == kBtfSub, "sub-tile length");
  __shared__ float2 s_y[2][NW][32];
  __shared__ float2 s_sub[S][32];
  __shared__ float2 s_C[32];
  __shared__ unsigned s_ticket;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_ticket = atomicAdd(a.ticket, 1u);
  __syncthreads();
  const unsigned tk = s_ticket;
  const int j = (int)(tk / (unsigned)a.ngroups);
  const int64_t grp = tk - (unsigned)j * (unsigned)a.ngroups;
  const int64_t bi = grp / a.nfb;
  const int64_t f = (grp - bi * a.nfb) * 32 + lane;
  const bool fv = f < a.F;
  const float2 lam = fv ? a.c1[f] : cz();
  const float2 c2 = fv ? a.c2[f] : cz();
  const float2 t1 = (DRIVE == kTwoTap && fv) ? a.tap1[f] : cz();
  const int64_t base = bi * a.T * a.F + f;  // element (bi, t, f) = base + t*F
  const int64_t tile0 = (int64_t)j * S * L;
  const float2 gK = c_pow2k(lam, ilog2(K));
  const float2 gL = c_pow2k(lam, kBtfLog2Sub);
  float2 Gw = cone();  // lam^(K*warp): gain from this warp's start back to the sub-tile start
  for (int w = 0; w < warp; ++w) Gw = c_mul(gK, Gw);

  // pass 1: sub-tile aggregates (zero entry), composed into the tile's.  With
  // one sub-tile (S == 1) the drive stays in registers for pass 2.
  float2 Xtile = cz();
  float2 x[K], xp, b[K];
#pragma unroll 1
  for (int s = 0; s < S; ++s) {
    const int64_t tw = tile0 + (int64_t)s * L + (int64_t)warp * K;
    if (s + 1 < S)
      btf_prefetch<K, DRIVE == kReal ? 4 : 8>(a.x, base - lane, tw + L, a, (int)(f - lane), lane);
    btf_drive<K, DRIVE, S == 1>(a, base, tw, fv, c2, t1, x, xp, b);
    float2 y = cz();
#pragma unroll
    for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
    s_y[s & 1][warp][lane] = y;
    __syncthreads();
    if (warp == 0) {  // only warp 0 needs the sub-tile and tile totals
      float2 X = cz();
#pragma unroll
      for (int w = 0; w < NW; ++w) X = c_fma(gK, X, s_y[s & 1][w][lane]);
      s_sub[s][lane] = X;
      Xtile = c_fma(gL, Xtile, X);
    }
  }
  if (warp == 0) {
    float2 C = cz();
    if (fv) {
      const int64_t row = bi * a.F + f;
      u64 *fl = a.flags + row * (int64_t)a.ntiles * 2;
      const bool has_next = j + 1 < a.ntiles;
      if (j == 0) {
        if (has_next) flag_publish2(fl, Xtile, kInclusive);
      } else {
        if (has_next) flag_publish2(fl + 2 * j, Xtile, kAggregate);
        const float2 M = c_pow2k(lam, a.log2L);
        C = lookback_const_win(fl, j, M);
        if (has_next) flag_publish2(fl + 2 * j, c_fma(M, C, Xtile), kInclusive);
      }
    }
    s_C[lane] = C;
  }
  __syncthreads();

  // pass 2: outputs, sub-tile by sub-tile from their entry states (saved
  // for the backward)
  float2 es = s_C[lane];
#pragma unroll 1
  for (int s = 0; s < S; ++s) {
    const int64_t tw = tile0 + (int64_t)s * L + (int64_t)warp * K;
    if (warp == 0 && fv && a.carries && tile0 + (int64_t)s * L < a.T)
      a.carries[(bi * a.F + f) * a.csub + (int64_t)j * S + s] = es;
    if constexpr (S > 1) {
      btf_drive<K, DRIVE, true>(a, base, tw, fv, c2, t1, x, xp, b);
      float2 y = cz();
#pragma unroll
      for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
      s_y[s & 1][warp][lane] = y;
      __syncthreads();
    }
    float2 Xw = cz();
    for (int w = 0; w < warp; ++w) Xw = c_fma(gK, Xw, s_y[s & 1][w][lane]);
    float2 e = c_fma(Gw, es, Xw);
    if (fv && tw + K <= a.T) {
      int64_t idx = base + tw * a.F;
#pragma unroll
      for (int k = 0; k < K; ++k, idx += a.F) {
        e = c_fma(lam, e, b[k]);
        btf_store_y<ABS>(a.out, idx, e);
      }
    } else {
#pragma unroll
      for (int k = 0; k < K; ++k) {
        e = c_fma(lam, e, b[k]);
        const int64_t t = tw + k;
        if (fv && t < a.T) btf_store_y<ABS>(a.out, base + t * a.F, e);
      }
    }
    es = c_fma(gL, es, s_sub[s][lane]);
  }
}

// ------------------------------------------------------------ backward
template <int NW, int K, int S, int DRIVE>
__global__ void __launch_bounds__(NW * 32) btf_bwd_kernel(const BtfArgs a) {
  constexpr int L = NW * K;
  static_assert(L == kBtfSub, "sub-tile length");
  __shared__ float4 s_yh[2][NW][32];   // (forward local y, reverse local h) per warp
  __shared__ float2 s_subr[S][32];     // reverse sub-tile aggregates
  __shared__ float2 s_red[3][NW][32];
  __shared__ float2 s_D[32];
  __shared__ unsigned s_ticket;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_ticket = atomicAdd(a.ticket, 1u);
  __syncthreads();
  const unsigned tk = s_ticket;
  const int p = (int)(tk / (unsigned)a.ngroups);
  const int64_t grp = tk - (unsigned)p * (unsigned)a.ngroups;
  const int j = a.ntiles - 1 - p;
  const int64_t bi = grp / a.nfb;
  const int64_t f = (grp - bi * a.nfb) * 32 + lane;
  const bool fv = f < a.F;
  const int64_t row = bi * a.F + f;
  const float2 lam = fv ? a.c1[f] : cz();
  const float2 c2 = fv ? a.c2[f] : cz();
  const float2 t1 = (DRIVE == kTwoTap && fv) ? a.tap1[f] : cz();
  const int64_t base = bi * a.T * a.F + f;
  const int64_t tile0 = (int64_t)j * S * L;
  const float2 mu = c_conj(lam);
  const float2 gK = c_pow2k(lam, ilog2(K)), muK = c_conj(gK);
  const float2 gL = c_pow2k(lam, kBtfLog2Sub), muL = c_conj(gL);
  float2 Gw = cone(), Grw = cone();  // lam^(K*warp), conj(lam)^(K*(NW-1-warp))
  for (int w = 0; w < warp; ++w) Gw = c_mul(gK, Gw);
  for (int w = NW - 1; w > warp; --w) Grw = c_mul(muK, Grw);

  // pass 1: reverse sub-tile aggregates (the forward's saved entry states
  // give each sub-tile's forward entry).  With one sub-tile (S == 1) the
  // drive, the loaded values and the warp exchange stay for pass 2.
  float2 Xrtile = cz(), pw = cone();
  float2 x[K], xp, b[K], go[K];
#pragma unroll 1
  for (int s = 0; s < S; ++s) {
    const int64_t tw = tile0 + (int64_t)s * L + (int64_t)warp * K;
    float2 y = cz(), h = cz();
    if constexpr (S == 1) {
      btf_drive<K, DRIVE, true>(a, base, tw, fv, c2, t1, x, xp, b);
#pragma unroll
      for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
    }
    if (s + 1 < S) btf_prefetch<K, 8>(a.gout, base - lane, tw + L, a, (int)(f - lane), lane);
    btf_load_go<K>(a, base, tw, fv, S == 1, go);
#pragma unroll
    for (int k = K - 1; k >= 0; --k) h = c_fma(mu, h, go[k]);
    s_yh[s & 1][warp][lane] = make_float4(y.x, y.y, h.x, h.y);
    __syncthreads();
    // reverse sub-tile totals by warp 1 (the tile total handed to warp 0
    // through s_D below)
    if (warp == 1) {
      float2 Xr = cz();
#pragma unroll
      for (int w = NW - 1; w >= 0; --w) {
        const float4 q = s_yh[s & 1][w][lane];
        Xr = c_fma(muK, Xr, make_float2(q.z, q.w));
      }
      s_subr[s][lane] = Xr;
      Xrtile = c_fma(pw, Xr, Xrtile);  // sub-tile s starts L*s steps into the tile
      pw = c_mul(muL, pw);
    }
  }
  if (warp == 1) s_D[lane] = Xrtile;
  __syncthreads();
  if (warp == 0) {
    float2 D = cz();
    const float2 Xrtile0 = s_D[lane];
    if (fv) {
      u64 *fl = a.flags + row * (int64_t)a.ntiles * 2;
      const bool has_next = p + 1 < a.ntiles;
      if (p == 0) {
        if (has_next) flag_publish2(fl, Xrtile0, kInclusive);
      } else {
        if (has_next) flag_publish2(fl + 2 * p, Xrtile0, kAggregate);
        const float2 M = c_pow2k(mu, a.log2L);
        D = lookback_const_win(fl, p, M);
        if (has_next) flag_publish2(fl + 2 * p, c_fma(M, D, Xrtile0), kInclusive);
      }
    }
    __syncwarp();
    s_D[lane] = D;
  }
  __syncthreads();

  // sub-tile entry states: forward C_s saved by the forward, reverse D_s (the
  // adjoint entering sub-tile s from its right) from the look-back
  float2 Ds = s_D[lane];

  // pass 2: sub-tiles from last to first.  The element-wise products run on
  // paired fp32 FMAs: conj(c) g = (c.x, c.x) g + (c.y, -c.y) (g.y, g.x), and
  // each sum conj(v) g accumulates v (g.x, g.x) and v (g.y, g.y) separately,
  // combined once at the end.
  const float2 C2X = make_float2(c2.x, c2.x), C2Y = make_float2(c2.y, -c2.y);
  const float2 T1X = make_float2(t1.x, t1.x), T1Y = make_float2(t1.y, -t1.y);
  float2 pc1 = cz(), qc1 = cz(), p1 = cz(), q1 = cz(), p2 = cz(), q2 = cz();
#pragma unroll 1
  for (int s = S - 1; s >= 0; --s) {
    const int64_t tw = tile0 + (int64_t)s * L + (int64_t)warp * K;
    if constexpr (S > 1) {
      btf_drive<K, DRIVE, true>(a, base, tw, fv, c2, t1, x, xp, b);
      btf_load_go<K>(a, base, tw, fv, true, go);
      float2 y = cz(), h = cz();
#pragma unroll
      for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
#pragma unroll
      for (int k = K - 1; k >= 0; --k) h = c_fma(mu, h, go[k]);
      s_yh[s & 1][warp][lane] = make_float4(y.x, y.y, h.x, h.y);
      __syncthreads();
    }
    float2 Xw = cz(), Xrw = cz();
    for (int w = 0; w < warp; ++w) {
      const float4 q = s_yh[s & 1][w][lane];
      Xw = c_fma(gK, Xw, make_float2(q.x, q.y));
    }
    for (int w = NW - 1; w > warp; --w) {
      const float4 q = s_yh[s & 1][w][lane];
      Xrw = c_fma(muK, Xrw, make_float2(q.z, q.w));
    }
    const float2 Cs = (fv && tile0 + (int64_t)s * L < a.T)
                          ? a.carries[row * a.csub + (int64_t)j * S + s]
                          : cz();
    float2 e = c_fma(Gw, Cs, Xw);
    float2 yprev[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      yprev[k] = e;
      e = c_fma(lam, e, b[k]);
    }
    float2 gnext = c_fma(Grw, Ds, Xrw);
    float2 gnsw = c_swap(gnext);
    const bool full = fv && tw + K <= a.T;
    int64_t idx = base + (tw + K - 1) * a.F;
#pragma unroll
    for (int k = K - 1; k >= 0; --k, idx -= a.F) {
      const float2 g = c_fma(mu, gnext, go[k]);
      const float2 gs = c_swap(g);
      const float2 gx = make_float2(g.x, g.x), gy = make_float2(g.y, g.y);
      const bool in = full || (fv && tw + k < a.T);
      if constexpr (DRIVE == kReal) {
        // grad of the real input: Re(conj(c2) g)
        if (in) __stcs(static_cast<float *>(a.out) + idx, fmaf(c2.x, g.x, c2.y * g.y));
        p1 = __ffma2_rn(make_float2(x[k].x, x[k].x), g, p1);  // conj(x) g, x real
      } else if constexpr (DRIVE == kPlain) {
        if (in) __stcs(static_cast<float2 *>(a.out) + idx, __ffma2_rn(C2X, g, __fmul2_rn(C2Y, gs)));
        p1 = __ffma2_rn(x[k], gx, p1);
        q1 = __ffma2_rn(x[k], gy, q1);
      } else {
        if (in)
          __stcs(static_cast<float2 *>(a.out) + idx,
                 __ffma2_rn(C2X, g, __ffma2_rn(C2Y, gs, __ffma2_rn(T1X, gnext,
                                                                    __fmul2_rn(T1Y, gnsw)))));
        p1 = __ffma2_rn(x[k], gx, p1);
        q1 = __ffma2_rn(x[k], gy, q1);
        const float2 xk1 = k > 0 ? x[k - 1] : xp;
        p2 = __ffma2_rn(xk1, gx, p2);
        q2 = __ffma2_rn(xk1, gy, q2);
      }
      pc1 = __ffma2_rn(yprev[k], gx, pc1);
      qc1 = __ffma2_rn(yprev[k], gy, qc1);
      gnext = g;
      gnsw = gs;
    }
    Ds = c_fma(muL, Ds, s_subr[s][lane]);  // adjoint entering sub-tile s-1
  }
  // conj(v) g = (v.x g.x + v.y g.y, v.x g.y - v.y g.x)
  s_red[0][warp][lane] = make_float2(pc1.x + qc1.y, qc1.x - pc1.y);
  s_red[1][warp][lane] = DRIVE == kReal ? p1 : make_float2(p1.x + q1.y, q1.x - p1.y);
  s_red[2][warp][lane] = make_float2(p2.x + q2.y, q2.x - p2.y);
  __syncthreads();
  if (warp < 3 && fv) {
    float2 sum = cz();
#pragma unroll
    for (int w = 0; w < NW; ++w) sum = c_add(sum, s_red[warp][w][lane]);
    a.partials[(row * a.ntiles + j) * 3 + warp] = sum;
  }
}

// TBPTT(1) surrogate backward in (B,T,F) layout (no temporal adjoint).  One
// CTA per (tile, chain) in blockIdx order; every sub-tile starts from the
// entry state the forward saved for it, so one pass suffices.
template <int NW, int K, int S, bool FUSE_ACT>
__global__ void __launch_bounds__(NW * 32) btf_tbptt_bwd_kernel(const BtfArgs a) {
  constexpr int L = NW * K;
  static_assert(L == kBtfSub, "sub-tile length");
  __shared__ float2 s_y[2][NW][32];
  __shared__ float2 s_first[2][NW + 1][32];
  __shared__ float2 s_red[3][NW][32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int j = (int)(blockIdx.x / (unsigned)a.ngroups);
  const int64_t grp = blockIdx.x - (unsigned)j * (unsigned)a.ngroups;
  const int64_t bi = grp / a.nfb;
  const int64_t f = (grp - bi * a.nfb) * 32 + lane;
  const bool fv = f < a.F;
  const int64_t row = bi * a.F + f;
  const float2 lam = fv ? a.c1[f] : cz();
  const float2 t0 = fv ? a.c2[f] : cz();
  const float2 t1 = fv ? a.tap1[f] : cz();
  const int64_t base = bi * a.T * a.F + f;
  const int64_t tile0 = (int64_t)j * S * L;
  const float2 *xs = static_cast<const float2 *>(a.x);
  const float2 gK = c_pow2k(lam, ilog2(K));
  float2 Gw = cone();
  for (int w = 0; w < warp; ++w) Gw = c_mul(gK, Gw);

  // element-wise products on paired fp32 FMAs, as in btf_bwd_kernel
  const float2 T0X = make_float2(t0.x, t0.x), T0Y = make_float2(t0.y, -t0.y);
  const float2 T1X = make_float2(t1.x, t1.x), T1Y = make_float2(t1.y, -t1.y);
  float2 pc1 = cz(), qc1 = cz(), p0 = cz(), q0 = cz(), p1 = cz(), q1 = cz();
#pragma unroll 1
  for (int s = 0; s < S; ++s) {
    const int64_t tw = tile0 + (int64_t)s * L + (int64_t)warp * K;
    const float2 es = (fv && tile0 + (int64_t)s * L < a.T)
                          ? a.carries[row * a.csub + (int64_t)j * S + s]
                          : cz();
    float2 x[K], xp, b[K], go[K];
    if (s + 1 < S) {
      btf_prefetch<K, 8>(a.x, base - lane, tw + L, a, (int)(f - lane), lane);
      btf_prefetch<K, 8>(a.gout, base - lane, tw + L, a, (int)(f - lane), lane);
    }
    btf_drive<K, kTwoTap, true>(a, base, tw, fv, t0, t1, x, xp, b);
    btf_load_go<K>(a, base, tw, fv, true, go);
    float2 y = cz();
#pragma unroll
    for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
    s_y[s & 1][warp][lane] = y;
    __syncthreads();
    float2 Xw = cz();
    for (int w = 0; w < warp; ++w) Xw = c_fma(gK, Xw, s_y[s & 1][w][lane]);
    float2 e = c_fma(Gw, es, Xw);
    float2 yprev[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      yprev[k] = e;
      e = c_fma(lam, e, b[k]);
      if (FUSE_ACT) go[k] = c_relu_mask(go[k], e);
    }
    s_first[s & 1][warp][lane] = go[0];
    if (warp == NW - 1) {
      // cotangent of the first sample after this sub-tile (its lag tap)
      const int64_t tn = tw + K;
      float2 g_next = cz();
      if (fv && tn < a.T) {
        g_next = a.gout[base + tn * a.F];
        if (FUSE_ACT) {
          const float2 yn = c_fma(lam, e, c_fma(t1, x[K - 1], c_mul(t0, xs[base + tn * a.F])));
          g_next = c_relu_mask(g_next, yn);
        }
      }
      s_first[s & 1][NW][lane] = g_next;
    }
    __syncthreads();
    const float2 gn = s_first[s & 1][warp + 1][lane];
    const bool full = fv && tw + K <= a.T;
    int64_t idx = base + tw * a.F;
#pragma unroll
    for (int k = 0; k < K; ++k, idx += a.F) {
      const float2 g = go[k];
      const float2 g1 = (k + 1 < K) ? go[k + 1] : gn;
      const float2 gs = c_swap(g), g1s = c_swap(g1);
      if (full || (fv && tw + k < a.T)) {
        __stcs(static_cast<float2 *>(a.out) + idx, __ffma2_rn(T0X, g, __fmul2_rn(T0Y, gs)));
        __stcs(a.out2 + idx, __ffma2_rn(T1X, g1, __fmul2_rn(T1Y, g1s)));
      }
      const float2 gx = make_float2(g.x, g.x), gy = make_float2(g.y, g.y);
      pc1 = __ffma2_rn(yprev[k], gx, pc1);
      qc1 = __ffma2_rn(yprev[k], gy, qc1);
      p0 = __ffma2_rn(x[k], gx, p0);
      q0 = __ffma2_rn(x[k], gy, q0);
      const float2 xk1 = k > 0 ? x[k - 1] : xp;
      p1 = __ffma2_rn(xk1, gx, p1);
      q1 = __ffma2_rn(xk1, gy, q1);
    }
  }
  // conj(v) g = (v.x g.x + v.y g.y, v.x g.y - v.y g.x)
  s_red[0][warp][lane] = make_float2(pc1.x + qc1.y, qc1.x - pc1.y);
  s_red[1][warp][lane] = make_float2(p0.x + q0.y, q0.x - p0.y);
  s_red[2][warp][lane] = make_float2(p1.x + q1.y, q1.x - p1.y);
  __syncthreads();
  if (warp < 3 && fv) {
    float2 sum = cz();
#pragma unroll
    for (int w = 0; w < NW; ++w) sum = c_add(sum, s_red[warp][w][lane]);
    a.partials[(row * a.ntiles + j) * 3 + warp] = sum;
  }
}

}  // namespace btfs
}  // namespace rqf
