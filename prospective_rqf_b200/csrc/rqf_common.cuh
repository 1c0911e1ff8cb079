// Device-side building blocks shared by the scan kernels:
//   * complex float arithmetic on float2 (re, im),
//   * the affine-pair composition used by every tile scan,
//   * CTA-wide scans of (gate, value) pairs in forward and reverse time,
//   * warp-private shared-memory transposes between the coalesced "striped"
//     order of a global load and the "blocked" order (K consecutive time
//     steps per thread) that the per-thread recurrence needs,
//   * decoupled look-back flags with bounded waits and a device error latch.
//
// The recurrence y[t] = a[t]*y[t-1] + b[t] over a segment is the affine map
// y_out = G*y_in + X with (G, X) the composition of the per-step pairs; the
// composition of an earlier segment (g1, x1) followed by a later one (g2, x2)
// is (g2*g1, g2*x1 + x2) — the operator of rqf_models/ops/scan.py:23-25 and
// chunked_scan_kernel.py:_affine_combine (:50-57).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rqf {

typedef unsigned long long u64;

// ---------------------------------------------------------------- complex
__device__ __forceinline__ float2 cz() { return make_float2(0.f, 0.f); }
__device__ __forceinline__ float2 cone() { return make_float2(1.f, 0.f); }
__device__ __forceinline__ float2 c_add(float2 a, float2 b) {
  return make_float2(a.x + b.x, a.y + b.y);
}
__device__ __forceinline__ float2 c_conj(float2 a) { return make_float2(a.x, -a.y); }
__device__ __forceinline__ float2 c_mul(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
// a*b + c
__device__ __forceinline__ float2 c_fma(float2 a, float2 b, float2 c) {
  return make_float2(fmaf(a.x, b.x, fmaf(-a.y, b.y, c.x)),
                     fmaf(a.x, b.y, fmaf(a.y, b.x, c.y)));
}
// conj(a)*b + c
__device__ __forceinline__ float2 c_cfma(float2 a, float2 b, float2 c) {
  return make_float2(fmaf(a.x, b.x, fmaf(a.y, b.y, c.x)),
                     fmaf(a.x, b.y, fmaf(-a.y, b.x, c.y)));
}
// Complex products on paired fp32 FMAs (__ffma2_rn, two lanes per
// instruction): for a fixed complex a, a * v = (a.x, a.x) * v + (-a.y, a.y) *
// (v.y, v.x).  cpair(a) holds the two constant pairs; the swapped operand
// (v.y, v.x) is passed in so a caller can reuse it.
struct CPair {
  float2 re, im;
};
__device__ __forceinline__ CPair cpair(float2 a) {
  return {make_float2(a.x, a.x), make_float2(-a.y, a.y)};
}
__device__ __forceinline__ float2 c_swap(float2 v) { return make_float2(v.y, v.x); }
// a * v + c
__device__ __forceinline__ float2 cp_fma(const CPair &a, float2 v, float2 vs, float2 c) {
  return __ffma2_rn(a.re, v, __ffma2_rn(a.im, vs, c));
}
// a * v
__device__ __forceinline__ float2 cp_mul(const CPair &a, float2 v, float2 vs) {
  return __ffma2_rn(a.re, v, __fmul2_rn(a.im, vs));
}
// split-ReLU: relu(Re) + i relu(Im)   (rqf_models/backbones/rqf/utils/activations.py:14-18)
__device__ __forceinline__ float2 c_relu(float2 a) {
  return make_float2(a.x > 0.f ? a.x : 0.f, a.y > 0.f ? a.y : 0.f);
}
// mask g by split-ReLU'(y): relu'(0) = 0, as fbt_scan_kernel.py:181-185
__device__ __forceinline__ float2 c_relu_mask(float2 g, float2 y) {
  return make_float2(y.x > 0.f ? g.x : 0.f, y.y > 0.f ? g.y : 0.f);
}

__device__ __forceinline__ float2 shfl_up2(float2 v, int d) {
  return make_float2(__shfl_up_sync(0xffffffffu, v.x, d), __shfl_up_sync(0xffffffffu, v.y, d));
}
__device__ __forceinline__ float2 shfl_down2(float2 v, int d) {
  return make_float2(__shfl_down_sync(0xffffffffu, v.x, d),
                     __shfl_down_sync(0xffffffffu, v.y, d));
}
__device__ __forceinline__ float2 shfl_xor2(float2 v, int d) {
  return make_float2(__shfl_xor_sync(0xffffffffu, v.x, d), __shfl_xor_sync(0xffffffffu, v.y, d));
}

// a^(2^s) in double precision: used for the per-tile gate lambda^L of a
// time-invariant scan (L a power of two) so that the look-back multiplier
// carries no fp32 accumulation of L products.
__device__ __forceinline__ float2 c_pow2k(float2 a, int s) {
  double re = a.x, im = a.y;
  for (int i = 0; i < s; ++i) {
    double nr = re * re - im * im;
    double ni = 2.0 * re * im;
    re = nr;
    im = ni;
  }
  return make_float2((float)re, (float)im);
}

// ---------------------------------------------------------------- errors
__device__ int g_rqf_error;  // first error code latched since the last clear

__device__ __forceinline__ void latch_error(int code) { atomicCAS(&g_rqf_error, 0, code); }

// ------------------------------------------------------- look-back flags
// A published tile value is stored as 64-bit words (status << 32 | float bits)
// so each word is single-copy atomic and carries its own status:
//   0 = nothing yet, 1 = tile aggregate, 2 = inclusive prefix.
constexpr unsigned kAggregate = 1u;
constexpr unsigned kInclusive = 2u;
// Upper bound of polls of one predecessor before giving up (~0.3 s).
constexpr unsigned kSpinLimit = 1u << 20;
constexpr int kErrLookbackTimeout = 3;

__device__ __forceinline__ void st_relaxed_u64(u64 *p, u64 v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ u64 ld_relaxed_u64(const u64 *p) {
  u64 v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ u64 pack_word(float v, unsigned status) {
  return ((u64)status << 32) | (u64)__float_as_uint(v);
}

// Publish a complex value (2 words).
__device__ __forceinline__ void flag_publish2(u64 *p, float2 v, unsigned status) {
  st_relaxed_u64(p + 0, pack_word(v.x, status));
  st_relaxed_u64(p + 1, pack_word(v.y, status));
}
// Publish (gate, value) (4 words).
__device__ __forceinline__ void flag_publish4(u64 *p, float2 g, float2 v, unsigned status) {
  st_relaxed_u64(p + 0, pack_word(g.x, status));
  st_relaxed_u64(p + 1, pack_word(g.y, status));
  st_relaxed_u64(p + 2, pack_word(v.x, status));
  st_relaxed_u64(p + 3, pack_word(v.y, status));
}

// Exclusive prefix of the tile at processing position `pos` (pos >= 1) of a
// row whose tiles all have the same time-invariant gate M (= lambda^L).
// flags points at the row's 2-word slots, indexed by processing position.
__device__ __forceinline__ float2 lookback_const(const u64 *flags, int pos, float2 M) {
  float2 acc = cz(), mult = cone();
  int i = pos - 1;
  unsigned spins = 0, ns = 32;
  while (i >= 0) {
    const u64 w0 = ld_relaxed_u64(flags + 2 * i);
    const u64 w1 = ld_relaxed_u64(flags + 2 * i + 1);
    const unsigned s0 = (unsigned)(w0 >> 32), s1 = (unsigned)(w1 >> 32);
    if (s0 == 0u || s0 != s1) {
      if (++spins > kSpinLimit) {
        latch_error(kErrLookbackTimeout);
        break;
      }
      __nanosleep(ns);
      ns = ns < 256u ? ns * 2u : 256u;
      continue;
    }
    const float2 v = make_float2(__uint_as_float((unsigned)w0), __uint_as_float((unsigned)w1));
    acc = c_fma(mult, v, acc);
    if (s0 == kInclusive) break;
    mult = c_mul(mult, M);
    --i;
    spins = 0;
    ns = 32;
  }
  return acc;
}

// lookback_const reading kLookbackWin predecessors per round trip: when many
// tiles of a row are in flight (few long rows split into many tiles), the
// aggregates to combine before the first inclusive prefix arrive together.
// Words after the first one not yet published are read again next round.
constexpr int kLookbackWin = 4;
__device__ __forceinline__ float2 lookback_const_win(const u64 *flags, int pos, float2 M) {
  float2 acc = cz(), mult = cone();
  int i = pos - 1;
  unsigned spins = 0, ns = 32;
  while (i >= 0) {
    u64 w[2 * kLookbackWin];
#pragma unroll
    for (int q = 0; q < kLookbackWin; ++q) {
      const int k = i - q >= 0 ? i - q : 0;
      w[2 * q] = ld_relaxed_u64(flags + 2 * k);
      w[2 * q + 1] = ld_relaxed_u64(flags + 2 * k + 1);
    }
    int used = 0;
    bool done = false, stalled = false;
#pragma unroll
    for (int q = 0; q < kLookbackWin; ++q) {
      if (done || stalled || i - q < 0) continue;
      const unsigned s0 = (unsigned)(w[2 * q] >> 32), s1 = (unsigned)(w[2 * q + 1] >> 32);
      if (s0 == 0u || s0 != s1) {
        stalled = true;
        continue;
      }
      const float2 v =
          make_float2(__uint_as_float((unsigned)w[2 * q]), __uint_as_float((unsigned)w[2 * q + 1]));
      acc = c_fma(mult, v, acc);
      ++used;
      if (s0 == kInclusive) {
        done = true;
        continue;
      }
      mult = c_mul(mult, M);
    }
    if (done) break;
    i -= used;
    if (used == 0) {  // the nearest unread predecessor has published nothing yet
      if (++spins > kSpinLimit) {
        latch_error(kErrLookbackTimeout);
        break;
      }
      __nanosleep(ns);
      ns = ns < 256u ? ns * 2u : 256u;
    } else {
      spins = 0;
      ns = 32;
    }
  }
  return acc;
}

// Same for tiles with their own gate aggregates (time-varying recurrences).
__device__ __forceinline__ float2 lookback_pair(const u64 *flags, int pos) {
  float2 acc = cz(), mult = cone();
  int i = pos - 1;
  unsigned spins = 0, ns = 32;
  while (i >= 0) {
    u64 w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) w[q] = ld_relaxed_u64(flags + 4 * i + q);
    const unsigned s = (unsigned)(w[0] >> 32);
    bool ok = s != 0u;
#pragma unroll
    for (int q = 1; q < 4; ++q) ok = ok && ((unsigned)(w[q] >> 32) == s);
    if (!ok) {
      if (++spins > kSpinLimit) {
        latch_error(kErrLookbackTimeout);
        break;
      }
      __nanosleep(ns);
      ns = ns < 256u ? ns * 2u : 256u;
      continue;
    }
    const float2 g = make_float2(__uint_as_float((unsigned)w[0]), __uint_as_float((unsigned)w[1]));
    const float2 v = make_float2(__uint_as_float((unsigned)w[2]), __uint_as_float((unsigned)w[3]));
    acc = c_fma(mult, v, acc);
    if (s == kInclusive) break;
    mult = c_mul(mult, g);
    --i;
    spins = 0;
    ns = 32;
  }
  return acc;
}

// --------------------------------------------------------- CTA scans
// Scan of per-thread affine pairs (g, a) over the CTA in increasing thread
// order.  Returns the exclusive composition (G, X) of all earlier threads and
// the CTA total (Gt, At).  s_warp needs NT/32 float4 slots.  Contains one
// __syncthreads(); every thread of the CTA must call it.
template <int NT>
__device__ __forceinline__ void cta_scan_fwd(float2 g, float2 a, float2 &G, float2 &X, float2 &Gt,
                                             float2 &At, float4 *s_warp) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float2 gp = shfl_up2(g, o), ap = shfl_up2(a, o);
    if (lane >= o) {
      a = c_fma(g, ap, a);
      g = c_mul(g, gp);
    }
  }
  float2 ge = shfl_up2(g, 1), ae = shfl_up2(a, 1);
  if (lane == 0) {
    ge = cone();
    ae = cz();
  }
  if (lane == 31) s_warp[warp] = make_float4(g.x, g.y, a.x, a.y);
  __syncthreads();
  float2 Gw = cone(), Xw = cz();
  float2 Gall = cone(), Xall = cz();
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const float4 q = s_warp[w];
    const float2 gw = make_float2(q.x, q.y), aw = make_float2(q.z, q.w);
    if (w == warp) {
      Gw = Gall;
      Xw = Xall;
    }
    Xall = c_fma(gw, Xall, aw);
    Gall = c_mul(gw, Gall);
  }
  X = c_fma(ge, Xw, ae);
  G = c_mul(ge, Gw);
  Gt = Gall;
  At = Xall;
}

// Reverse-time counterpart: threads composed from the last to the first.
// (G, X) composes all LATER threads; (Gt, At) is the CTA total.
template <int NT>
__device__ __forceinline__ void cta_scan_rev(float2 g, float2 a, float2 &G, float2 &X, float2 &Gt,
                                             float2 &At, float4 *s_warp) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float2 gp = shfl_down2(g, o), ap = shfl_down2(a, o);
    if (lane + o < 32) {
      a = c_fma(g, ap, a);
      g = c_mul(g, gp);
    }
  }
  float2 ge = shfl_down2(g, 1), ae = shfl_down2(a, 1);
  if (lane == 31) {
    ge = cone();
    ae = cz();
  }
  if (lane == 0) s_warp[warp] = make_float4(g.x, g.y, a.x, a.y);
  __syncthreads();
  float2 Gw = cone(), Xw = cz();
  float2 Gall = cone(), Xall = cz();
#pragma unroll
  for (int w = NW - 1; w >= 0; --w) {
    const float4 q = s_warp[w];
    const float2 gw = make_float2(q.x, q.y), aw = make_float2(q.z, q.w);
    if (w == warp) {
      Gw = Gall;
      Xw = Xall;
    }
    Xall = c_fma(gw, Xall, aw);
    Gall = c_mul(gw, Gall);
  }
  X = c_fma(ge, Xw, ae);
  G = c_mul(ge, Gw);
  Gt = Gall;
  At = Xall;
}

// ------------------------------------------- time-invariant CTA scans
// For a constant gate lambda the composition of n steps has gate lambda^n.
// Building lambda^n by repeated multiplication of one rounded lambda^K makes
// its phase error grow linearly with n (255 products per 2048-sample tile),
// which breaks fp32 parity for undamped poles (|lambda| -> 1) over long
// sequences.  Instead every power is taken from a table pw[i] = lambda^(2^i)
// built in double precision, so each power carries at most log2(n) roundings.

// Fill pw[0..n) with lambda^(2^i) (one thread; double precision squaring).
__device__ __forceinline__ void pow2_table(float2 lam, float2 *pw, int n) {
  double re = lam.x, im = lam.y;
  for (int i = 0; i < n; ++i) {
    pw[i] = make_float2((float)re, (float)im);
    const double nr = re * re - im * im;
    const double ni = 2.0 * re * im;
    re = nr;
    im = ni;
  }
}

// lambda^(2^s * n) from the table (conjugated when CONJ).
template <bool CONJ>
__device__ __forceinline__ float2 pow_from_table(const float2 *pw, int s, unsigned n) {
  float2 r = cone();
  for (int i = 0; n; ++i, n >>= 1)
    if (n & 1u) r = c_mul(r, CONJ ? c_conj(pw[s + i]) : pw[s + i]);
  return r;
}

// Forward scan of per-thread aggregates `a` (K samples each, zero entry) with
// the constant gate lambda: returns the exclusive composition (G, X) of the
// earlier threads (G = lambda^(K*tid)) and the CTA total value At.
template <int NT, int LK>
__device__ __forceinline__ void cta_scan_const_fwd(float2 a, const float2 *pw, float2 &G, float2 &X,
                                                   float2 &At, float2 *s_warp) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int d = 0; d < 5; ++d) {
    const int o = 1 << d;
    const float2 v = shfl_up2(a, o);
    if (lane >= o) a = c_fma(pw[LK + d], v, a);
  }
  float2 ae = shfl_up2(a, 1);
  if (lane == 0) ae = cz();
  if (lane == 31) s_warp[warp] = a;
  __syncthreads();
  const float2 gw = pw[LK + 5];  // lambda^(32K)
  float2 Xw = cz(), Xall = cz();
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    if (w == warp) Xw = Xall;
    Xall = c_fma(gw, Xall, s_warp[w]);
  }
  X = c_fma(pow_from_table<false>(pw, LK, lane), Xw, ae);
  G = pow_from_table<false>(pw, LK, threadIdx.x);
  At = Xall;
}

// Reverse-time counterpart with gate conj(lambda): (G, X) compose the LATER
// threads (G = conj(lambda)^(K*(NT-1-tid))); At is the CTA total.
template <int NT, int LK>
__device__ __forceinline__ void cta_scan_const_rev(float2 a, const float2 *pw, float2 &G, float2 &X,
                                                   float2 &At, float2 *s_warp) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int d = 0; d < 5; ++d) {
    const int o = 1 << d;
    const float2 v = shfl_down2(a, o);
    if (lane + o < 32) a = c_fma(c_conj(pw[LK + d]), v, a);
  }
  float2 ae = shfl_down2(a, 1);
  if (lane == 31) ae = cz();
  if (lane == 0) s_warp[warp] = a;
  __syncthreads();
  const float2 gw = c_conj(pw[LK + 5]);
  float2 Xw = cz(), Xall = cz();
#pragma unroll
  for (int w = NW - 1; w >= 0; --w) {
    if (w == warp) Xw = Xall;
    Xall = c_fma(gw, Xall, s_warp[w]);
  }
  X = c_fma(pow_from_table<true>(pw, LK, 31 - lane), Xw, ae);
  G = pow_from_table<true>(pw, LK, NT - 1 - threadIdx.x);
  At = Xall;
}

// Cross-warp step of the constant-gate CTA scans: from the per-warp totals
// s_warp[0..NW) (each warp spanning 32K samples, gate pw[g0] = lambda^(32K)),
// Xw = the composition of the warps before this one (after it when REV, gate
// conj(lambda)) and Xall = the CTA total.  Lanes 0..NW-1 of every warp run a
// log2(NW)-step shuffle scan (gate pw[g0+d] for distance 2^d) instead of each
// thread composing all NW totals serially; lanes >= NW hold zero, so the
// neighbour of the first (last when REV) warp reads zero.
template <int NW, bool REV>
__device__ __forceinline__ void warp_totals(const float2 *s_warp, const float2 *pw, int g0,
                                            float2 &Xw, float2 &Xall) {
  static_assert(NW >= 1 && NW < 32 && (NW & (NW - 1)) == 0, "NW must be a power of two < 32");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float2 v = lane < NW ? s_warp[lane] : cz();
#pragma unroll
  for (int d = 0; (1 << d) < NW; ++d) {
    const int o = 1 << d;
    if constexpr (REV) {
      const float2 u = shfl_down2(v, o);
      if (lane + o < NW) v = c_fma(c_conj(pw[g0 + d]), u, v);
    } else {
      const float2 u = shfl_up2(v, o);
      if (lane >= o) v = c_fma(pw[g0 + d], u, v);
    }
  }
  const int src = REV ? warp + 1 : (warp - 1) & 31;
  Xw = make_float2(__shfl_sync(0xffffffffu, v.x, src), __shfl_sync(0xffffffffu, v.y, src));
  const int tot = REV ? 0 : NW - 1;
  Xall = make_float2(__shfl_sync(0xffffffffu, v.x, tot), __shfl_sync(0xffffffffu, v.y, tot));
}

// Scans for the row-sequential kernels, where the state entering the tile is
// known before the scan: it is folded into the first thread's aggregate, so
// the scan directly yields each thread's entry state E and the state after the
// tile At, and no per-thread power lambda^(K*tid) is needed.  lanepow is
// lambda^(K*lane) (forward) or conj(lambda)^(K*(31-lane)) (reverse), cached
// per row by the caller.
template <int NT, int LK>
__device__ __forceinline__ void cta_scan_entry_fwd(float2 a, float2 entry, const float2 *pw,
                                                   float2 lanepow, float2 &E, float2 &At,
                                                   float2 *s_warp) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) a = c_fma(pw[LK], entry, a);
#pragma unroll
  for (int d = 0; d < 5; ++d) {
    const int o = 1 << d;
    const float2 v = shfl_up2(a, o);
    if (lane >= o) a = c_fma(pw[LK + d], v, a);
  }
  float2 ae = shfl_up2(a, 1);
  if (lane == 0) ae = cz();
  if (lane == 31) s_warp[warp] = a;
  __syncthreads();
  float2 Xw, Xall;
  warp_totals<NW, false>(s_warp, pw, LK + 5, Xw, Xall);
  E = threadIdx.x == 0 ? entry : c_fma(lanepow, Xw, ae);
  At = Xall;
}

template <int NT, int LK>
__device__ __forceinline__ void cta_scan_entry_rev(float2 a, float2 entry, const float2 *pw,
                                                   float2 lanepow, float2 &E, float2 &At,
                                                   float2 *s_warp) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == NT - 1) a = c_fma(c_conj(pw[LK]), entry, a);
#pragma unroll
  for (int d = 0; d < 5; ++d) {
    const int o = 1 << d;
    const float2 v = shfl_down2(a, o);
    if (lane + o < 32) a = c_fma(c_conj(pw[LK + d]), v, a);
  }
  float2 ae = shfl_down2(a, 1);
  if (lane == 31) ae = cz();
  if (lane == 0) s_warp[warp] = a;
  __syncthreads();
  float2 Xw, Xall;
  warp_totals<NW, true>(s_warp, pw, LK + 5, Xw, Xall);
  E = threadIdx.x == NT - 1 ? entry : c_fma(lanepow, Xw, ae);
  At = Xall;
}

// Cross-warp step of the time-varying-gate CTA scans: s_warp[w] = (gate, value)
// of warp w's samples as a float4.  Lanes 0..NW-1 of every warp compose them
// with a log2(NW)-step shuffle scan; lanes >= NW hold the identity (1, 0).
// Xw = the value entering this warp, Xall = the CTA total, as warp_totals.
template <int NW, bool REV>
__device__ __forceinline__ void warp_pair_totals(const float4 *s_warp, float2 &Xw, float2 &Xall) {
  static_assert(NW >= 1 && NW < 32 && (NW & (NW - 1)) == 0, "NW must be a power of two < 32");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float2 g = cone(), v = cz();
  if (lane < NW) {
    const float4 q = s_warp[lane];
    g = make_float2(q.x, q.y);
    v = make_float2(q.z, q.w);
  }
#pragma unroll
  for (int o = 1; o < NW; o <<= 1) {
    const float2 gp = REV ? shfl_down2(g, o) : shfl_up2(g, o);
    const float2 vp = REV ? shfl_down2(v, o) : shfl_up2(v, o);
    if (REV ? lane + o < NW : lane >= o) {
      v = c_fma(g, vp, v);
      g = c_mul(g, gp);
    }
  }
  const int src = REV ? warp + 1 : (warp - 1) & 31;
  Xw = make_float2(__shfl_sync(0xffffffffu, v.x, src), __shfl_sync(0xffffffffu, v.y, src));
  const int tot = REV ? 0 : NW - 1;
  Xall = make_float2(__shfl_sync(0xffffffffu, v.x, tot), __shfl_sync(0xffffffffu, v.y, tot));
}

// Generic (time-varying gate) counterparts of cta_scan_entry_*: each thread
// contributes the composition (g, a) of its K samples; the known entry state
// is folded into the first thread (last thread in reverse).  s_warp needs
// NT/32 float4 slots and must not be reused before the next __syncthreads.
template <int NT>
__device__ __forceinline__ void cta_scan_pair_entry_fwd(float2 g, float2 a, float2 entry,
                                                        float2 &E, float2 &At, float4 *s_warp) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) a = c_fma(g, entry, a);
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float2 gp = shfl_up2(g, o), ap = shfl_up2(a, o);
    if (lane >= o) {
      a = c_fma(g, ap, a);
      g = c_mul(g, gp);
    }
  }
  float2 ge = shfl_up2(g, 1), ae = shfl_up2(a, 1);
  if (lane == 0) {
    ge = cone();
    ae = cz();
  }
  if (lane == 31) s_warp[warp] = make_float4(g.x, g.y, a.x, a.y);
  __syncthreads();
  float2 Xw, Xall;
  warp_pair_totals<NW, false>(s_warp, Xw, Xall);
  E = threadIdx.x == 0 ? entry : c_fma(ge, Xw, ae);
  At = Xall;
}

template <int NT>
__device__ __forceinline__ void cta_scan_pair_entry_rev(float2 g, float2 a, float2 entry,
                                                        float2 &E, float2 &At, float4 *s_warp) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == NT - 1) a = c_fma(g, entry, a);
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float2 gp = shfl_down2(g, o), ap = shfl_down2(a, o);
    if (lane + o < 32) {
      a = c_fma(g, ap, a);
      g = c_mul(g, gp);
    }
  }
  float2 ge = shfl_down2(g, 1), ae = shfl_down2(a, 1);
  if (lane == 31) {
    ge = cone();
    ae = cz();
  }
  if (lane == 0) s_warp[warp] = make_float4(g.x, g.y, a.x, a.y);
  __syncthreads();
  float2 Xw, Xall;
  warp_pair_totals<NW, true>(s_warp, Xw, Xall);
  E = threadIdx.x == NT - 1 ? entry : c_fma(ge, Xw, ae);
  At = Xall;
}

// Sum a complex value over the CTA; the result is valid in thread 0.
// s_red needs NT/32 float2 slots.  Contains one __syncthreads().
template <int NT>
__device__ __forceinline__ float2 cta_sum(float2 v, float2 *s_red) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = c_add(v, shfl_xor2(v, o));
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  float2 s = cz();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int w = 0; w < NW; ++w) s = c_add(s, s_red[w]);
  }
  return s;
}

// --------------------------------------------- warp-private transposes
// A warp owns 32*K consecutive complex samples.  "Striped": lane l holds the
// float4 pairs v*32 + l (v < K/2) — what a coalesced 16-byte load returns.
// "Blocked": lane l holds samples l*K .. l*K+K-1.  The XOR swizzle on the
// float4 slot index keeps both access patterns free of bank conflicts for
// K in {4, 8, 16}.
template <int K>
__device__ __forceinline__ int swz(int p) {
  return p ^ ((p >> 3) & (K / 2 - 1));
}

template <int K>
__device__ __forceinline__ void striped_to_blocked(float4 *wbuf, const float4 (&s)[K / 2],
                                                   float2 (&b)[K], int lane) {
#pragma unroll
  for (int v = 0; v < K / 2; ++v) wbuf[swz<K>(v * 32 + lane)] = s[v];
  __syncwarp();
#pragma unroll
  for (int m = 0; m < K / 2; ++m) {
    const float4 q = wbuf[swz<K>(lane * (K / 2) + m)];
    b[2 * m] = make_float2(q.x, q.y);
    b[2 * m + 1] = make_float2(q.z, q.w);
  }
  __syncwarp();
}

template <int K>
__device__ __forceinline__ void blocked_to_striped(float4 *wbuf, const float2 (&b)[K],
                                                   float4 (&s)[K / 2], int lane) {
#pragma unroll
  for (int m = 0; m < K / 2; ++m)
    wbuf[swz<K>(lane * (K / 2) + m)] =
        make_float4(b[2 * m].x, b[2 * m].y, b[2 * m + 1].x, b[2 * m + 1].y);
  __syncwarp();
#pragma unroll
  for (int v = 0; v < K / 2; ++v) s[v] = wbuf[swz<K>(v * 32 + lane)];
  __syncwarp();
}

// ---------------------------------------------------- cp.async staging
// Asynchronous global -> shared copies (the copy engine path that bypasses
// registers).  `pred == false` zero-fills the destination without reading
// global memory (the source address is still kept inside the tensor).
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool pred) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n)
               : "memory");
}
// Unpredicated form: the whole 16 bytes are in range.
__device__ __forceinline__ void cp_async16_full(void *smem, const void *gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async8(void *smem, const void *gmem, bool pred) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  const int n = pred ? 8 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(s), "l"(gmem), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem, bool pred) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  const int n = pred ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Read this thread's K blocked samples from a warp region written in the
// swizzled striped order (see striped_to_blocked).
template <int K>
__device__ __forceinline__ void read_blocked(const float4 *wbuf, float2 (&b)[K], int lane) {
#pragma unroll
  for (int m = 0; m < K / 2; ++m) {
    const float4 q = wbuf[swz<K>(lane * (K / 2) + m)];
    b[2 * m] = make_float2(q.x, q.y);
    b[2 * m + 1] = make_float2(q.z, q.w);
  }
}

// Sample q (0 <= q < 32K) of a warp region stored in swizzled striped order.
template <int K>
__device__ __forceinline__ float2 read_sample(const float4 *wbuf, int q) {
  const float4 v = wbuf[swz<K>(q >> 1)];
  return (q & 1) ? make_float2(v.z, v.w) : make_float2(v.x, v.y);
}

// Streaming 16-byte load / store (data is touched once per kernel).
__device__ __forceinline__ float4 ld_stream4(const float2 *p) {
  return __ldcs(reinterpret_cast<const float4 *>(p));
}
__device__ __forceinline__ void st_stream4(float2 *p, float4 v) {
  __stcs(reinterpret_cast<float4 *>(p), v);
}

}  // namespace rqf
