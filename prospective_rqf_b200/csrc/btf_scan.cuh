// Diagonal scans in (batch, time, filters) layout — filters innermost.
//
// Serves rqf_models/ops/chunked_scan_kernel.py:_triton_chunked_scan (:340)
// and _triton_chunked_scan_prospective (:506) without their (B,T,F) <-> (B,F,T)
// permutes (chunked_scan_kernel.py:212-214, :249, :272-275, :302):
//   PLAIN    y[t] = c1*y[t-1] + c2*u[t]                 (u complex)
//   REAL     same with u real (scan.py:366 promotes; the values are identical)
//   TWO_TAP  y[t] = c1*y[t-1] + tap0*x[t] + tap1*x[t-1]
//
// Work decomposition.  A "chain" is one batch index and a block of 32 adjacent
// channels: lane = channel, so each time step of a chain is one coalesced
// 256-byte row.  A sub-tile is 64 time steps of a chain; each of the 8 warps
// runs its lanes' recurrences serially over 8 consecutive steps and the warps
// are composed through shared memory.  A tile is S consecutive sub-tiles (the
// forward S <= 4, the backward S <= 2); the per-tile entry states saved by the
// forward are kept per sub-tile, so the two directions may tile differently.
//
// One CTA per tile, in atomic-ticket order (tile-major across chains, so the
// resident CTAs spread over the chains and every tile a look-back waits on
// belongs to a CTA that is already running).  The whole tile is staged in
// shared memory by cp.async at the start (one commit group per sub-tile, all
// in flight together), so each sample crosses HBM once and no pass re-reads
// global memory:
//   pass 1  per sub-tile, the drive (stored over the input in shared memory
//           for complex inputs), the warps' aggregates with zero entry, each
//           thread's prefix over the earlier warps, the sub-tile total;
//   link    the tile total, a decoupled look-back (several predecessors per
//           round trip) for the tile's entry, the inclusive prefix, the
//           sub-tile entry states (saved for the backward);
//   pass 2  the outputs from the entry states, reading the stored drive.
// A header of per-channel constants (c1 and its powers from a
// double-precision table, the drive coefficients, the saved entry states)
// rides in the first copy group.
//
// The backward (tiles in reverse time order) recomputes y from the saved
// entry states and fuses the adjoint with grad_u / grad_x and the
// coefficient-gradient partial sums (one partial per tile, reduced in fixed
// order afterwards).  The TBPTT(1) backward has no adjoint: its sub-tiles are
// independent, each starting from its saved entry state.
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
  float2 *carries;     // (B*F, nsub): entry state of every sub-tile, row = b*F + f
  float2 *partials;    // (B*F, ntiles, 3)
  u64 *flags;          // (B*F, ntiles, 2)
  unsigned *ticket;
  const float2 *pw;    // (kBtfPowLevels, F): c1^(2^i)
  // multi-oscillator scans: F = Fin << log2n oscillator channels, the
  // C-weights cw (F,), inputs / outputs (B,T,Fin), the C-weight gradient's
  // partials (B*F, ntiles, 3; slot 0).  Otherwise cw = null, Fin = F, log2n = 0.
  const float2 *cw;
  float2 *partials2;
  int64_t Fin;
  int log2n;
  int64_t B, T, F;
  int nfb;      // channel blocks of 32
  int ngroups;  // chains: B * nfb
  int nsub;     // sub-tiles along time
  int ntiles;   // tiles of this launch along time: ceil(nsub / S)
  int S;        // sub-tiles per tile of this launch
  int log2S;
};

constexpr int kBtfSub = 64;  // time steps of a sub-tile
constexpr int kBtfLog2Sub = 6;
constexpr int kBtfWarps = 8;
constexpr int kBtfK = kBtfSub / kBtfWarps;  // steps per thread
constexpr int kBtfThreads = kBtfWarps * 32;
constexpr int kBtfMaxFwdS = 4, kBtfMaxBwdS = 2, kBtfTbpttS = 4;
constexpr int kBtfPowLevels = kBtfLog2Sub + 3;  // c1^(2^i), i <= log2(64 * 4)
static_assert(kBtfK == 8, "lambda^(8*warp) is assembled from the 8/16/32 power rows");

// Header rows (one float2 per lane = channel); kHCarry + s holds the saved
// entry state of the tile's sub-tile s (backward kinds).
enum BtfHdr { kHLam = 0, kHC2, kHT1, kHPow8, kHPow16, kHPow32, kHPow64, kHGate, kHCarry };

template <int DRIVE>
struct BtfElem {
  using T = float2;
};
template <>
struct BtfElem<kReal> {
  using T = float;
};

// One tile: chain (b, 32-channel block) and time tile j.
struct BtfTile {
  int64_t b, f0;
  int j;    // time tile
  int pos;  // processing position along the chain (look-back order)
};

__device__ __forceinline__ BtfTile btf_decode(const BtfArgs &a, unsigned tk, bool reverse) {
  BtfTile t;
  const int p = (int)(tk / (unsigned)a.ngroups);
  const int64_t grp = tk - (unsigned)p * (unsigned)a.ngroups;
  t.b = grp / a.nfb;
  t.f0 = (grp - t.b * a.nfb) * 32;
  t.pos = p;
  t.j = reverse ? a.ntiles - 1 - p : p;
  return t;
}

// Tile of this CTA: one atomic ticket, taken by thread 0.
__device__ __forceinline__ unsigned btf_ticket(const BtfArgs &a, unsigned *s_tk) {
  if (threadIdx.x == 0) *s_tk = atomicAdd(a.ticket, 1u);
  __syncthreads();
  return *s_tk;
}

// Copy rows [r0, r1) of a (B,T,F) tensor into a shared region of 32-element
// rows: region row r holds time step t0 + r (zero outside [0, T) and for
// channels >= F).  VEC: 16-byte copies (F a multiple of the elements per 16
// bytes and a 16-byte aligned tensor), else one element per copy.
template <typename E, bool VEC>
__device__ __forceinline__ void btf_copy_rows(E *dst, const E *src, const BtfArgs &a,
                                              const BtfTile &tl, int64_t t0, int r0, int r1) {
  const int tid = threadIdx.x;
  if constexpr (VEC) {
    constexpr int PER = 16 / (int)sizeof(E);  // elements per chunk
    constexpr int CPR = 32 / PER;             // chunks per row
    constexpr int RSTEP = kBtfThreads / CPR;  // rows per pass of the CTA
    const int q = tid % CPR;
    const int64_t f = tl.f0 + (int64_t)q * PER;
    const bool fv = f < a.F;
    int r = r0 + tid / CPR;
    int64_t t = t0 + r;
    int64_t off = (tl.b * a.T + t) * a.F + f;
    for (; r < r1; r += RSTEP, t += RSTEP, off += (int64_t)RSTEP * a.F) {
      const bool ok = fv && t >= 0 && t < a.T;
      cp_async16(dst + r * 32 + q * PER, ok ? src + off : src, ok);
    }
  } else {
    const int lane = tid & 31, warp = tid >> 5;
    const int64_t f = tl.f0 + lane;
    const bool fv = f < a.F;
    int r = r0 + warp;
    int64_t t = t0 + r;
    int64_t off = (tl.b * a.T + t) * a.F + f;
    for (; r < r1; r += kBtfWarps, t += kBtfWarps, off += (int64_t)kBtfWarps * a.F) {
      const bool ok = fv && t >= 0 && t < a.T;
      if constexpr (sizeof(E) == 8)
        cp_async8(dst + r * 32 + lane, ok ? src + off : src, ok);
      else
        cp_async4(dst + r * 32 + lane, ok ? src + off : src, ok);
    }
  }
}

// Multi-oscillator inputs: rows of a (B,T,Fin) tensor holding the 32 >> log2n
// input channels whose oscillators the chain's lanes carry, channel
// (f0 >> log2n) + q in column q of a 32-element row.
template <typename E>
__device__ __forceinline__ void btf_copy_narrow(E *dst, const E *src, const BtfArgs &a,
                                                const BtfTile &tl, int64_t t0, int r0, int r1) {
  const int q = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t fi = (tl.f0 >> a.log2n) + q;
  const bool fv = q < (32 >> a.log2n) && fi < a.Fin;
  int r = r0 + warp;
  int64_t t = t0 + r;
  int64_t off = (tl.b * a.T + t) * a.Fin + fi;
  for (; r < r1; r += kBtfWarps, t += kBtfWarps, off += (int64_t)kBtfWarps * a.Fin) {
    const bool ok = fv && t >= 0 && t < a.T;
    if constexpr (sizeof(E) == 8)
      cp_async8(dst + r * 32 + q, ok ? src + off : src, ok);
    else
      cp_async4(dst + r * 32 + q, ok ? src + off : src, ok);
  }
}

// Header copies: rows kHLam..kHGate (one per warp) and, for NCARRY > 0, the
// saved entry states of sub-tiles first_sub .. first_sub+NCARRY-1 (warp 0).
template <int DRIVE, int NCARRY>
__device__ __forceinline__ void btf_copy_header(float2 *hdr, const BtfArgs &a, const BtfTile &tl,
                                                int log2_tile, int first_sub) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t f = tl.f0 + lane;
  const bool fv = f < a.F;
  const int64_t fc = fv ? f : 0;
  const float2 *src;
  bool ok = fv;
  switch (warp) {
    case kHLam: src = a.pw + fc; break;
    case kHC2: src = a.c2 + fc; break;
    case kHT1:  // tap1, or the C-weight of a multi-oscillator scan
      src = DRIVE == kTwoTap ? a.tap1 + fc : (a.cw ? a.cw + fc : a.c2);
      ok = fv && (DRIVE == kTwoTap || a.cw != nullptr);
      break;
    case kHPow8: src = a.pw + 3 * a.F + fc; break;
    case kHPow16: src = a.pw + 4 * a.F + fc; break;
    case kHPow32: src = a.pw + 5 * a.F + fc; break;
    case kHPow64: src = a.pw + 6 * a.F + fc; break;
    default: src = a.pw + (int64_t)log2_tile * a.F + fc; break;  // kHGate: lambda^(tile)
  }
  cp_async8(hdr + warp * 32 + lane, src, ok);
  if (NCARRY > 0 && warp == 0) {
#pragma unroll
    for (int q = 0; q < NCARRY; ++q) {
      const bool okc = fv && first_sub + q < a.nsub;
      cp_async8(hdr + (kHCarry + q) * 32 + lane,
                okc ? a.carries + (tl.b * a.F + fc) * a.nsub + first_sub + q : a.carries, okc);
    }
  }
}

// Per-tile constants of this lane's channel, from the header.
struct BtfConst {
  float2 lam, c2, t1, gK, gL, M;
  float2 Gw;   // lambda^(8*warp): from the sub-tile start to this warp's first step
  float2 Grw;  // conj(lambda)^(8*(7-warp)): from the sub-tile end back to this warp's end
};
__device__ __forceinline__ float2 btf_pow8n(const float2 *hdr, int lane, int n) {
  float2 g = cone();  // lambda^(8n), n < 8, from the lambda^8/16/32 rows
  if (n & 1) g = hdr[kHPow8 * 32 + lane];
  if (n & 2) g = c_mul(g, hdr[kHPow16 * 32 + lane]);
  if (n & 4) g = c_mul(g, hdr[kHPow32 * 32 + lane]);
  return g;
}
__device__ __forceinline__ BtfConst btf_consts(const float2 *hdr, int lane, int warp) {
  BtfConst c;
  c.lam = hdr[kHLam * 32 + lane];
  c.c2 = hdr[kHC2 * 32 + lane];
  c.t1 = hdr[kHT1 * 32 + lane];
  c.gK = hdr[kHPow8 * 32 + lane];
  c.gL = hdr[kHPow64 * 32 + lane];
  c.M = hdr[kHGate * 32 + lane];
  c.Gw = btf_pow8n(hdr, lane, warp);
  c.Grw = c_conj(btf_pow8n(hdr, lane, kBtfWarps - 1 - warp));
  return c;
}

// K + 1 consecutive rows (from row r) of this lane's channel: v[0] is the step
// before the thread's first.
template <typename E>
__device__ __forceinline__ void btf_rows9(const E *rows, int r, int col, float2 (&v)[kBtfK + 1]) {
#pragma unroll
  for (int k = 0; k <= kBtfK; ++k) {
    if constexpr (sizeof(E) == 4)
      v[k] = make_float2(rows[(r + k) * 32 + col], 0.f);
    else
      v[k] = rows[(r + k) * 32 + col];
  }
}

template <int DRIVE>
__device__ __forceinline__ float2 btf_drive1(const BtfConst &c, float2 x, float2 xprev) {
  return DRIVE == kTwoTap ? c_fma(c.t1, xprev, c_mul(c.c2, x)) : c_mul(c.c2, x);
}

// Forward output: the complex state, or (ABS) its magnitude |y| as float, the
// inference epilogue of rqf_models/ops/scan.py:sequential_scan_abs (:381-432).
template <bool ABS>
__device__ __forceinline__ void btf_store_y(void *out, int64_t idx, float2 e) {
  if constexpr (ABS)
    __stcs(static_cast<float *>(out) + idx, sqrtf(fmaf(e.x, e.x, e.y * e.y)));
  else
    __stcs(static_cast<float2 *>(out) + idx, e);
}

// Sum over the 1 << log2n adjacent lanes holding one filter's oscillators.
__device__ __forceinline__ float2 btf_group_sum(float2 v, int log2n) {
  for (int o = 1; o < (1 << log2n); o <<= 1) v = c_add(v, shfl_xor2(v, o));
  return v;
}

// Composition of the 8 warps' values v[w] with gate g per warp: sum g^(7-w) v[w].
__device__ __forceinline__ float2 btf_total8(const float2 (*v)[32], float2 g, int lane) {
  float2 X = cz();
#pragma unroll
  for (int w = 0; w < kBtfWarps; ++w) X = c_fma(g, X, v[w][lane]);
  return X;
}

template <int N>
__device__ __forceinline__ void cp_async_wait_rt(int n) {  // n < N pending groups
  if constexpr (N > 1) {
    if (n >= N - 1) {
      cp_async_wait<N - 1>();
      return;
    }
    cp_async_wait_rt<N - 1>(n);
  } else {
    cp_async_wait<0>();
  }
}

// Dynamic shared memory of the kernels below (bytes).
template <int DRIVE, int S>
__host__ __device__ constexpr size_t btf_fwd_smem() {
  return (size_t)kHCarry * 32 * sizeof(float2) +
         (size_t)(kBtfSub * S + 1) * 32 * sizeof(typename BtfElem<DRIVE>::T);
}
template <int DRIVE, int S>
__host__ __device__ constexpr size_t btf_bwd_smem() {
  return (size_t)(kHCarry + S) * 32 * sizeof(float2) +
         (size_t)(kBtfSub * S + 1) * 32 * sizeof(typename BtfElem<DRIVE>::T) +
         (size_t)kBtfSub * S * 32 * sizeof(float2);
}
constexpr size_t kBtfTbpttStage = (size_t)(kHCarry + 1) * 32 * sizeof(float2) +
                                  2 * (size_t)(kBtfSub + 1) * 32 * sizeof(float2);
constexpr size_t btf_tbptt_smem() { return 2 * kBtfTbpttStage; }

// ------------------------------------------------------------ forward
// ABS: write |y| (float) instead of y; a null carries pointer skips the saved
// entry states (no backward follows).  MOSC (PLAIN / REAL drives): the lanes
// are oscillators, 1 << log2n per input channel, and the output is their
// C-weighted sum per channel.
template <int DRIVE, bool VECX, int S, bool ABS = false, bool MOSC = false>
__global__ void __launch_bounds__(kBtfThreads, 3) btf_fwd_kernel(const BtfArgs a) {
  using E = typename BtfElem<DRIVE>::T;
  extern __shared__ __align__(16) unsigned char btf_dsm[];
  __shared__ float2 s_y[2][kBtfWarps][32];
  __shared__ float2 s_X[S][32];
  __shared__ float2 s_C[S][32];
  __shared__ float2 s_xl[32];  // TWO_TAP: x of the last step of the previous sub-tile
  __shared__ unsigned s_tk;
  static_assert(!MOSC || DRIVE != kTwoTap, "multi-oscillator scans have a one-tap drive");
  constexpr bool STORE_B = DRIVE != kReal && !MOSC;  // the drive replaces x in shared memory
  float2 *hdr = reinterpret_cast<float2 *>(btf_dsm);
  E *xs = reinterpret_cast<E *>(btf_dsm + (size_t)kHCarry * 32 * sizeof(float2));
  float2 *bs = reinterpret_cast<float2 *>(xs);  // the drive, when STORE_B
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const BtfTile tl = btf_decode(a, btf_ticket(a, &s_tk), false);
  const int64_t ts0 = (int64_t)tl.j * S * kBtfSub;  // first step of the tile; row r = step ts0-1+r

#pragma unroll
  for (int s = 0; s < S; ++s) {
    if (s == 0) btf_copy_header<DRIVE, 0>(hdr, a, tl, kBtfLog2Sub + a.log2S, 0);
    if constexpr (MOSC)
      btf_copy_narrow<E>(xs, static_cast<const E *>(a.x), a, tl, ts0 - 1, kBtfSub * s + 1,
                         kBtfSub * (s + 1) + 1);
    else
      btf_copy_rows<E, VECX>(xs, static_cast<const E *>(a.x), a, tl, ts0 - 1,
                             s > 0 ? kBtfSub * s + 1 : (DRIVE == kTwoTap ? 0 : 1),
                             kBtfSub * (s + 1) + 1);
    cp_async_commit();
  }

  BtfConst c{};
  float2 Xw[S];
  const int col = MOSC ? (lane >> a.log2n) : lane;  // x column of this lane
  const int rw = warp * kBtfK;  // row of the step before this thread's first (in a sub-tile)
#pragma unroll
  for (int s = 0; s < S; ++s) {
    cp_async_wait_rt<S>(S - 1 - s);
    __syncthreads();
    if (s == 0) c = btf_consts(hdr, lane, warp);
    float2 v[kBtfK + 1];
    btf_rows9(xs, kBtfSub * s + rw, col, v);
    if (DRIVE == kTwoTap && s > 0 && warp == 0) v[0] = s_xl[lane];
    float2 b[kBtfK];
#pragma unroll
    for (int k = 0; k < kBtfK; ++k) b[k] = btf_drive1<DRIVE>(c, v[k + 1], v[k]);
    float2 y = cz();
#pragma unroll
    for (int k = 0; k < kBtfK; ++k) y = c_fma(c.lam, y, b[k]);
    s_y[s & 1][warp][lane] = y;
    __syncthreads();  // aggregates complete; every x of this sub-tile has been read
    if constexpr (STORE_B) {
#pragma unroll
      for (int k = 0; k < kBtfK; ++k) bs[(kBtfSub * s + rw + 1 + k) * 32 + lane] = b[k];
      if (DRIVE == kTwoTap && warp == kBtfWarps - 1) s_xl[lane] = v[kBtfK];
    }
    float2 X = cz();
    for (int w = 0; w < warp; ++w) X = c_fma(c.gK, X, s_y[s & 1][w][lane]);
    Xw[s] = X;
    if (warp == (s & 7)) s_X[s][lane] = btf_total8(s_y[s & 1], c.gK, lane);
  }
  __syncthreads();
  const int64_t f = tl.f0 + lane;
  if (warp == 0) {  // link: tile total, look-back, entry states of the sub-tiles
    float2 XT = cz();
#pragma unroll
    for (int s = 0; s < S; ++s) XT = c_fma(c.gL, XT, s_X[s][lane]);
    float2 C = cz();
    if (f < a.F) {
      const int64_t row = tl.b * a.F + f;
      u64 *fl = a.flags + row * (int64_t)a.ntiles * 2;
      const bool has_next = tl.j + 1 < a.ntiles;
      if (tl.j == 0) {
        if (has_next) flag_publish2(fl, XT, kInclusive);
      } else {
        if (has_next) flag_publish2(fl + 2 * tl.j, XT, kAggregate);
        C = lookback_const_win(fl, tl.j, c.M);
        if (has_next) flag_publish2(fl + 2 * tl.j, c_fma(c.M, C, XT), kInclusive);
      }
    }
#pragma unroll
    for (int s = 0; s < S; ++s) {
      s_C[s][lane] = C;
      const int sub = tl.j * S + s;
      if (a.carries && f < a.F && sub < a.nsub) a.carries[(tl.b * a.F + f) * a.nsub + sub] = C;
      C = c_fma(c.gL, C, s_X[s][lane]);
    }
  }
  __syncthreads();
  // pass 2: outputs
  if constexpr (MOSC) {  // C-weighted sum over each filter's oscillators
    const bool lead = (lane & ((1 << a.log2n) - 1)) == 0 && f < a.F;
    int64_t yo = (tl.b * a.T + ts0 + rw) * a.Fin + (f >> a.log2n);
#pragma unroll 1
    for (int s = 0; s < S; ++s, yo += (int64_t)kBtfSub * a.Fin) {
      float2 e = c_fma(c.Gw, s_C[s][lane], Xw[s]);
      const int64_t left = a.T - (ts0 + kBtfSub * s + rw);
      const int kmax = left < kBtfK ? (int)left : kBtfK;
      float2 v[kBtfK + 1];
      btf_rows9(xs, kBtfSub * s + rw, col, v);
      int64_t p = yo;
#pragma unroll
      for (int k = 0; k < kBtfK; ++k, p += a.Fin) {
        e = c_fma(c.lam, e, btf_drive1<DRIVE>(c, v[k + 1], v[k]));
        const float2 o = btf_group_sum(c_mul(c.t1, e), a.log2n);
        if (lead && k < kmax) btf_store_y<ABS>(a.out, p, o);
      }
    }
  } else if (f < a.F) {
    int64_t yo = (tl.b * a.T + ts0 + rw) * a.F + f;
#pragma unroll 1
    for (int s = 0; s < S; ++s, yo += (int64_t)kBtfSub * a.F) {
      float2 e = c_fma(c.Gw, s_C[s][lane], Xw[s]);
      const int64_t left = a.T - (ts0 + kBtfSub * s + rw);
      const int kmax = left < kBtfK ? (int)left : kBtfK;
      float2 b[kBtfK];
      if constexpr (STORE_B) {
#pragma unroll
        for (int k = 0; k < kBtfK; ++k) b[k] = bs[(kBtfSub * s + rw + 1 + k) * 32 + lane];
      } else {
        float2 v[kBtfK + 1];
        btf_rows9(xs, kBtfSub * s + rw, lane, v);
#pragma unroll
        for (int k = 0; k < kBtfK; ++k) b[k] = btf_drive1<DRIVE>(c, v[k + 1], v[k]);
      }
      int64_t p = yo;
#pragma unroll
      for (int k = 0; k < kBtfK; ++k, p += a.F) {
        e = c_fma(c.lam, e, b[k]);
        if (k < kmax) btf_store_y<ABS>(a.out, p, e);
      }
    }
  }
}

// ------------------------------------------------------------ backward
// Tiles run in reverse time order (processing position p = tile ntiles-1-p).
// MOSC: multi-oscillator scan (see the forward); the cotangent of oscillator s
// is conj(cw_s) gy[f], grad_u[f] sums conj(c2_s) g_s over f's oscillators, and
// grad_cw_s = sum conj(y_s[t]) gy[t, f] goes to the second partials array.
template <int DRIVE, bool VECX, bool VECG, int S, bool MOSC = false>
__global__ void __launch_bounds__(kBtfThreads, 2) btf_bwd_kernel(const BtfArgs a) {
  static_assert(!MOSC || DRIVE != kTwoTap, "multi-oscillator scans have a one-tap drive");
  using E = typename BtfElem<DRIVE>::T;
  extern __shared__ __align__(16) unsigned char btf_dsm[];
  __shared__ float4 s_yh[S][kBtfWarps][32];  // (forward y, reverse h) per warp
  __shared__ float2 s_H[S][32];               // reverse sub-tile totals
  __shared__ float2 s_D[32];
  __shared__ float2 s_red[MOSC ? 4 : 3][kBtfWarps][32];
  __shared__ unsigned s_tk;
  float2 *hdr = reinterpret_cast<float2 *>(btf_dsm);
  E *xs = reinterpret_cast<E *>(btf_dsm + (size_t)(kHCarry + S) * 32 * sizeof(float2));
  float2 *gs = reinterpret_cast<float2 *>(reinterpret_cast<unsigned char *>(xs) +
                                          (size_t)(kBtfSub * S + 1) * 32 * sizeof(E));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const BtfTile tl = btf_decode(a, btf_ticket(a, &s_tk), true);
  const int64_t ts0 = (int64_t)tl.j * S * kBtfSub;

#pragma unroll
  for (int s = 0; s < S; ++s) {
    if (s == 0) btf_copy_header<DRIVE, S>(hdr, a, tl, kBtfLog2Sub + a.log2S, tl.j * S);
    if constexpr (MOSC) {
      btf_copy_narrow<E>(xs, static_cast<const E *>(a.x), a, tl, ts0 - 1, kBtfSub * s + 1,
                         kBtfSub * (s + 1) + 1);
      btf_copy_narrow<float2>(gs, a.gout, a, tl, ts0, kBtfSub * s, kBtfSub * (s + 1));
    } else {
      btf_copy_rows<E, VECX>(xs, static_cast<const E *>(a.x), a, tl, ts0 - 1,
                             s > 0 ? kBtfSub * s + 1 : (DRIVE == kTwoTap ? 0 : 1),
                             kBtfSub * (s + 1) + 1);
      btf_copy_rows<float2, VECG>(gs, a.gout, a, tl, ts0, kBtfSub * s, kBtfSub * (s + 1));
    }
    cp_async_commit();
  }

  BtfConst c{};
  const int rw = warp * kBtfK;
  const int col = MOSC ? (lane >> a.log2n) : lane;  // x / cotangent column of this lane
  // cotangent of this lane's state at stage row r
  auto gcot = [&](int r) {
    const float2 g = gs[r * 32 + col];
    return MOSC ? c_cfma(c.t1, g, cz()) : g;
  };
#pragma unroll
  for (int s = 0; s < S; ++s) {
    cp_async_wait_rt<S>(S - 1 - s);
    __syncthreads();
    if (s == 0) c = btf_consts(hdr, lane, warp);
    float2 v[kBtfK + 1];
    btf_rows9(xs, kBtfSub * s + rw, col, v);
    float2 y = cz(), h = cz();
#pragma unroll
    for (int k = 0; k < kBtfK; ++k) y = c_fma(c.lam, y, btf_drive1<DRIVE>(c, v[k + 1], v[k]));
    const float2 mu = c_conj(c.lam);
#pragma unroll
    for (int k = kBtfK - 1; k >= 0; --k) h = c_fma(mu, h, gcot(kBtfSub * s + rw + k));
    s_yh[s][warp][lane] = make_float4(y.x, y.y, h.x, h.y);
  }
  __syncthreads();
  const float2 mu = c_conj(c.lam), muK = c_conj(c.gK), muL = c_conj(c.gL);
  if (warp < S) {  // reverse sub-tile totals
    float2 H = cz();
#pragma unroll
    for (int w = kBtfWarps - 1; w >= 0; --w)
      H = c_fma(muK, H, make_float2(s_yh[warp][w][lane].z, s_yh[warp][w][lane].w));
    s_H[warp][lane] = H;
  }
  __syncthreads();
  const int64_t f = tl.f0 + lane;
  const bool fv = f < a.F;
  if (warp == 0) {  // link: reverse tile total (sub-tile q sits 64q steps in), look-back
    float2 HT = s_H[S - 1][lane];
#pragma unroll
    for (int q = S - 2; q >= 0; --q) HT = c_fma(muL, HT, s_H[q][lane]);
    float2 D = cz();
    if (fv) {
      const int64_t row = tl.b * a.F + f;
      u64 *fl = a.flags + row * (int64_t)a.ntiles * 2;
      const bool has_next = tl.pos + 1 < a.ntiles;
      const float2 Mr = c_conj(c.M);
      if (tl.pos == 0) {
        if (has_next) flag_publish2(fl, HT, kInclusive);
      } else {
        if (has_next) flag_publish2(fl + 2 * tl.pos, HT, kAggregate);
        D = lookback_const_win(fl, tl.pos, Mr);
        if (has_next) flag_publish2(fl + 2 * tl.pos, c_fma(Mr, D, HT), kInclusive);
      }
    }
    s_D[lane] = D;
  }
  __syncthreads();
  float2 Ds = s_D[lane];  // adjoint entering the last sub-tile from its right
  float2 acc_c1 = cz(), acc_1 = cz(), acc_2 = cz(), acc_w = cz();
#pragma unroll 1
  for (int s = S - 1; s >= 0; --s) {
    float2 Xw = cz(), Xrw = cz();
    for (int w = 0; w < warp; ++w)
      Xw = c_fma(c.gK, Xw, make_float2(s_yh[s][w][lane].x, s_yh[s][w][lane].y));
    for (int w = kBtfWarps - 1; w > warp; --w)
      Xrw = c_fma(muK, Xrw, make_float2(s_yh[s][w][lane].z, s_yh[s][w][lane].w));
    float2 e = c_fma(c.Gw, hdr[(kHCarry + s) * 32 + lane], Xw);
    float2 gnext = c_fma(c.Grw, Ds, Xrw);
    float2 v[kBtfK + 1];
    btf_rows9(xs, kBtfSub * s + rw, col, v);
    float2 yprev[kBtfK];
#pragma unroll
    for (int k = 0; k < kBtfK; ++k) {
      yprev[k] = e;
      e = c_fma(c.lam, e, btf_drive1<DRIVE>(c, v[k + 1], v[k]));
      if constexpr (MOSC) acc_w = c_cfma(e, gs[(kBtfSub * s + rw + k) * 32 + col], acc_w);
    }
    const int64_t t0 = ts0 + kBtfSub * s + rw;
    const int64_t left = a.T - t0;
    const int kmax = !fv ? 0 : (left < kBtfK ? (int)left : kBtfK);
    const int64_t obase = (tl.b * a.T + t0) * a.F + f;
#pragma unroll
    for (int k = kBtfK - 1; k >= 0; --k) {
      const float2 g = c_fma(mu, gnext, gcot(kBtfSub * s + rw + k));
      if constexpr (MOSC) {  // grad_u[f]: the filter's oscillators summed
        const float2 gu = btf_group_sum(c_cfma(c.c2, g, cz()), a.log2n);
        const bool lead = (lane & ((1 << a.log2n) - 1)) == 0 && k < kmax;
        const int64_t ui = (tl.b * a.T + t0 + k) * a.Fin + (f >> a.log2n);
        if (DRIVE == kReal) {
          if (lead) __stcs(static_cast<float *>(a.out) + ui, gu.x);
          acc_1 = make_float2(fmaf(v[k + 1].x, g.x, acc_1.x), fmaf(v[k + 1].x, g.y, acc_1.y));
        } else {
          if (lead) __stcs(static_cast<float2 *>(a.out) + ui, gu);
          acc_1 = c_cfma(v[k + 1], g, acc_1);
        }
      } else if constexpr (DRIVE == kReal) {
        // grad of the real input: Re(conj(c2) g)
        if (k < kmax)
          __stcs(static_cast<float *>(a.out) + obase + k * a.F, c.c2.x * g.x + c.c2.y * g.y);
        acc_1 = make_float2(fmaf(v[k + 1].x, g.x, acc_1.x), fmaf(v[k + 1].x, g.y, acc_1.y));
      } else if constexpr (DRIVE == kPlain) {
        if (k < kmax) __stcs(static_cast<float2 *>(a.out) + obase + k * a.F, c_cfma(c.c2, g, cz()));
        acc_1 = c_cfma(v[k + 1], g, acc_1);
      } else {
        if (k < kmax)
          __stcs(static_cast<float2 *>(a.out) + obase + k * a.F,
                 c_cfma(c.t1, gnext, c_cfma(c.c2, g, cz())));
        acc_1 = c_cfma(v[k + 1], g, acc_1);
        acc_2 = c_cfma(v[k], g, acc_2);
      }
      acc_c1 = c_cfma(yprev[k], g, acc_c1);
      gnext = g;
    }
    if (s > 0) Ds = c_fma(muL, Ds, s_H[s][lane]);  // adjoint entering sub-tile s-1 from its right
  }
  // per-tile partial sums, fixed order over the warps
  s_red[0][warp][lane] = acc_c1;
  s_red[1][warp][lane] = acc_1;
  s_red[2][warp][lane] = acc_2;
  if constexpr (MOSC) s_red[3][warp][lane] = acc_w;
  __syncthreads();
  if (warp < (MOSC ? 4 : 3) && fv) {
    float2 sum = cz();
#pragma unroll
    for (int w = 0; w < kBtfWarps; ++w) sum = c_add(sum, s_red[warp][w][lane]);
    const int64_t slot = ((tl.b * a.F + f) * a.ntiles + tl.j) * 3;
    if (warp < 3)
      a.partials[slot + warp] = sum;
    else
      a.partials2[slot] = sum;
  }
}

// TBPTT(1) surrogate backward in (B,T,F) layout: no temporal adjoint, so the
// sub-tiles are independent, each starting from its saved entry state.  A CTA
// takes kBtfTbpttS consecutive sub-tiles of a chain through a two-stage ring;
// grad_zw[t] = conj(tap1) g[t+1] reads the cotangent row after each thread's
// steps from the stage (the row after the sub-tile is copied with it).
template <bool VECX>
__global__ void __launch_bounds__(kBtfThreads, 2) btf_tbptt_bwd_kernel(const BtfArgs a) {
  extern __shared__ __align__(16) unsigned char btf_dsm[];
  __shared__ float2 s_y[2][kBtfWarps][32];
  __shared__ float2 s_red[3][kBtfWarps][32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const BtfTile tl = btf_decode(a, blockIdx.x, false);  // independent tiles: no ticket
  constexpr int S = kBtfTbpttS;
  constexpr size_t kHdr = (size_t)(kHCarry + 1) * 32 * sizeof(float2);
  constexpr size_t kRows = (size_t)(kBtfSub + 1) * 32 * sizeof(float2);
  auto issue = [&](int s) {
    if (s < S) {
      unsigned char *st = btf_dsm + (s & 1) * kBtfTbpttStage;
      float2 *hdr = reinterpret_cast<float2 *>(st);
      const int sub = tl.j * S + s;
      if (s == 0) {
        btf_copy_header<kTwoTap, 1>(hdr, a, tl, kBtfLog2Sub, sub);
      } else if (warp == 0) {  // the entry state of this sub-tile
        const int64_t ff = tl.f0 + lane;
        const bool ok = ff < a.F && sub < a.nsub;
        cp_async8(hdr + kHCarry * 32 + lane,
                  ok ? a.carries + (tl.b * a.F + ff) * a.nsub + sub : a.carries, ok);
      }
      const int64_t t0 = (int64_t)sub * kBtfSub;
      btf_copy_rows<float2, VECX>(reinterpret_cast<float2 *>(st + kHdr),
                                  static_cast<const float2 *>(a.x), a, tl, t0 - 1, 0, kBtfSub + 1);
      btf_copy_rows<float2, VECX>(reinterpret_cast<float2 *>(st + kHdr + kRows), a.gout, a, tl, t0,
                                  0, kBtfSub + 1);
    }
    cp_async_commit();
  };
  issue(0);

  BtfConst c{};
  float2 acc_c1 = cz(), acc_t0 = cz(), acc_t1 = cz();
  const int64_t f = tl.f0 + lane;
  const bool fv = f < a.F;
  const int rw = warp * kBtfK;
#pragma unroll 1
  for (int s = 0; s < S; ++s) {
    cp_async_wait<0>();
    __syncthreads();
    issue(s + 1);
    const unsigned char *st = btf_dsm + (s & 1) * kBtfTbpttStage;
    const float2 *hdr = reinterpret_cast<const float2 *>(st);
    const float2 *xs = reinterpret_cast<const float2 *>(st + kHdr);
    const float2 *gs = reinterpret_cast<const float2 *>(st + kHdr + kRows);
    if (s == 0) c = btf_consts(hdr, lane, warp);
    const float2 C = hdr[kHCarry * 32 + lane];
    float2 v[kBtfK + 1];
    btf_rows9(xs, rw, lane, v);
    float2 b[kBtfK];
#pragma unroll
    for (int k = 0; k < kBtfK; ++k) b[k] = btf_drive1<kTwoTap>(c, v[k + 1], v[k]);
    float2 y = cz();
#pragma unroll
    for (int k = 0; k < kBtfK; ++k) y = c_fma(c.lam, y, b[k]);
    s_y[s & 1][warp][lane] = y;
    __syncthreads();
    float2 Xw = cz();
    for (int w = 0; w < warp; ++w) Xw = c_fma(c.gK, Xw, s_y[s & 1][w][lane]);
    float2 e = c_fma(c.Gw, C, Xw);
    const int64_t t0 = (int64_t)(tl.j * S + s) * kBtfSub + rw;
    const int64_t left = a.T - t0;
    const int kmax = !fv ? 0 : (left < kBtfK ? (int)left : kBtfK);
    const int64_t obase = (tl.b * a.T + t0) * a.F + f;
#pragma unroll
    for (int k = 0; k < kBtfK; ++k) {
      const float2 yp = e;
      e = c_fma(c.lam, e, b[k]);
      const float2 g = gs[(rw + k) * 32 + lane];
      const float2 g1 = gs[(rw + k + 1) * 32 + lane];  // zero after the sequence
      if (k < kmax) {
        __stcs(static_cast<float2 *>(a.out) + obase + k * a.F, c_cfma(c.c2, g, cz()));
        __stcs(a.out2 + obase + k * a.F, c_cfma(c.t1, g1, cz()));
      }
      acc_c1 = c_cfma(yp, g, acc_c1);
      acc_t0 = c_cfma(v[k + 1], g, acc_t0);
      acc_t1 = c_cfma(v[k], g, acc_t1);
    }
  }
  s_red[0][warp][lane] = acc_c1;
  s_red[1][warp][lane] = acc_t0;
  s_red[2][warp][lane] = acc_t1;
  __syncthreads();
  if (warp < 3 && fv) {
    float2 sum = cz();
#pragma unroll
    for (int w = 0; w < kBtfWarps; ++w) sum = c_add(sum, s_red[warp][w][lane]);
    a.partials[((tl.b * a.F + f) * a.ntiles + tl.j) * 3 + warp] = sum;
  }
}

// c1^(2^i) for i < kBtfPowLevels in double precision, one thread per channel:
// pw[i*F + f].
__global__ void btf_pow_table_kernel(const float2 *__restrict__ c1, float2 *__restrict__ pw,
                                     int64_t F) {
  const int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= F) return;
  double re = c1[f].x, im = c1[f].y;
  for (int i = 0; i < kBtfPowLevels; ++i) {
    pw[i * F + f] = make_float2((float)re, (float)im);
    const double nr = re * re - im * im;
    const double ni = 2.0 * re * im;
    re = nr;
    im = ni;
  }
}

}  // namespace rqf
