// Two-tap prospective scan in (filters, batch, time) layout — time innermost.
//
// Recurrence (rqf_models/ops/fbt_scan_kernel.py:_fbt_prospective_kernel :34-110):
//   y[t] = c1*y[t-1] + tap0*z[t] + tap1*z[t-1],   y[-1] = z[-1] = 0,
// one independent row per (channel f, batch b): row = f*batch + b.
//
// Work decomposition (B200-first, not the reference's one-program-per-row
// serial chunk loop):
//   * one CTA = one tile of NT*K consecutive samples of one row; each thread
//     owns K consecutive samples in registers (coalesced 16-byte loads through
//     a warp-private swizzled transpose);
//   * in-tile carries: per-thread serial recurrence, warp-shuffle
//     Kogge-Stone scan of affine pairs, cross-warp composition in shared
//     memory;
//   * cross-tile carries: decoupled look-back over the row's earlier tiles,
//     CTAs ordered by an atomic ticket so every awaited tile belongs to a CTA
//     that is already running (bounded waits, error latch);
//   * the forward stores one carry (entry state) per tile; the backward
//     recomputes y from it, so no (F,B,T) state is saved or re-read, and fuses
//     the split-ReLU mask, the reverse adjoint scan, grad_z and the
//     grad_c1/grad_tap0/grad_tap1 reductions (deterministic per-tile partials).
#pragma once

#include "rqf_common.cuh"

namespace rqf {

struct FbtArgs {
  const float2 *c1, *tap0, *tap1;  // (F,)
  const float2 *z;                 // (rows, T)
  const float2 *gout;              // (rows, T) cotangent (backward)
  const float2 *skip;              // (rows, T) added to the forward output, or null
  float2 *out;                     // forward: act / raw; backward: grad_z
  float2 *out2;                    // TBPTT backward: grad_zw, or grad_z + grad_zw with wsum
  int wsum;                        // TBPTT backward: out2 = grad_z + grad_zw (the weight's operand)
  float2 *carries;                 // entry states, see kFbtSlots
  float2 *partials;                // (rows, ntiles, 3)
  u64 *flags;                      // (rows, ntiles, 2)
  unsigned *ticket;
  int64_t rows, T;
  int batch;   // rows per channel
  int ntiles;  // tiles per row
  int log2L;   // log2(tile length)
};

constexpr int kFbtThreads = 256;
constexpr int kFbtK = 8;
constexpr int kFbtTile = kFbtThreads * kFbtK;  // 2048 samples
constexpr int kFbtLog2Tile = 11;
// Saved context of the forward: one entry state per thread of every tile,
// (rows, ntiles, kFbtSlots) complex, slot 0 being the tile's own entry, and
// one marker element after them.  Every (F,B,T) forward — the persistent row
// kernels, the look-back tile kernels and the projection's scan epilogue —
// writes every slot and the marker (1, 0), and computes each output from its
// thread's entry with the drive of fbt_drive and y = c1 y + b.  Every
// backward starts each thread from that entry with the same operations, so
// it replays the forward's states bit for bit (the split-ReLU decisions of a
// state within rounding of zero included) whichever kernel family ran the
// forward.  A backward that finds the marker unset scans from the tile entry.
constexpr int kFbtSlots = kFbtThreads;
__host__ __device__ __forceinline__ int64_t fbt_slot(int64_t row, int ntiles, int j) {
  return (row * ntiles + j) * kFbtSlots;
}
__host__ __device__ __forceinline__ int64_t fbt_marker(int64_t rows, int ntiles) {
  return rows * ntiles * kFbtSlots;
}
constexpr int kPowTable = 12;  // lambda^(2^i), i <= log2(tile)

// Two-tap drive of K consecutive samples, b[k] = tap0 z[k] + tap1 z[k-1]
// (zp = the sample before z[0]), on paired FMAs.
template <int K>
__device__ __forceinline__ void fbt_drive(float2 t0, float2 t1, const float2 (&z)[K], float2 zp,
                                          float2 (&b)[K]) {
  const CPair T0 = cpair(t0), T1 = cpair(t1);
  float2 sp = c_swap(zp);
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float2 sk = c_swap(z[k]);
    b[k] = cp_fma(T0, z[k], sk, cp_mul(T1, k > 0 ? z[k - 1] : zp, sp));
    sp = sk;
  }
}

// Load the K samples [tfirst, tfirst+K) of this thread (blocked order).
template <int K, bool VEC>
__device__ __forceinline__ void fbt_load(const float2 *__restrict__ row, int64_t wstart,
                                         int64_t tfirst, int64_t T, float2 (&x)[K], float4 *wbuf,
                                         int lane) {
  if constexpr (VEC) {
    float4 s[K / 2];
#pragma unroll
    for (int v = 0; v < K / 2; ++v) {
      const int64_t t = wstart + 2 * (v * 32 + lane);
      s[v] = (t < T) ? ld_stream4(row + t) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    striped_to_blocked<K>(wbuf, s, x, lane);
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t t = tfirst + k;
      x[k] = (t < T) ? __ldcs(row + t) : cz();
    }
  }
}

template <int K, bool VEC>
__device__ __forceinline__ void fbt_store(float2 *__restrict__ row, int64_t wstart, int64_t tfirst,
                                          int64_t T, const float2 (&x)[K], float4 *wbuf,
                                          int lane) {
  if constexpr (VEC) {
    float4 s[K / 2];
    blocked_to_striped<K>(wbuf, x, s, lane);
#pragma unroll
    for (int v = 0; v < K / 2; ++v) {
      const int64_t t = wstart + 2 * (v * 32 + lane);
      if (t < T) st_stream4(row + t, s[v]);
    }
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t t = tfirst + k;
      if (t < T) __stcs(row + t, x[k]);
    }
  }
}

// ------------------------------------------------------------ forward
template <int NT, int K, bool VEC, bool FUSE_ACT>
__global__ void __launch_bounds__(NT) fbt_fwd_kernel(const FbtArgs a) {
  constexpr int NW = NT / 32, L = NT * K;
  constexpr int LK = (K == 4) ? 2 : (K == 8) ? 3 : 4;
  __shared__ __align__(16) float4 s_buf[NW][16 * K];
  __shared__ float2 s_warp[NW];
  __shared__ float2 s_pw[kPowTable];
  __shared__ unsigned s_ticket;
  __shared__ float2 s_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    const unsigned t = atomicAdd(a.ticket, 1u);
    s_ticket = t;
    pow2_table(a.c1[(t / (unsigned)a.ntiles) / a.batch], s_pw, kPowTable);
  }
  __syncthreads();
  const unsigned tk = s_ticket;
  const int64_t row = tk / (unsigned)a.ntiles;
  const int j = (int)(tk - (unsigned)(row * a.ntiles));
  const int f = (int)(row / a.batch);
  const float2 lam = a.c1[f], t0 = a.tap0[f], t1 = a.tap1[f];
  const float2 *zrow = a.z + row * a.T;
  const int64_t wstart = (int64_t)j * L + (int64_t)warp * 32 * K;
  const int64_t tfirst = wstart + lane * K;

  float2 z[K];
  fbt_load<K, VEC>(zrow, wstart, tfirst, a.T, z, s_buf[warp], lane);
  float2 zp = shfl_up2(z[K - 1], 1);
  if (lane == 0) zp = (tfirst > 0 && tfirst - 1 < a.T) ? zrow[tfirst - 1] : cz();

  float2 b[K];
  fbt_drive<K>(t0, t1, z, zp, b);
  float2 y = cz();
#pragma unroll
  for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);

  float2 G, X, At;
  cta_scan_const_fwd<NT, LK>(y, s_pw, G, X, At, s_warp);

  if (tid == 0) {
    u64 *fl = a.flags + row * (int64_t)a.ntiles * 2;
    const bool has_next = j + 1 < a.ntiles;
    float2 C = cz();
    if (j == 0) {
      if (has_next) flag_publish2(fl, At, kInclusive);
    } else {
      if (has_next) flag_publish2(fl + 2 * j, At, kAggregate);
      const float2 M = s_pw[a.log2L];
      C = lookback_const(fl, j, M);
      if (has_next) flag_publish2(fl + 2 * j, c_fma(M, C, At), kInclusive);
    }
    if (tk == 0) a.carries[fbt_marker(a.rows, a.ntiles)] = make_float2(1.f, 0.f);
    s_carry = C;
  }
  __syncthreads();
  // every thread's entry state (slot 0: the tile's own entry)
  float2 e = tid == 0 ? s_carry : c_fma(G, s_carry, X);
  a.carries[fbt_slot(row, a.ntiles, j) + tid] = e;
  float2 o[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    e = c_fma(lam, e, b[k]);
    o[k] = FUSE_ACT ? c_relu(e) : e;
  }
  if (a.skip) {
    float2 sk[K];
    fbt_load<K, VEC>(a.skip + row * a.T, wstart, tfirst, a.T, sk, s_buf[warp], lane);
#pragma unroll
    for (int k = 0; k < K; ++k) o[k] = c_add(o[k], sk[k]);
  }
  fbt_store<K, VEC>(a.out + row * a.T, wstart, tfirst, a.T, o, s_buf[warp], lane);
}

// ------------------------------------------------ full-BPTT backward
template <int NT, int K, bool VEC, bool FUSE_ACT>
__global__ void __launch_bounds__(NT) fbt_bwd_kernel(const FbtArgs a) {
  constexpr int NW = NT / 32;
  constexpr int L = NT * K;
  constexpr int LK = (K == 4) ? 2 : (K == 8) ? 3 : 4;
  __shared__ __align__(16) float4 s_buf[NW][16 * K];
  __shared__ float2 s_warp_f[NW];
  __shared__ float2 s_warp_r[NW];
  __shared__ float2 s_pw[kPowTable];
  __shared__ float2 s_red[3][NW];
  __shared__ unsigned s_ticket;
  __shared__ float2 s_entry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    const unsigned t = atomicAdd(a.ticket, 1u);
    s_ticket = t;
    pow2_table(a.c1[(t / (unsigned)a.ntiles) / a.batch], s_pw, kPowTable);
  }
  __syncthreads();
  const unsigned tk = s_ticket;
  const int64_t row = tk / (unsigned)a.ntiles;
  const int p = (int)(tk - (unsigned)(row * a.ntiles));  // processing position
  const int j = a.ntiles - 1 - p;                         // tile index in time
  const int f = (int)(row / a.batch);
  const float2 lam = a.c1[f], t0 = a.tap0[f], t1 = a.tap1[f];
  const float2 C = a.carries[fbt_slot(row, a.ntiles, j)];
  const bool per_thread = __ldg(a.carries + fbt_marker(a.rows, a.ntiles)).x == 1.f;
  const float2 *zrow = a.z + row * a.T;
  const float2 *grow = a.gout + row * a.T;
  const int64_t wstart = (int64_t)j * L + (int64_t)warp * 32 * K;
  const int64_t tfirst = wstart + lane * K;

  float2 z[K], go[K];
  fbt_load<K, VEC>(zrow, wstart, tfirst, a.T, z, s_buf[warp], lane);
  fbt_load<K, VEC>(grow, wstart, tfirst, a.T, go, s_buf[warp], lane);
  float2 zp = shfl_up2(z[K - 1], 1);
  if (lane == 0) zp = (tfirst > 0 && tfirst - 1 < a.T) ? zrow[tfirst - 1] : cz();

  // Replay the forward states of this tile from the saved entries (or, with
  // the marker unset, from a scan of the tile entry carry).
  float2 b[K];
  fbt_drive<K>(t0, t1, z, zp, b);
  float2 e;
  if (per_thread) {
    e = a.carries[fbt_slot(row, a.ntiles, j) + tid];
  } else {
    float2 y = cz();
#pragma unroll
    for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
    float2 G, X, At;
    cta_scan_const_fwd<NT, LK>(y, s_pw, G, X, At, s_warp_f);
    e = c_fma(G, C, X);
  }
  float2 yprev[K];  // y[t-1] per sample; reuse b[] storage for the masked cotangent
#pragma unroll
  for (int k = 0; k < K; ++k) {
    yprev[k] = e;
    e = c_fma(lam, e, b[k]);
    b[k] = FUSE_ACT ? c_relu_mask(go[k], e) : go[k];
  }

  // Reverse adjoint: g[t] = gbar[t] + conj(c1) g[t+1], g[T] = 0.
  const float2 mu = c_conj(lam);
  float2 h = cz();
#pragma unroll
  for (int k = K - 1; k >= 0; --k) h = c_fma(mu, h, b[k]);
  float2 Gr, Xr, Art;
  cta_scan_const_rev<NT, LK>(h, s_pw, Gr, Xr, Art, s_warp_r);
  if (tid == 0) {
    u64 *fl = a.flags + row * (int64_t)a.ntiles * 2;
    const bool has_next = p + 1 < a.ntiles;
    float2 D = cz();
    if (p == 0) {
      if (has_next) flag_publish2(fl, Art, kInclusive);
    } else {
      if (has_next) flag_publish2(fl + 2 * p, Art, kAggregate);
      const float2 M = c_conj(s_pw[a.log2L]);
      D = lookback_const(fl, p, M);
      if (has_next) flag_publish2(fl + 2 * p, c_fma(M, D, Art), kInclusive);
    }
    s_entry = D;
  }
  __syncthreads();
  float2 gnext = c_fma(Gr, s_entry, Xr);
  float2 acc_c1 = cz(), acc_t0 = cz(), acc_t1 = cz();
  float2 gz[K];
#pragma unroll
  for (int k = K - 1; k >= 0; --k) {
    const float2 g = c_fma(mu, gnext, b[k]);
    gz[k] = c_cfma(t1, gnext, c_cfma(t0, g, cz()));
    acc_c1 = c_cfma(yprev[k], g, acc_c1);
    acc_t0 = c_cfma(z[k], g, acc_t0);
    acc_t1 = c_cfma(k > 0 ? z[k - 1] : zp, g, acc_t1);
    gnext = g;
  }
  fbt_store<K, VEC>(a.out + row * a.T, wstart, tfirst, a.T, gz, s_buf[warp], lane);

  // Deterministic per-tile partial sums of the coefficient gradients.
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc_c1 = c_add(acc_c1, shfl_xor2(acc_c1, o));
    acc_t0 = c_add(acc_t0, shfl_xor2(acc_t0, o));
    acc_t1 = c_add(acc_t1, shfl_xor2(acc_t1, o));
  }
  if (lane == 0) {
    s_red[0][warp] = acc_c1;
    s_red[1][warp] = acc_t0;
    s_red[2][warp] = acc_t1;
  }
  __syncthreads();
  if (tid < 3) {
    float2 s = cz();
#pragma unroll
    for (int w = 0; w < NW; ++w) s = c_add(s, s_red[tid][w]);
    a.partials[(row * a.ntiles + j) * 3 + tid] = s;
  }
}

// -------------------------------------------------- TBPTT(1) backward
// No temporal adjoint: g = gout (masked by split-ReLU'(y) when FUSE_ACT);
// grad_z = conj(tap0) g[t]; grad_zw[t] = conj(tap1) g[t+1];
// partials of conj(y[t-1]) g, conj(z[t]) g, conj(z[t-1]) g.
// One CTA per (row, tile) in blockIdx order; y recomputed from the carries.
template <int NT, int K, bool VEC, bool FUSE_ACT>
__global__ void __launch_bounds__(NT) fbt_tbptt_bwd_kernel(const FbtArgs a) {
  constexpr int NW = NT / 32;
  constexpr int L = NT * K;
  constexpr int LK = (K == 4) ? 2 : (K == 8) ? 3 : 4;
  __shared__ __align__(16) float4 s_buf[NW][16 * K];
  __shared__ float2 s_warp_f[NW];
  __shared__ float2 s_pw[kPowTable];
  __shared__ float2 s_first[NW + 1];
  __shared__ float2 s_red[3][NW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) pow2_table(a.c1[(blockIdx.x / (unsigned)a.ntiles) / a.batch], s_pw, kPowTable);
  const int64_t row = blockIdx.x / (unsigned)a.ntiles;
  const int j = (int)(blockIdx.x - (unsigned)(row * a.ntiles));
  const int f = (int)(row / a.batch);
  const float2 lam = a.c1[f], t0 = a.tap0[f], t1 = a.tap1[f];
  const float2 C = a.carries[fbt_slot(row, a.ntiles, j)];
  const bool per_thread = __ldg(a.carries + fbt_marker(a.rows, a.ntiles)).x == 1.f;
  const float2 *zrow = a.z + row * a.T;
  const float2 *grow = a.gout + row * a.T;
  const int64_t wstart = (int64_t)j * L + (int64_t)warp * 32 * K;
  const int64_t tfirst = wstart + lane * K;

  float2 z[K], go[K];
  fbt_load<K, VEC>(zrow, wstart, tfirst, a.T, z, s_buf[warp], lane);
  fbt_load<K, VEC>(grow, wstart, tfirst, a.T, go, s_buf[warp], lane);
  float2 zp = shfl_up2(z[K - 1], 1);
  if (lane == 0) zp = (tfirst > 0 && tfirst - 1 < a.T) ? zrow[tfirst - 1] : cz();

  float2 b[K];
  fbt_drive<K>(t0, t1, z, zp, b);
  __syncthreads();  // s_pw
  float2 e;
  if (per_thread) {
    e = a.carries[fbt_slot(row, a.ntiles, j) + tid];
  } else {
    float2 y = cz();
#pragma unroll
    for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
    float2 G, X, At;
    cta_scan_const_fwd<NT, LK>(y, s_pw, G, X, At, s_warp_f);
    e = c_fma(G, C, X);
  }
  float2 yprev[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    yprev[k] = e;
    e = c_fma(lam, e, b[k]);
    go[k] = FUSE_ACT ? c_relu_mask(go[k], e) : go[k];
  }
  // g at the sample after this thread's last one.
  float2 gn = shfl_down2(go[0], 1);
  if (lane == 0) s_first[warp] = go[0];
  if (tid == NT - 1) {
    const int64_t tn = (int64_t)(j + 1) * L;  // first sample of the next tile
    float2 g_next = cz();
    if (tn < a.T) {
      g_next = grow[tn];
      if (FUSE_ACT) {
        // the next tile's first state, as that tile's thread 0 replays it
        const float2 zn = zrow[tn];
        const CPair T0 = cpair(t0), T1 = cpair(t1);
        const float2 bn = cp_fma(T0, zn, c_swap(zn), cp_mul(T1, z[K - 1], c_swap(z[K - 1])));
        const float2 en = per_thread ? a.carries[fbt_slot(row, a.ntiles, j + 1)] : e;
        g_next = c_relu_mask(g_next, c_fma(lam, en, bn));
      }
    }
    s_first[NW] = g_next;
  }
  __syncthreads();
  if (lane == 31) gn = s_first[warp + 1];

  float2 acc_c1 = cz(), acc_t0 = cz(), acc_t1 = cz();
  float2 dz[K], dzw[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float2 g = go[k];
    const float2 g1 = (k + 1 < K) ? go[k + 1] : gn;
    dz[k] = c_cfma(t0, g, cz());
    dzw[k] = c_cfma(t1, g1, a.wsum ? dz[k] : cz());
    acc_c1 = c_cfma(yprev[k], g, acc_c1);
    acc_t0 = c_cfma(z[k], g, acc_t0);
    acc_t1 = c_cfma(k > 0 ? z[k - 1] : zp, g, acc_t1);
  }
  fbt_store<K, VEC>(a.out + row * a.T, wstart, tfirst, a.T, dz, s_buf[warp], lane);
  fbt_store<K, VEC>(a.out2 + row * a.T, wstart, tfirst, a.T, dzw, s_buf[warp], lane);

#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc_c1 = c_add(acc_c1, shfl_xor2(acc_c1, o));
    acc_t0 = c_add(acc_t0, shfl_xor2(acc_t0, o));
    acc_t1 = c_add(acc_t1, shfl_xor2(acc_t1, o));
  }
  if (lane == 0) {
    s_red[0][warp] = acc_c1;
    s_red[1][warp] = acc_t0;
    s_red[2][warp] = acc_t1;
  }
  __syncthreads();
  if (tid < 3) {
    float2 s = cz();
#pragma unroll
    for (int w = 0; w < NW; ++w) s = c_add(s, s_red[tid][w]);
    a.partials[(row * a.ntiles + j) * 3 + tid] = s;
  }
}

}  // namespace rqf
