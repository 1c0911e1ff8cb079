// Persistent row-sequential variant of the (F,B,T) two-tap scan, used when
// there are at least as many rows as resident CTAs (the benchmarked waveform
// and selective layers have 2k-8k rows of 4k-16k samples).
//
// Each CTA owns rows blockIdx.x, blockIdx.x + gridDim.x, ... and walks each
// row tile by tile, keeping the recurrence carry on chip between tiles, so no
// inter-CTA communication (tickets, flags, look-back) is needed.  Because the
// state entering a tile is known before the tile is scanned, it is folded into
// the first thread's aggregate (cta_scan_entry_*), which removes the per-thread
// gate powers of the look-back kernels.  The memory system is kept busy by an
// S-stage cp.async pipeline: while tile i is computed, the inputs of the next
// S-1 tiles (possibly of the next rows) are in flight into swizzled shared
// memory.  Work cursors are advanced incrementally (no integer division in the
// loop).
//
// Same tile length and saved-context layout as fbt_scan.cuh (kFbtSlots), so
// the forward and backward of either variant pair up.  The forward saves every
// thread's entry state, so the backward replays each thread's states from its
// own entry without a forward scan of the tile.
#pragma once

#include "fbt_scan.cuh"

namespace rqf {

constexpr int kRowsFwdStages = 3;
constexpr int kRowsBwdStages = 2;  // 2 x 32 KB stages: 3 CTAs per SM

template <int NT, int K, int NIN, int S>
constexpr size_t fbt_rows_smem_bytes() {
  return (size_t)S * NIN * NT * (K / 2) * sizeof(float4);
}

// Work cursor over (row, tile) items of this CTA.
struct RowCursor {
  int row, j, stage;
  __device__ __forceinline__ void advance(int ntiles, int G, int S) {
    if (++j == ntiles) {
      j = 0;
      row += G;
    }
    stage = (stage + 1 == S) ? 0 : stage + 1;
  }
};

// Power table for the row being issued into stage `s`: copied from the
// previous stage for later tiles of the same row, built in double precision
// for a row's first tile.  Called by one thread, in issue order.
template <int S>
__device__ __forceinline__ void stage_table(float2 (*s_pw)[kPowTable], int s, bool first_tile,
                                            const float2 *c1, int f) {
  if (!first_tile) {
    const int sp = (s + S - 1) % S;
#pragma unroll
    for (int i = 0; i < kPowTable; ++i) s_pw[s][i] = s_pw[sp][i];
  } else {
    pow2_table(c1[f], s_pw[s], kPowTable);
  }
}

// The striped slot v*32 + lane of a warp region swizzles to v*32 + swz(lane)
// when K <= 8 (the swizzle only mixes bits 3-4 of the slot into bits 0-1), so
// each lane addresses its slots and samples from one base plus constants.
// A warp region lying wholly inside the row (every tile but a row's last)
// takes the copies without per-copy bounds tests.
template <int K>
__device__ __forceinline__ void fbt_issue_tile(float4 *wbuf, const float2 *row, int wstart, int T,
                                               int lane) {
  static_assert(K <= 8, "slot swizzle decomposition needs K <= 8");
  float4 *dst = wbuf + swz<K>(lane);
  const float2 *src = row + wstart + 2 * lane;
  if (wstart + 32 * K <= T) {
#pragma unroll
    for (int v = 0; v < K / 2; ++v) cp_async16_full(dst + 32 * v, src + 64 * v);
  } else {
#pragma unroll
    for (int v = 0; v < K / 2; ++v) {
      const bool in = wstart + 2 * lane + 64 * v < T;
      cp_async16(dst + 32 * v, in ? src + 64 * v : row, in);
    }
  }
}

template <int K>
__device__ __forceinline__ void fbt_store_tile(float4 *wbuf, const float2 (&o)[K], float2 *row,
                                               int wstart, int T, int lane) {
  static_assert(K <= 8, "slot swizzle decomposition needs K <= 8");
#pragma unroll
  for (int m = 0; m < K / 2; ++m)
    wbuf[swz<K>(lane * (K / 2) + m)] =
        make_float4(o[2 * m].x, o[2 * m].y, o[2 * m + 1].x, o[2 * m + 1].y);
  __syncwarp();
  const float4 *sp = wbuf + swz<K>(lane);
  float2 *dp = row + wstart + 2 * lane;
  if (wstart + 32 * K <= T) {
#pragma unroll
    for (int v = 0; v < K / 2; ++v) st_stream4(dp + 64 * v, sp[32 * v]);
  } else {
#pragma unroll
    for (int v = 0; v < K / 2; ++v)
      if (wstart + 2 * lane + 64 * v < T) st_stream4(dp + 64 * v, sp[32 * v]);
  }
}

// ------------------------------------------------------------ forward
// SKIP: the stage also carries the same tile of `skip`, added to the output
// (the Pure RQF complex skip connection h = out + h, fused).
template <int NT, int K, int S, bool FUSE_ACT, bool SKIP = false>
__global__ void __launch_bounds__(NT) fbt_fwd_rows_kernel(const FbtArgs a) {
  constexpr int NW = NT / 32, L = NT * K, LK = (K == 4) ? 2 : (K == 8) ? 3 : 4;
  constexpr int WSZ = 16 * K;  // float4 slots per warp region
  constexpr int NIN = SKIP ? 2 : 1;
  extern __shared__ __align__(16) float4 dsm[];  // [S][NIN inputs][NW][WSZ]
  __shared__ float2 s_pw[S][kPowTable];
  __shared__ float2 s_warp[NW];
  __shared__ float2 s_zlast;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, rows = (int)a.rows, T = (int)a.T, ntiles = a.ntiles;
  const int wofs = warp * 32 * K;

  static_assert(NT == kFbtSlots, "one saved entry state per thread");
  if (blockIdx.x == 0 && tid == 0)
    a.carries[fbt_marker(a.rows, ntiles)] = make_float2(1.f, 0.f);  // every slot written
  RowCursor ic{(int)blockIdx.x, 0, 0};  // next item to issue
  auto issue = [&]() {
    if (ic.row < rows) {
      fbt_issue_tile<K>(dsm + (size_t)ic.stage * NIN * NW * WSZ + warp * WSZ,
                        a.z + (size_t)ic.row * T, ic.j * L + wofs, T, lane);
      if constexpr (SKIP)
        fbt_issue_tile<K>(dsm + ((size_t)ic.stage * NIN + 1) * NW * WSZ + warp * WSZ,
                          a.skip + (size_t)ic.row * T, ic.j * L + wofs, T, lane);
      if (tid == 0) stage_table<S>(s_pw, ic.stage, ic.j == 0, a.c1, ic.row / a.batch);
      ic.advance(ntiles, G, S);
    }
    cp_async_commit();
  };

#pragma unroll
  for (int s = 0; s < S - 1; ++s) issue();
  RowCursor pc{(int)blockIdx.x, 0, 0};  // item being processed
  float2 carry = cz(), lam = cz(), t0 = cz(), t1 = cz(), lanepow = cz();
  while (pc.row < rows) {
    cp_async_wait<S - 2>();
    __syncthreads();
    issue();
    const float2 *pw = s_pw[pc.stage];
    if (pc.j == 0) {  // new row: per-row constants
      const int f = pc.row / a.batch;
      lam = pw[0];
      t0 = a.tap0[f];
      t1 = a.tap1[f];
      lanepow = pow_from_table<false>(pw, LK, lane);
      carry = cz();
    }
    float4 *wbuf = dsm + (size_t)pc.stage * NIN * NW * WSZ + warp * WSZ;
    float2 z[K];
    read_blocked<K>(wbuf, z, lane);
    float2 zp = shfl_up2(z[K - 1], 1);
    if (lane == 0) {
      if (warp > 0)
        zp = read_sample<K>(wbuf - WSZ, 32 * K - 1);
      else
        zp = (pc.j > 0) ? s_zlast : cz();
    }
    float2 b[K];
    fbt_drive<K>(t0, t1, z, zp, b);
    float2 y = cz();
#pragma unroll
    for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
    float2 e, At;
    cta_scan_entry_fwd<NT, LK>(y, carry, pw, lanepow, e, At, s_warp);
    if (tid == NT - 1) s_zlast = z[K - 1];
    // every thread's entry state (slot 0: the tile's own entry, e == carry)
    a.carries[fbt_slot(pc.row, ntiles, pc.j) + tid] = e;
    carry = At;  // entry of the next tile of this row
    float2 o[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      e = c_fma(lam, e, b[k]);
      o[k] = FUSE_ACT ? c_relu(e) : e;
    }
    if constexpr (SKIP) {
      float2 sk[K];
      read_blocked<K>(wbuf + NW * WSZ, sk, lane);
#pragma unroll
      for (int k = 0; k < K; ++k) o[k] = c_add(o[k], sk[k]);
    }
    fbt_store_tile<K>(wbuf, o, a.out + (size_t)pc.row * T, pc.j * L + wofs, T, lane);
    pc.advance(ntiles, G, S);
  }
  cp_async_wait<0>();
}

// ------------------------------------------------ full-BPTT backward
// Tiles of a row in reverse time order; the adjoint carry g[tile end] stays
// on chip.  Coefficient-gradient partial sums accumulate over the whole row
// and are written once per row: partials[row*3 + {0,1,2}].
template <int NT, int K, int S, bool FUSE_ACT>
__global__ void __launch_bounds__(NT, 3) fbt_bwd_rows_kernel(const FbtArgs a) {
  constexpr int NW = NT / 32, L = NT * K, LK = (K == 4) ? 2 : (K == 8) ? 3 : 4;
  constexpr int WSZ = 16 * K;
  extern __shared__ __align__(16) float4 dsm[];  // [S][2 inputs][NW][WSZ]
  __shared__ float2 s_pw[S][kPowTable];
  __shared__ float2 s_meta[S][2];  // {entry carry C, z sample before the tile}
  __shared__ float2 s_ent[S][NT];  // this tile's per-thread entry states, when saved
  __shared__ float2 s_warp_f[NW];
  __shared__ float2 s_warp_r[NW];
  __shared__ float2 s_red[3][NW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, rows = (int)a.rows, T = (int)a.T, ntiles = a.ntiles;
  const int wofs = warp * 32 * K;
  constexpr size_t stage_sz = (size_t)2 * NW * WSZ;
  static_assert(NT == kFbtSlots, "one saved entry state per thread");
  // The forward saved every thread's entry state (row kernels) or only the
  // tiles' (look-back kernels): one uniform branch per launch.
  const bool per_thread = __ldg(a.carries + fbt_marker(a.rows, ntiles)).x == 1.f;

  // j counts processed tiles of the row; the tile index in time is ntiles-1-j.
  RowCursor ic{(int)blockIdx.x, 0, 0};
  auto issue = [&]() {
    if (ic.row < rows) {
      const int jt = ntiles - 1 - ic.j;
      float4 *base = dsm + ic.stage * stage_sz;
      const size_t roff = (size_t)ic.row * T;
      fbt_issue_tile<K>(base + warp * WSZ, a.z + roff, jt * L + wofs, T, lane);
      fbt_issue_tile<K>(base + (NW + warp) * WSZ, a.gout + roff, jt * L + wofs, T, lane);
      if (per_thread) cp_async8(&s_ent[ic.stage][tid], a.carries + fbt_slot(ic.row, ntiles, jt) + tid,
                                true);
      if (tid == 0) {
        const int t0 = jt * L;
        cp_async8(&s_meta[ic.stage][0], a.carries + fbt_slot(ic.row, ntiles, jt), true);
        cp_async8(&s_meta[ic.stage][1], a.z + roff + (t0 > 0 ? t0 - 1 : 0), t0 > 0);
        stage_table<S>(s_pw, ic.stage, ic.j == 0, a.c1, ic.row / a.batch);
      }
      ic.advance(ntiles, G, S);
    }
    cp_async_commit();
  };

#pragma unroll
  for (int s = 0; s < S - 1; ++s) issue();
  RowCursor pc{(int)blockIdx.x, 0, 0};
  float2 dcarry = cz(), lam = cz(), t0 = cz(), t1 = cz(), lpow_f = cz(), lpow_r = cz();
  float2 acc_c1 = cz(), acc_t0 = cz(), acc_t1 = cz();
  while (pc.row < rows) {
    cp_async_wait<S - 2>();
    __syncthreads();
    issue();
    const int s = pc.stage;
    const int jt = ntiles - 1 - pc.j;
    const float2 *pw = s_pw[s];
    if (pc.j == 0) {
      const int f = pc.row / a.batch;
      lam = pw[0];
      t0 = a.tap0[f];
      t1 = a.tap1[f];
      lpow_f = pow_from_table<false>(pw, LK, lane);
      lpow_r = pow_from_table<true>(pw, LK, 31 - lane);
      dcarry = cz();
    }
    float4 *zbuf = dsm + s * stage_sz + warp * WSZ;
    float4 *gbuf = dsm + s * stage_sz + (NW + warp) * WSZ;
    float2 z[K], go[K];
    read_blocked<K>(zbuf, z, lane);
    read_blocked<K>(gbuf, go, lane);
    float2 zp = shfl_up2(z[K - 1], 1);
    if (lane == 0) zp = warp > 0 ? read_sample<K>(zbuf - WSZ, 32 * K - 1) : s_meta[s][1];

    float2 b[K];
    fbt_drive<K>(t0, t1, z, zp, b);
    float2 e;
    if (per_thread) {
      e = s_ent[s][tid];
    } else {
      float2 y = cz(), At;
#pragma unroll
      for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
      cta_scan_entry_fwd<NT, LK>(y, s_meta[s][0], pw, lpow_f, e, At, s_warp_f);
    }
    float2 yprev[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      yprev[k] = e;
      e = c_fma(lam, e, b[k]);
      b[k] = FUSE_ACT ? c_relu_mask(go[k], e) : go[k];
    }
    const float2 mu = c_conj(lam);
    float2 h = cz();
#pragma unroll
    for (int k = K - 1; k >= 0; --k) h = c_fma(mu, h, b[k]);
    float2 gnext, Art;
    cta_scan_entry_rev<NT, LK>(h, dcarry, pw, lpow_r, gnext, Art, s_warp_r);
    dcarry = Art;  // g at this tile's first sample: right entry of the tile before it
    float2 gz[K];
    // Element-wise products on paired fp32 FMAs: conj(t) g = (t.x, t.x) * g +
    // (t.y, -t.y) * (g.y, g.x); the sums conj(v) g accumulate v * (g.x, g.x) and
    // v * (g.y, g.y) in two pairs, combined once per tile.
    const float2 T0X = make_float2(t0.x, t0.x), T0Y = make_float2(t0.y, -t0.y);
    const float2 T1X = make_float2(t1.x, t1.x), T1Y = make_float2(t1.y, -t1.y);
    float2 pc1 = cz(), qc1 = cz(), pt0 = cz(), qt0 = cz(), pt1 = cz(), qt1 = cz();
    float2 gsw = make_float2(gnext.y, gnext.x);
#pragma unroll
    for (int k = K - 1; k >= 0; --k) {
      const float2 g = c_fma(mu, gnext, b[k]);
      const float2 gs = make_float2(g.y, g.x);
      gz[k] = __ffma2_rn(T0X, g, __ffma2_rn(T0Y, gs, __ffma2_rn(T1X, gnext, __fmul2_rn(T1Y, gsw))));
      const float2 gx = make_float2(g.x, g.x), gy = make_float2(g.y, g.y);
      pc1 = __ffma2_rn(yprev[k], gx, pc1);
      qc1 = __ffma2_rn(yprev[k], gy, qc1);
      pt0 = __ffma2_rn(z[k], gx, pt0);
      qt0 = __ffma2_rn(z[k], gy, qt0);
      const float2 zk1 = k > 0 ? z[k - 1] : zp;
      pt1 = __ffma2_rn(zk1, gx, pt1);
      qt1 = __ffma2_rn(zk1, gy, qt1);
      gnext = g;
      gsw = gs;
    }
    // conj(v) g = (v.x g.x + v.y g.y, v.x g.y - v.y g.x)
    acc_c1 = c_add(acc_c1, make_float2(pc1.x + qc1.y, qc1.x - pc1.y));
    acc_t0 = c_add(acc_t0, make_float2(pt0.x + qt0.y, qt0.x - pt0.y));
    acc_t1 = c_add(acc_t1, make_float2(pt1.x + qt1.y, qt1.x - pt1.y));
    fbt_store_tile<K>(gbuf, gz, a.out + (size_t)pc.row * T, jt * L + wofs, T, lane);
    if (jt == 0) {  // row finished: deterministic CTA reduction of the row's sums
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
        float2 sum = cz();
#pragma unroll
        for (int w = 0; w < NW; ++w) sum = c_add(sum, s_red[tid][w]);
        a.partials[(size_t)pc.row * 3 + tid] = sum;
      }
      acc_c1 = acc_t0 = acc_t1 = cz();
    }
    pc.advance(ntiles, G, S);
  }
  cp_async_wait<0>();
}

// -------------------------------------------------- TBPTT(1) backward
// No temporal adjoint, so tiles run in time order with only the forward
// states replayed from the stored entry carries.  grad_zw[t] = conj(tap1) *
// g[t+1] for the last sample of a tile needs g of the next tile's first
// sample: the next tile (same CTA, next item) writes that one element.
template <int NT, int K, int S, bool FUSE_ACT>
__global__ void __launch_bounds__(NT, 3) fbt_tbptt_rows_kernel(const FbtArgs a) {
  constexpr int NW = NT / 32, L = NT * K, LK = (K == 4) ? 2 : (K == 8) ? 3 : 4;
  constexpr int WSZ = 16 * K;
  extern __shared__ __align__(16) float4 dsm[];  // [S][2 inputs][NW][WSZ]
  __shared__ float2 s_pw[S][kPowTable];
  __shared__ float2 s_meta[S][2];  // {entry carry C, z sample before the tile}
  __shared__ float2 s_ent[S][NT];  // this tile's per-thread entry states, when saved
  __shared__ float2 s_warp_f[NW];
  __shared__ float2 s_gfirst[NW];
  __shared__ float2 s_red[3][NW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, rows = (int)a.rows, T = (int)a.T, ntiles = a.ntiles;
  const int wofs = warp * 32 * K;
  constexpr size_t stage_sz = (size_t)2 * NW * WSZ;
  static_assert(NT == kFbtSlots, "one saved entry state per thread");
  const bool per_thread = __ldg(a.carries + fbt_marker(a.rows, ntiles)).x == 1.f;

  RowCursor ic{(int)blockIdx.x, 0, 0};
  auto issue = [&]() {
    if (ic.row < rows) {
      float4 *base = dsm + ic.stage * stage_sz;
      const size_t roff = (size_t)ic.row * T;
      fbt_issue_tile<K>(base + warp * WSZ, a.z + roff, ic.j * L + wofs, T, lane);
      fbt_issue_tile<K>(base + (NW + warp) * WSZ, a.gout + roff, ic.j * L + wofs, T, lane);
      if (per_thread)
        cp_async8(&s_ent[ic.stage][tid], a.carries + fbt_slot(ic.row, ntiles, ic.j) + tid, true);
      if (tid == 0) {
        const int t0 = ic.j * L;
        cp_async8(&s_meta[ic.stage][0], a.carries + fbt_slot(ic.row, ntiles, ic.j), true);
        cp_async8(&s_meta[ic.stage][1], a.z + roff + (t0 > 0 ? t0 - 1 : 0), t0 > 0);
        stage_table<S>(s_pw, ic.stage, ic.j == 0, a.c1, ic.row / a.batch);
      }
      ic.advance(ntiles, G, S);
    }
    cp_async_commit();
  };

#pragma unroll
  for (int s = 0; s < S - 1; ++s) issue();
  RowCursor pc{(int)blockIdx.x, 0, 0};
  float2 lam = cz(), t0c = cz(), t1c = cz(), lpow = cz();
  float2 acc_c1 = cz(), acc_t0 = cz(), acc_t1 = cz();
  while (pc.row < rows) {
    cp_async_wait<S - 2>();
    __syncthreads();
    issue();
    const int s = pc.stage;
    const float2 *pw = s_pw[s];
    if (pc.j == 0) {
      const int f = pc.row / a.batch;
      lam = pw[0];
      t0c = a.tap0[f];
      t1c = a.tap1[f];
      lpow = pow_from_table<false>(pw, LK, lane);
    }
    float4 *zbuf = dsm + s * stage_sz + warp * WSZ;
    float4 *gbuf = dsm + s * stage_sz + (NW + warp) * WSZ;
    const size_t roff = (size_t)pc.row * T;
    const int tile0 = pc.j * L;
    float2 z[K], go[K];
    read_blocked<K>(zbuf, z, lane);
    read_blocked<K>(gbuf, go, lane);
    float2 zp = shfl_up2(z[K - 1], 1);
    if (lane == 0) zp = warp > 0 ? read_sample<K>(zbuf - WSZ, 32 * K - 1) : s_meta[s][1];
    // The drive exactly as every forward forms it (fbt_drive), so the
    // replayed states, and with them the split-ReLU decisions, are the
    // forward's bit for bit.
    float2 b[K];
    fbt_drive<K>(t0c, t1c, z, zp, b);
    float2 e;
    if (per_thread) {
      e = s_ent[s][tid];
    } else {
      float2 y = cz(), At;
#pragma unroll
      for (int k = 0; k < K; ++k) y = c_fma(lam, y, b[k]);
      cta_scan_entry_fwd<NT, LK>(y, s_meta[s][0], pw, lpow, e, At, s_warp_f);
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const float2 yp = e;
      e = c_fma(lam, e, b[k]);
      go[k] = FUSE_ACT ? c_relu_mask(go[k], e) : go[k];
      acc_c1 = c_cfma(yp, go[k], acc_c1);
      acc_t0 = c_cfma(z[k], go[k], acc_t0);
      acc_t1 = c_cfma(k > 0 ? z[k - 1] : zp, go[k], acc_t1);
    }
    float2 gn = shfl_down2(go[0], 1);
    if (lane == 0) s_gfirst[warp] = go[0];
    __syncthreads();
    if (lane == 31) gn = warp + 1 < NW ? s_gfirst[warp + 1] : cz();
    float2 dz[K], dzw[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      dz[k] = c_cfma(t0c, go[k], cz());
      dzw[k] = c_cfma(t1c, k + 1 < K ? go[k + 1] : gn, a.wsum ? dz[k] : cz());
    }
    // The lag tap of the tile before's last sample.  With wsum that tile
    // stored its grad_z there (the same CTA, ordered by the loop's barrier),
    // so this adds to it.
    if (tid == 0 && pc.j > 0)
      __stcs(a.out2 + roff + tile0 - 1,
             c_cfma(t1c, go[0], a.wsum ? __ldcg(a.out2 + roff + tile0 - 1) : cz()));
    fbt_store_tile<K>(gbuf, dz, a.out + roff, tile0 + wofs, T, lane);
    // grad_zw staged through the z region (every warp has read its z samples
    // before the scan barrier).  The tile's last sample needs g of the next
    // tile: unless this is the row's last tile, only the first half of that
    // pair is stored here and the next tile stores the other (with wsum the
    // whole pair is stored, the last sample holding its grad_z, which the
    // next tile completes).
    const int last = tile0 + L - 1;
#pragma unroll
    for (int m = 0; m < K / 2; ++m)
      zbuf[swz<K>(lane * (K / 2) + m)] =
          make_float4(dzw[2 * m].x, dzw[2 * m].y, dzw[2 * m + 1].x, dzw[2 * m + 1].y);
    __syncwarp();
#pragma unroll
    for (int v = 0; v < K / 2; ++v) {
      const int t = tile0 + wofs + 2 * (v * 32 + lane);
      if (t >= T) continue;
      const float4 q = zbuf[swz<K>(v * 32 + lane)];
      if (t + 1 == last && pc.j + 1 < ntiles && !a.wsum)
        __stcs(a.out2 + roff + t, make_float2(q.x, q.y));
      else
        st_stream4(a.out2 + roff + t, q);
    }
    if (pc.j + 1 == ntiles) {  // row finished
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
        float2 sum = cz();
#pragma unroll
        for (int w = 0; w < NW; ++w) sum = c_add(sum, s_red[tid][w]);
        a.partials[(size_t)pc.row * 3 + tid] = sum;
      }
      acc_c1 = acc_t0 = acc_t1 = cz();
    }
    pc.advance(ntiles, G, S);
  }
  cp_async_wait<0>();
}

}  // namespace rqf
