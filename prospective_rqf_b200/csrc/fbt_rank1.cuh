// The first Pure RQF block over a rank-1 input (input_dims == 1: the waveform
// classification models, one input channel), with the block's drive and skip made
// inside the (F,B,T) row kernels from the 4-byte input instead of read from
// HBM (rqf_models/backbones/rqf/pure.py:_forward_fbt_stack :510-534 and
// PureRQFBlock._forward_fbt :212-243):
//
//   z[f, b, t]  = u[f] x[b, t] + beta[f]       (u = W w_in, beta = W b_in)
//   h0[f, b, t] = w[f] x[b, t] + bb[f]         (the input projection, real)
//   out         = act(y) + h0                  y the two-tap scan of z
//
// with the same fmaf operations as lowrank_drive_kernel, so z and h0 are the
// values that kernel would have written.  The forward saves the (F,B,T)
// context of the row kernels (every thread's entry state, the marker), and
// the backward replays the states from it, regenerating z from x.  The
// backward writes no grad_z: its only consumers are the row sums
//
//   G[f]  = (sum_{b,t} gz x, sum_{b,t} gz)     gW = G [w_in, b_in]^T
//   Gs[f] = (sum_{b,t} g x,  sum_{b,t} g)      the skip's part of the input
//                                              projection's cotangent
//
// which it accumulates per row beside the coefficient sums (reduced over the
// batch in a fixed order in double by reduce_rows4_kernel).  So the block
// moves 4 bytes of input per sample plus its output (forward) or its output
// cotangent (backward), against z, h0 and gz in the general path.  The same
// backward kernel also serves the block's TBPTT(1) surrogate (TRUNC: no
// adjoint recursion, and the row sums of grad_z plus the lag cotangent for
// the weight cotangent; pure.py:184-187).
//
// Tiling, pipeline and scans are those of fbt_rows.cuh (kFbtThreads threads x
// kFbtK samples per tile); x tiles are 4 bytes per sample, staged by cp.async
// (16-byte pieces: T must be a multiple of 4) into the first half of each
// warp's stage region, whose 2 KB then stage the outputs.
#pragma once

#include "fbt_rows.cuh"

namespace rqf {

struct Rank1Args {
  const float2 *u, *beta;  // (F,) complex; beta may be null
  const float *w, *bb;     // (F,) real; w null: no skip; bb may be null
  const float *x;          // (B, T) real
  float2 *rowsums;         // backward: (rows, 4) {sum gz x, sum gz, sum g x, sum g}
};

// Slot of lane l's q-th 16-byte piece of x in its warp region (8 floats per
// lane): the XOR keeps the reads of a quarter warp on distinct banks.
__device__ __forceinline__ int r1_slot(int lane, int q) { return 2 * lane + (q ^ ((lane >> 2) & 1)); }

template <int K>
__device__ __forceinline__ void r1_issue_x(float4 *wbuf, const float *xrow, int wstart, int T,
                                           int lane) {
  static_assert(K == 8, "8 samples (two 16-byte pieces) per lane");
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int t = wstart + 8 * lane + 4 * q;  // T % 4 == 0: a piece is wholly in or out
    const bool in = t < T;
    cp_async16(wbuf + r1_slot(lane, q), in ? xrow + t : xrow, in);
  }
}

template <int K>
__device__ __forceinline__ void r1_read_x(const float4 *wbuf, float (&xv)[K], int lane) {
  const float4 a = wbuf[r1_slot(lane, 0)], b = wbuf[r1_slot(lane, 1)];
  xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
  xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
}
// The last sample of a warp region (lane 31's second piece).
__device__ __forceinline__ float r1_last_x(const float4 *wbuf) { return wbuf[r1_slot(31, 1)].w; }

__device__ __forceinline__ float2 r1_z(float2 u, float2 be, float xv) {
  return make_float2(fmaf(u.x, xv, be.x), fmaf(u.y, xv, be.y));
}

// ------------------------------------------------------------ forward
template <int NT, int K, int S, bool FUSE_ACT>
__global__ void __launch_bounds__(NT) fbt_rank1_fwd_kernel(const FbtArgs a, const Rank1Args r) {
  constexpr int NW = NT / 32, L = NT * K, LK = (K == 4) ? 2 : (K == 8) ? 3 : 4;
  constexpr int WSZ = 16 * K;  // float4 slots per warp region: x in the first 64, outputs in all
  extern __shared__ __align__(16) float4 dsm[];  // [S][NW][WSZ]
  __shared__ float2 s_pw[S][kPowTable];
  __shared__ float2 s_warp[NW];
  __shared__ float2 s_zlast;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, rows = (int)a.rows, T = (int)a.T, ntiles = a.ntiles;
  const int wofs = warp * 32 * K;
  const bool skip = r.w != nullptr;

  static_assert(NT == kFbtSlots, "one saved entry state per thread");
  if (blockIdx.x == 0 && tid == 0)
    a.carries[fbt_marker(a.rows, ntiles)] = make_float2(1.f, 0.f);  // every slot written
  RowCursor ic{(int)blockIdx.x, 0, 0};
  auto issue = [&]() {
    if (ic.row < rows) {
      const int b = ic.row % a.batch;
      r1_issue_x<K>(dsm + ((size_t)ic.stage * NW + warp) * WSZ, r.x + (size_t)b * T,
                    ic.j * L + wofs, T, lane);
      if (tid == 0) stage_table<S>(s_pw, ic.stage, ic.j == 0, a.c1, ic.row / a.batch);
      ic.advance(ntiles, G, S);
    }
    cp_async_commit();
  };

#pragma unroll
  for (int s = 0; s < S - 1; ++s) issue();
  RowCursor pc{(int)blockIdx.x, 0, 0};
  float2 carry = cz(), lam = cz(), t0 = cz(), t1 = cz(), lanepow = cz(), u = cz(), be = cz();
  float wf = 0.f, bf = 0.f;
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
      u = r.u[f];
      be = r.beta ? r.beta[f] : cz();
      wf = skip ? r.w[f] : 0.f;
      bf = r.bb ? r.bb[f] : 0.f;
      lanepow = pow_from_table<false>(pw, LK, lane);
      carry = cz();
    }
    float4 *wbuf = dsm + ((size_t)pc.stage * NW + warp) * WSZ;
    float xv[K];
    r1_read_x<K>(wbuf, xv, lane);
    float2 z[K];
#pragma unroll
    for (int k = 0; k < K; ++k) z[k] = r1_z(u, be, xv[k]);
    float2 zp = shfl_up2(z[K - 1], 1);
    if (lane == 0) {
      if (warp > 0)
        zp = r1_z(u, be, r1_last_x(wbuf - WSZ));
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
    a.carries[fbt_slot(pc.row, ntiles, pc.j) + tid] = e;
    carry = At;
    float2 o[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      e = c_fma(lam, e, b[k]);
      o[k] = FUSE_ACT ? c_relu(e) : e;
      if (skip) o[k] = c_add(o[k], make_float2(fmaf(wf, xv[k], bf), 0.f));
    }
    fbt_store_tile<K>(wbuf, o, a.out + (size_t)pc.row * T, pc.j * L + wofs, T, lane);
    pc.advance(ntiles, G, S);
  }
  cp_async_wait<0>();
}

// ------------------------------------------------------------ backward
// Tiles of a row in reverse time order, as fbt_bwd_rows_kernel, with z made
// from x and the forward's per-thread entry states (required: the forward of
// this file saves them).  Per row: the coefficient sums into a.partials
// (rows, 3) and the row sums into r.rowsums (rows, 4; rows, 6 with TRUNC);
// the plain sums (sum gz, sum g, sum gsum: the bias's terms) only with WSUM,
// zero otherwise.
// TRUNC: the TBPTT(1) surrogate (the (F,B,T) TBPTT(1) kernels' gradients):
// no adjoint recursion, d[t] = mask(y[t]) g[t]; grad_z[t] = conj(tap0) d[t]
// and the lag tap's cotangent conj(tap1) d[t+1], whose sum with it (gsum)
// takes the weight cotangent.  Row sums: {sum gz x, sum gz, sum g x, sum g,
// sum gsum x, sum gsum}.
template <int NT, int K, int S, bool FUSE_ACT, bool WSUM, bool TRUNC = false>
__global__ void __launch_bounds__(NT, 3) fbt_rank1_bwd_kernel(const FbtArgs a, const Rank1Args r) {
  constexpr int NW = NT / 32, L = NT * K, LK = (K == 4) ? 2 : (K == 8) ? 3 : 4;
  constexpr int WSZ = 16 * K;
  extern __shared__ __align__(16) float4 dsm[];  // [S][2 inputs][NW][WSZ]
  __shared__ float2 s_pw[S][kPowTable];
  __shared__ float s_xprev[S];     // x at the sample before the tile
  __shared__ float2 s_ent[S][NT];  // this tile's per-thread entry states
  __shared__ float2 s_warp_r[NW];
  __shared__ float2 s_red[7][NW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, rows = (int)a.rows, T = (int)a.T, ntiles = a.ntiles;
  const int wofs = warp * 32 * K;
  constexpr size_t stage_sz = (size_t)2 * NW * WSZ;
  static_assert(NT == kFbtSlots, "one saved entry state per thread");
  if (blockIdx.x == 0 && tid == 0 && __ldg(a.carries + fbt_marker(a.rows, ntiles)).x != 1.f)
    latch_error(5);  // RQF_ERR_ARGUMENT: the context lacks the per-thread entries

  RowCursor ic{(int)blockIdx.x, 0, 0};
  auto issue = [&]() {
    if (ic.row < rows) {
      const int jt = ntiles - 1 - ic.j;
      float4 *base = dsm + ic.stage * stage_sz;
      const size_t roff = (size_t)ic.row * T;
      const float *xrow = r.x + (size_t)(ic.row % a.batch) * T;
      r1_issue_x<K>(base + warp * WSZ, xrow, jt * L + wofs, T, lane);
      fbt_issue_tile<K>(base + (NW + warp) * WSZ, a.gout + roff, jt * L + wofs, T, lane);
      cp_async8(&s_ent[ic.stage][tid], a.carries + fbt_slot(ic.row, ntiles, jt) + tid, true);
      if (tid == 0) {
        const int t0 = jt * L;
        cp_async4(&s_xprev[ic.stage], xrow + (t0 > 0 ? t0 - 1 : 0), t0 > 0);
        stage_table<S>(s_pw, ic.stage, ic.j == 0, a.c1, ic.row / a.batch);
      }
      ic.advance(ntiles, G, S);
    }
    cp_async_commit();
  };

#pragma unroll
  for (int s = 0; s < S - 1; ++s) issue();
  RowCursor pc{(int)blockIdx.x, 0, 0};
  float2 dcarry = cz(), lam = cz(), t0 = cz(), t1 = cz(), lpow_r = cz(), u = cz(), be = cz();
  // Running sums of the row, all linear in the adjoint d because z is rank 1
  // in x (z = u x + beta, and z = 0 before the row's first sample):
  //   acc_c1  sum conj(y[t-1]) d[t] as its (g.x, g.x), (g.y, g.y) pair halves
  //   sd      sum d[t]             sxd  sum x[t] d[t]      sxpd  sum x[t-1] d[t]
  //   sgx     sum x[t] g[t]        sg   sum g[t] (WSUM)     g the output cotangent
  // so that, with d0 = d at the row's first sample and d past the row zero,
  //   sum conj(z[t]) d[t]     = conj(u) sxd  + conj(beta) sd
  //   sum conj(z[t-1]) d[t]   = conj(u) sxpd + conj(beta) (sd - d0)
  //   sum gz x = conj(tap0) sxd + conj(tap1) sxpd     (sum x[t] d[t+1] = sxpd)
  //   sum gz   = conj(tap0) sd  + conj(tap1) (sd - d0)
  // with gz[t] = conj(tap0) d[t] + conj(tap1) d[t+1].
  float2 pc1r = cz(), qc1r = cz(), sd = cz(), sxd = cz(), sxpd = cz(), sgx = cz(), sg = cz();
  float2 d0 = cz();
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
      u = r.u[f];
      be = r.beta ? r.beta[f] : cz();
      lpow_r = pow_from_table<true>(pw, LK, 31 - lane);
      dcarry = cz();
    }
    float4 *xbuf = dsm + s * stage_sz + warp * WSZ;
    float4 *gbuf = dsm + s * stage_sz + (NW + warp) * WSZ;
    float xv[K];
    r1_read_x<K>(xbuf, xv, lane);
    float2 go[K];
    read_blocked<K>(gbuf, go, lane);
    // x before the thread's first sample (zero before the row's first)
    float xp = __shfl_up_sync(0xffffffffu, xv[K - 1], 1);
    if (lane == 0) xp = warp > 0 ? r1_last_x(xbuf - WSZ) : (jt > 0 ? s_xprev[s] : 0.f);
    const bool row_start = jt == 0 && tid == 0;
    float2 b[K];
    {
      float2 z[K];
#pragma unroll
      for (int k = 0; k < K; ++k) z[k] = r1_z(u, be, xv[k]);
      fbt_drive<K>(t0, t1, z, row_start ? cz() : r1_z(u, be, xp), b);
    }
    float2 e = s_ent[s][tid];
    float2 yprev[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      yprev[k] = e;
      e = c_fma(lam, e, b[k]);
      b[k] = FUSE_ACT ? c_relu_mask(go[k], e) : go[k];
      sgx = __ffma2_rn(make_float2(xv[k], xv[k]), go[k], sgx);  // go dies here
      if constexpr (WSUM) sg = c_add(sg, go[k]);
    }
    const float2 mu = c_conj(lam);
    float2 gnext = cz();
    if constexpr (!TRUNC) {
      float2 h = cz();
#pragma unroll
      for (int k = K - 1; k >= 0; --k) h = c_fma(mu, h, b[k]);
      float2 Art;
      cta_scan_entry_rev<NT, LK>(h, dcarry, pw, lpow_r, gnext, Art, s_warp_r);
      dcarry = Art;
    }
    float2 pc1 = cz(), qc1 = cz();
#pragma unroll
    for (int k = K - 1; k >= 0; --k) {
      const float2 g = TRUNC ? b[k] : c_fma(mu, gnext, b[k]);
      const float2 xx = make_float2(xv[k], xv[k]);
      const float xpk = k > 0 ? xv[k - 1] : xp;
      sd = c_add(sd, g);
      sxd = __ffma2_rn(xx, g, sxd);
      sxpd = __ffma2_rn(make_float2(xpk, xpk), g, sxpd);
      pc1 = __ffma2_rn(yprev[k], make_float2(g.x, g.x), pc1);
      qc1 = __ffma2_rn(yprev[k], make_float2(g.y, g.y), qc1);
      gnext = g;
    }
    if (row_start) d0 = gnext;  // d at the row's first sample
    pc1r = c_add(pc1r, pc1);
    qc1r = c_add(qc1r, qc1);
    if (jt == 0) {  // row finished: deterministic CTA reduction of the row's sums
      auto warp_sum = [&](float2 v, int q) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = c_add(v, shfl_xor2(v, o));
        if (lane == 0) s_red[q][warp] = v;
      };
      warp_sum(make_float2(pc1r.x + qc1r.y, qc1r.x - pc1r.y), 0);
      warp_sum(sd, 1);
      warp_sum(sxd, 2);
      warp_sum(sxpd, 3);
      warp_sum(sgx, 4);
      warp_sum(sg, 5);
      if (tid == 0) s_red[6][0] = d0;
      __syncthreads();
      if (tid < 6) {
        float2 sum = cz();
#pragma unroll
        for (int w = 0; w < NW; ++w) sum = c_add(sum, s_red[tid][w]);
        s_red[tid][0] = sum;  // each thread reads and writes only its own q
      }
      __syncthreads();
      if (tid < (TRUNC ? 9 : 7)) {
        const float2 Sd = s_red[1][0], Sxd = s_red[2][0], Sxpd = s_red[3][0];
        const float2 Sd1 = make_float2(Sd.x - s_red[6][0].x, Sd.y - s_red[6][0].y);  // d past t = 0
        const float2 cu = c_conj(u), cb = c_conj(be), ct0 = c_conj(t0), ct1 = c_conj(t1);
        // with the adjoint recursion gz[t] = conj(tap0) d[t] + conj(tap1) d[t+1]
        // (sum x[t] d[t+1] = sxpd); TRUNC: gz[t] = conj(tap0) d[t], and gsum has
        // the recursion's form
        const float2 lag_x = c_add(c_mul(ct0, Sxd), c_mul(ct1, Sxpd));
        const float2 lag_1 = WSUM ? c_add(c_mul(ct0, Sd), c_mul(ct1, Sd1)) : cz();
        float2 v;
        switch (tid) {
          case 0: v = s_red[0][0]; break;                                  // conj(y[t-1]) d
          case 1: v = c_add(c_mul(cu, Sxd), c_mul(cb, Sd)); break;        // conj(z[t]) d
          case 2: v = c_add(c_mul(cu, Sxpd), c_mul(cb, Sd1)); break;      // conj(z[t-1]) d
          case 3: v = TRUNC ? c_mul(ct0, Sxd) : lag_x; break;             // sum gz x
          case 4: v = TRUNC ? (WSUM ? c_mul(ct0, Sd) : cz()) : lag_1; break;  // sum gz
          case 5: v = s_red[4][0]; break;                                  // sum g x
          case 6: v = s_red[5][0]; break;                                  // sum g
          case 7: v = lag_x; break;                                        // sum gsum x
          default: v = lag_1; break;                                       // sum gsum
        }
        if (tid < 3)
          a.partials[(size_t)pc.row * 3 + tid] = v;
        else
          r.rowsums[(size_t)pc.row * (TRUNC ? 6 : 4) + (tid - 3)] = v;
      }
      pc1r = qc1r = sd = sxd = sxpd = sgx = sg = d0 = cz();
    }
    pc.advance(ntiles, G, S);
  }
  cp_async_wait<0>();
}

// The sum over the batch of rowsums[(f * batch + b) * R + q], R = 4 or 6, in
// increasing b, in double: q = 0, 1 into gzx[f * 2 + q], q = 2, 3 into
// gsx[f * 2 + q - 2], q = 4, 5 into gwx[f * 2 + q - 4] (gsx, gwx may be null).
// One thread per (f, q).
__global__ void reduce_rows4_kernel(const float2 *__restrict__ rowsums, float2 *__restrict__ gzx,
                                    float2 *__restrict__ gsx, float2 *__restrict__ gwx,
                                    long long F, int batch, int R) {
  const long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e >= F * R) return;
  const long long f = e / R;
  const int q = (int)(e - f * R);
  float2 *dst = q < 2 ? gzx + f * 2 + q
                : q < 4 ? (gsx ? gsx + f * 2 + (q - 2) : nullptr)
                        : (gwx ? gwx + f * 2 + (q - 4) : nullptr);
  if (!dst) return;
  double re = 0.0, im = 0.0;
  for (int b = 0; b < batch; ++b) {
    const float2 v = rowsums[(f * batch + b) * R + q];
    re += v.x;
    im += v.y;
  }
  *dst = make_float2((float)re, (float)im);
}

}  // namespace rqf
