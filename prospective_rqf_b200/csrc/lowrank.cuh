// The first block of the Pure RQF stack over a low-rank input projection
// (rqf_models/backbones/rqf/pure.py:_forward_fbt_stack :510-534).  The
// projected input h0 = w_in x (+ b_in) has rank <= I (+1) with I = input_dims
// (1 for the waveform models), so the block's projection z0 = W h0 equals
// U x (+ beta) with U = W w_in (F x I) and beta = W b_in, and its weight
// cotangent gz0 h0^H equals (gz0 x^T) w_in^T (+ (gz0 1) b_in^T).  Two
// HBM-bound kernels replace the F x F projection GEMMs of that block:
//
//   lowrank_drive_kernel   z0 = U x + beta and h0 = w_in x + b_in (complex,
//                          zero imaginary part), written in one pass;
//   rowdot_*_kernel        out[f][j] = sum_n A[f][n] x_j[n] for a complex
//                          (F, N) A and real rows x_j (x_I = 1 gives the row
//                          sums), in a fixed order: per-(row, chunk) partial
//                          sums reduced in double, then summed over chunks
//                          in chunk order.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rqf {
namespace lowrank {

constexpr int kMaxRank = 4;        // input channels handled (I <= kMaxRank)
constexpr int kMaxCols = kMaxRank + 1;  // + the row sum
constexpr int kRowdotThreads = 256;
constexpr long long kRowdotChunk = 16384;  // samples per partial

// z[f][n] = sum_i U[f][i] x[i][n] + beta[f];  h[f][n] = sum_i w[f][i] x[i][n] + b[f].
// U, beta complex; w, b real; beta, b, h may be null.  Two samples per thread.
__global__ void __launch_bounds__(256)
lowrank_drive_kernel(const float2 *__restrict__ U, const float2 *__restrict__ beta,
                     const float *__restrict__ w, const float *__restrict__ b,
                     const float *__restrict__ x, float2 *__restrict__ z, float2 *__restrict__ h,
                     long long F, long long N, int I) {
  const long long pairs = N >> 1;  // N is even
  const long long total = F * pairs;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long f = e / pairs;
    const long long n = (e - f * pairs) * 2;
    float2 z0 = beta ? beta[f] : make_float2(0.f, 0.f), z1 = z0;
    float h0 = b ? b[f] : 0.f, h1 = h0;
    for (int i = 0; i < I; ++i) {
      const float2 xv = *reinterpret_cast<const float2 *>(x + (long long)i * N + n);
      const float2 u = U[f * I + i];
      z0.x = fmaf(u.x, xv.x, z0.x);
      z0.y = fmaf(u.y, xv.x, z0.y);
      z1.x = fmaf(u.x, xv.y, z1.x);
      z1.y = fmaf(u.y, xv.y, z1.y);
      if (h) {
        const float wv = w[f * I + i];
        h0 = fmaf(wv, xv.x, h0);
        h1 = fmaf(wv, xv.y, h1);
      }
    }
    reinterpret_cast<float4 *>(z + f * N + n)[0] = make_float4(z0.x, z0.y, z1.x, z1.y);
    if (h) reinterpret_cast<float4 *>(h + f * N + n)[0] = make_float4(h0, 0.f, h1, 0.f);
  }
}

// One CTA per (row f, chunk c): partials[(f * chunks + c) * J + j] for the J =
// I + with_sum columns.  Each thread sums a strided subset in fp32 (at most
// kRowdotChunk / (2 * kRowdotThreads) = 32 pairs), the CTA combines the
// threads in double in a fixed tree.
__global__ void __launch_bounds__(kRowdotThreads)
rowdot_partial_kernel(const float2 *__restrict__ A, const float *__restrict__ x,
                      double2 *__restrict__ partials, long long N, int I, int with_sum,
                      int chunks) {
  const long long f = blockIdx.y;
  const int c = blockIdx.x;
  const int J = I + with_sum;
  const long long n0 = (long long)c * kRowdotChunk;
  const long long n1 = n0 + kRowdotChunk < N ? n0 + kRowdotChunk : N;
  float2 acc[kMaxCols];
#pragma unroll
  for (int j = 0; j < kMaxCols; ++j) acc[j] = make_float2(0.f, 0.f);
  const float2 *row = A + f * N;
  // kUnroll pairs per thread per iteration, loaded before any is used, so
  // that each thread keeps kUnroll 16-byte loads in flight
  constexpr int kUnroll = 4;
  constexpr long long kStep = 2LL * kRowdotThreads;
  long long n = n0 + 2 * threadIdx.x;
  for (; n + (kUnroll - 1) * kStep < n1; n += kUnroll * kStep) {
    float4 a[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) a[u] = *reinterpret_cast<const float4 *>(row + n + u * kStep);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long m = n + u * kStep;
#pragma unroll
      for (int j = 0; j < kMaxCols; ++j) {
        if (j >= J) break;
        float2 xv = make_float2(1.f, 1.f);
        if (j < I) xv = *reinterpret_cast<const float2 *>(x + (long long)j * N + m);
        acc[j].x = fmaf(a[u].x, xv.x, fmaf(a[u].z, xv.y, acc[j].x));
        acc[j].y = fmaf(a[u].y, xv.x, fmaf(a[u].w, xv.y, acc[j].y));
      }
    }
  }
  for (; n < n1; n += kStep) {
    const float4 a = *reinterpret_cast<const float4 *>(row + n);  // samples n, n + 1
#pragma unroll
    for (int j = 0; j < kMaxCols; ++j) {
      if (j >= J) break;
      float2 xv = make_float2(1.f, 1.f);
      if (j < I) xv = *reinterpret_cast<const float2 *>(x + (long long)j * N + n);
      acc[j].x = fmaf(a.x, xv.x, fmaf(a.z, xv.y, acc[j].x));
      acc[j].y = fmaf(a.y, xv.x, fmaf(a.w, xv.y, acc[j].y));
    }
  }
  __shared__ double2 red[kRowdotThreads];
  for (int j = 0; j < J; ++j) {
    red[threadIdx.x] = make_double2(acc[j].x, acc[j].y);
    __syncthreads();
    for (int s = kRowdotThreads / 2; s > 0; s >>= 1) {
      if (threadIdx.x < s) {
        red[threadIdx.x].x += red[threadIdx.x + s].x;
        red[threadIdx.x].y += red[threadIdx.x + s].y;
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) partials[(f * chunks + c) * J + j] = red[0];
    __syncthreads();
  }
}

// out[f * J + j] = sum over chunks in order (double), as complex64.
__global__ void rowdot_finish_kernel(const double2 *__restrict__ partials, float2 *__restrict__ out,
                                     long long F, int J, int chunks) {
  const long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e >= F * J) return;
  const long long f = e / J;
  const int j = (int)(e - f * J);
  double re = 0.0, im = 0.0;
  for (int c = 0; c < chunks; ++c) {
    const double2 v = partials[(f * chunks + c) * J + j];
    re += v.x;
    im += v.y;
  }
  out[e] = make_float2((float)re, (float)im);
}

}  // namespace lowrank
}  // namespace rqf
