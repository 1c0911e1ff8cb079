// Hidden layer of the mean-pooled per-timestep readout
// (train.py:ComplexReadoutClassifier :74-136: Linear(2F, H) -> ReLU ->
// Linear(H, C) per step, logits mean-pooled over time).  With the output
// layer applied after pooling, the hidden layer only has to deliver
//
//   pooled[h, b] = (1/T) sum_t relu(Re z[h, b, t] + bias[h])
//
// where Re z = Re(V h_enc) is the real part of the complex projection of the
// encoder state (rqf_projection_real_out writes it as float32), and its
// backward only needs the ReLU mask:
//
//   g[h, b, t] = mask[h, b, t] * gpool[h, b] / T
//
// Both kernels work one (h, b) row of T samples per CTA, one 32-sample word of
// the bit mask per warp iteration (bit t % 32 of word t / 32), and reduce in a
// fixed order (deterministic).  Both are HBM-bound: the forward reads Re z
// once (4 bytes per sample) and writes 1 bit; the backward reads the bit and writes
// the real cotangent (4 bytes) that the real-operand projection GEMMs take.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rqf {
namespace readout {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__global__ void __launch_bounds__(kThreads)
relu_pool_kernel(const float *__restrict__ z, const float *__restrict__ bias,
                 uint32_t *__restrict__ mask, float *__restrict__ pooled, int batch,
                 long long T, long long words) {
  const long long row = blockIdx.x;  // h * batch + b
  const float bh = bias ? bias[row / batch] : 0.f;
  const float *zr = z + row * T;
  uint32_t *mr = mask + row * words;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float acc = 0.f;
  // four words per warp iteration, their loads issued before any is used
  constexpr int kU = 4;
  for (long long w0 = warp; w0 < words; w0 += kU * kWarps) {
    float v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long t = (w0 + u * kWarps) * 32 + lane;
      v[u] = t < T ? zr[t] : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long w = w0 + u * kWarps;
      const float x = v[u] + bh;
      const bool on = x > 0.f;  // false past T (and for whole words past the end)
      const uint32_t bits = __ballot_sync(0xffffffffu, on);
      if (lane == 0 && w < words) mr[w] = bits;
      if (on) acc += x;
    }
  }
  __shared__ double red[kThreads];
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = kThreads / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) pooled[row] = (float)(red[0] / (double)T);
}

// g[row, t] = mask ? scale[row] : 0; counts[row] = number of set bits.
__global__ void __launch_bounds__(kThreads)
relu_pool_backward_kernel(const uint32_t *__restrict__ mask, const float *__restrict__ scale,
                          float *__restrict__ gc, float *__restrict__ counts, long long T,
                          long long words) {
  const long long row = blockIdx.x;
  const float s = scale[row];
  const uint32_t *mr = mask + row * words;
  float *gr = gc + row * T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int cnt = 0;
  for (long long w = warp; w < words; w += kWarps) {
    const uint32_t bits = mr[w];
    const long long t = w * 32 + lane;
    if (t < T) gr[t] = ((bits >> lane) & 1u) ? s : 0.f;
    if (lane == 0) cnt += __popc(bits);
  }
  __shared__ int red[kThreads];
  red[threadIdx.x] = cnt;
  __syncthreads();
  for (int k = kThreads / 2; k > 0; k >>= 1) {
    if (threadIdx.x < k) red[threadIdx.x] += red[threadIdx.x + k];
    __syncthreads();
  }
  if (threadIdx.x == 0 && counts) counts[row] = (float)red[0];
}

}  // namespace readout
}  // namespace rqf
