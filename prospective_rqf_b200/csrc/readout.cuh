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

#include "rqf_common.cuh"

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

// The per-step hidden layer's bias and ReLU in place: z[row, t] = relu(z +
// bias[row / batch]) and its mask bits (as relu_pool_kernel writes them).
__global__ void __launch_bounds__(kThreads)
bias_relu_kernel(float *__restrict__ z, const float *__restrict__ bias, uint32_t *__restrict__ mask,
                 int batch, long long T, long long words) {
  const long long row = blockIdx.x;
  const float bh = bias ? bias[row / batch] : 0.f;
  float *zr = z + row * T;
  uint32_t *mr = mask + row * words;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
      const long long w = w0 + u * kWarps, t = w * 32 + lane;
      const float x = v[u] + bh;
      const bool on = x > 0.f;
      const uint32_t bits = __ballot_sync(0xffffffffu, on);
      if (lane == 0 && w < words) mr[w] = bits;
      if (t < T) zr[t] = on ? x : 0.f;
    }
  }
}

// Its backward: g[row, t] = mask ? gy[row, t] : 0, and rowsum[row] = sum_t g
// (in double, fixed order): the bias's cotangent before the sum over batch.
__global__ void __launch_bounds__(kThreads)
bias_relu_backward_kernel(const float *__restrict__ gy, const uint32_t *__restrict__ mask,
                          float *__restrict__ g, float *__restrict__ rowsum, long long T,
                          long long words) {
  const long long row = blockIdx.x;
  const float *gr = gy + row * T;
  float *out = g + row * T;
  const uint32_t *mr = mask + row * words;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double acc = 0.0;
  for (long long w = warp; w < words; w += kWarps) {
    const uint32_t bits = mr[w];
    const long long t = w * 32 + lane;
    if (t < T) {
      const float v = ((bits >> lane) & 1u) ? gr[t] : 0.f;
      out[t] = v;
      acc += v;
    }
  }
  __shared__ double red[kThreads];
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int k = kThreads / 2; k > 0; k >>= 1) {
    if (threadIdx.x < k) red[threadIdx.x] += red[threadIdx.x + k];
    __syncthreads();
  }
  if (threadIdx.x == 0 && rowsum) rowsum[row] = (float)red[0];
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

// ------------------------------------------------ per-step cross entropy
// The loss of per-timestep logits (train.py:per_step_cross_entropy :663-674:
// torch cross_entropy over the (batch*time, classes) view, the label of batch
// row b for each of its time steps, label smoothing eps, mean reduction),
// read in the layout the readout's output GEMM writes: logits (C, N) with
// sample n = b T + t.  Per sample:
//   loss_n = lse_n - (1 - eps) l[y] - (eps / C) sum_c l[c],
//   dl[c]  = (softmax_c - (1 - eps) [c == y] - eps / C) g / N,
// with lse_n = m + log sum_c exp(l[c] - m) in one pass (running maximum m).
// The sum over samples is per block in double, then over blocks in a fixed
// order (deterministic).  A label outside [0, C) latches RQF_ERR_ARGUMENT
// and counts as class 0.
constexpr int kCeThreads = 256;

__device__ __forceinline__ void ce_lse(const float *__restrict__ l, long long N, long long n, int C,
                                       float &lse, float &sum) {
  float m = -INFINITY, s = 0.f;
  sum = 0.f;
  for (int c = 0; c < C; ++c) {
    const float v = l[(long long)c * N + n];
    sum += v;
    if (v > m) {
      s = s * expf(m - v) + 1.f;
      m = v;
    } else {
      s += expf(v - m);
    }
  }
  lse = m + logf(s);
}

__device__ __forceinline__ int ce_label(const long long *labels, long long n, long long T, int C) {
  const long long y = labels[n / T];
  if (y < 0 || y >= C) {
    latch_error(5);
    return 0;
  }
  return (int)y;
}

__global__ void __launch_bounds__(kCeThreads) ce_forward_kernel(
    const float *__restrict__ logits, const long long *__restrict__ labels, long long N,
    long long T, int C, float eps, double *__restrict__ partials) {
  const long long n = (long long)blockIdx.x * kCeThreads + threadIdx.x;
  double loss = 0.0;
  if (n < N) {
    float lse, sum;
    ce_lse(logits, N, n, C, lse, sum);
    const int y = ce_label(labels, n, T, C);
    loss = (double)lse - (1.0 - (double)eps) * (double)logits[(long long)y * N + n] -
           ((double)eps / C) * (double)sum;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) loss += __shfl_xor_sync(0xffffffffu, loss, o);
  __shared__ double s_w[kCeThreads / 32];
  if ((threadIdx.x & 31) == 0) s_w[threadIdx.x >> 5] = loss;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < kCeThreads / 32; ++w) t += s_w[w];
    partials[blockIdx.x] = t;
  }
}

// loss = (sum of the block partials, in block order) / N; one warp.
__global__ void ce_finalize_kernel(const double *__restrict__ partials, long long blocks,
                                   long long N, float *__restrict__ loss) {
  double t = 0.0;
  for (long long b = threadIdx.x; b < blocks; b += 32) t += partials[b];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if (threadIdx.x == 0) *loss = (float)(t / (double)N);
}

// grad_logits (C, N) for the upstream gradient *grad_loss of the mean loss.
__global__ void __launch_bounds__(kCeThreads) ce_backward_kernel(
    const float *__restrict__ logits, const long long *__restrict__ labels,
    const float *__restrict__ grad_loss, long long N, long long T, int C, float eps,
    float *__restrict__ grad_logits) {
  const long long n = (long long)blockIdx.x * kCeThreads + threadIdx.x;
  if (n >= N) return;
  float lse, sum;
  ce_lse(logits, N, n, C, lse, sum);
  const int y = ce_label(labels, n, T, C);
  const float g = *grad_loss / (float)N, off = eps / (float)C;
  for (int c = 0; c < C; ++c) {
    const long long i = (long long)c * N + n;
    const float p = expf(logits[i] - lse);
    grad_logits[i] = (p - (c == y ? 1.f - eps : 0.f) - off) * g;
  }
}

}  // namespace readout
}  // namespace rqf
