// Deterministic reduction of per-(row, tile) partial sums into per-channel
// coefficient gradients.  The reference accumulates these with fp32
// tl.atomic_add in nondeterministic order (chunked_scan_kernel.py:206-209,
// fbt_scan_kernel.py:237-242, :567-572); here every tile writes its partial
// and one CTA per channel sums them in fixed order in double precision.
#pragma once

#include "rqf_common.cuh"

namespace rqf {

// partials: (rows, ntiles, 3) float2.  Row of (channel f, i-th member) is
// f*stride_f + i*stride_i, i < members.  Outputs (may be null): complex (F,).
__global__ void __launch_bounds__(256)
    reduce_partials_kernel(const float2 *__restrict__ partials, float2 *__restrict__ o0,
                           float2 *__restrict__ o1, float2 *__restrict__ o2, int64_t members,
                           int64_t stride_f, int64_t stride_i, int ntiles) {
  __shared__ double s[6][8];
  const int64_t f = blockIdx.x;
  double acc[6] = {0, 0, 0, 0, 0, 0};
  const int64_t n = members * ntiles;
  for (int64_t idx = threadIdx.x; idx < n; idx += blockDim.x) {
    const int64_t i = idx / ntiles;
    const int64_t jj = idx - i * ntiles;
    const int64_t row = f * stride_f + i * stride_i;
    const float2 *p = partials + (row * ntiles + jj) * 3;
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const float2 v = p[q];
      acc[2 * q] += (double)v.x;
      acc[2 * q + 1] += (double)v.y;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int q = 0; q < 6; ++q) {
    double v = acc[q];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) s[q][warp] = v;
  }
  __syncthreads();
  if (threadIdx.x < 6) {
    double v = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += s[threadIdx.x][w];
    float2 *dst = threadIdx.x < 2 ? o0 : (threadIdx.x < 4 ? o1 : o2);
    if (dst) reinterpret_cast<float *>(dst + f)[threadIdx.x & 1] = (float)v;
  }
}

}  // namespace rqf
