// Allocation-free variant of rqf_fbt_prospective_backward (declared in
// include/rqf_b200.h): the scratch buffer is a fixed file-scope __device__
// array instead of caller-provided memory.  Included by rqf_b200.cu after the
// regular entry points, which it calls unchanged.
#pragma once

#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB per device
constexpr int kNoAllocMaxDevices = 64;

// One instance per device that loads the library, held until process exit.
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void *g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once
// per device.  Host code must not pass the symbol itself to a kernel: on the
// host it only names a stand-in, not device memory.  The cached address stays
// valid for the life of the device's primary context; after cudaDeviceReset
// the module may be loaded again elsewhere, so this entry point does not
// support a process that resets a device it has already been called on.
int noalloc_scratch(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RQF_ERR_LAUNCH;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return RQF_ERR_CAPACITY;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return RQF_ERR_LAUNCH;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return RQF_OK;
}

}  // namespace

extern "C" int rqf_fbt_prospective_backward_noalloc(
    const float *c1, const float *tap0, const float *tap1, const float *z, const float *carries,
    const float *grad_out, float *grad_z, float *grad_c1, float *grad_tap0, float *grad_tap1,
    int64_t filters, int64_t batch, int64_t time, int fuse_act, rqf_stream_t stream) {
  const int dims = fbt_dims_ok(filters, batch, time);  // before any size product
  if (dims != RQF_OK) return dims;
  if (rqf_fbt_scratch_bytes(filters, batch, time) > kNoAllocScratchBytes) return RQF_ERR_CAPACITY;
  void *scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != RQF_OK) return st;
  return rqf_fbt_prospective_backward(c1, tap0, tap1, z, carries, grad_out, grad_z, grad_c1,
                                      grad_tap0, grad_tap1, scratch, filters, batch, time,
                                      fuse_act, stream);
}
