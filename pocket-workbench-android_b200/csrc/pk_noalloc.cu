// pk_noalloc.cu -- the fixed device scratch behind pk_matmul_noalloc.
//
// The array lives in the library's own device image (uninitialised, so it
// costs no file size); the driver reserves it when the module is loaded on
// a device.  Its address differs per device and is looked up once per
// device, with that device current, through cudaGetSymbolAddress.
#include <cuda_runtime.h>

#include <mutex>

#include "pk.h"

namespace pk {

static __device__ __align__(256) unsigned char g_noalloc_scratch[PK_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_addr[kMaxDevices] = {};
}  // namespace

// Device address of the scratch on the current device (set up on first use).
cudaError_t noalloc_scratch(void **ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_addr[dev] = p;
  }
  *ptr = g_addr[dev];
  return cudaSuccess;
}

}  // namespace pk
