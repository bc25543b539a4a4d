// The library's fixed device scratch: backing store of salt_conv_layer_forward_noalloc, the one
// entry point that allocates no device memory.  It sits in a translation unit of its own, with
// no kernels, so that it forms a module of its own: a process that never asks for its address
// does not load it under lazy module loading.
#include <mutex>

#include "salt_layers.cuh"

namespace salt {

static __device__ __align__(256) unsigned char g_fixed_scratch[SALT_NOALLOC_SCRATCH_BYTES];

// Device address of g_fixed_scratch on the current device.  The first call on a device looks
// the address up (cudaGetSymbolAddress, which loads the module); later calls read a cache.  A
// context reset (cudaDeviceReset) reloads the module, and the cached address is then stale.
cudaError_t fixed_scratch_address(void** ptr) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static void* cache[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fixed_scratch);
    if (e != cudaSuccess) return e;
    if (!p) return cudaErrorInvalidSymbol;
    cache[dev] = p;
  }
  *ptr = cache[dev];
  return cudaSuccess;
}

}  // namespace salt
