// Host-to-device transfer of event streams that moves only the real events.
//
// A batch of streams is (B, capacity) row-major, but a sample's events past min(n_real,
// capacity) are pads that no layer reads when the first layer cannot fire on pads (v_th_int > 0,
// decay codes in range): conv layers gather only real events (connectivity/conv.py:145-172; the
// catch-up column of a position without events has Δt = 0 whatever the pad times), FC layers mask
// pads to identity steps (connectivity/fc.py:26-29).  With event counts spread over 10x
// (log-uniform), the real events are a fraction of the rows, so this kernel reads each row of a
// pinned (page-locked, device-mapped) host buffer only up to its n_real, over the host link, into
// the device buffer; the pads of the device rows keep whatever they held.
#include "salt_layers.cuh"

namespace salt {

// A few persistent blocks loop over the rows (16-byte loads where both rows allow them).  The
// host reads in flight slow a layer running beside the gather, in proportion to their number
// (measured against configuration 3's forward, 5.63 ms alone: 32 x 512 threads 7.68 ms per
// overlapped step, 148 x 128 8.42, 32 x 128 6.23, 16 x 256 5.98, the gather alone 5.1-5.8 ms),
// so the kernel keeps just enough of them to stay near the host link's rate.
__global__ void __launch_bounds__(kGatherThreads)
gather_rows_kernel(const float* __restrict__ ht, const int32_t* __restrict__ hs,
                   const int32_t* __restrict__ n_real, int32_t batch, int32_t capacity,
                   int64_t host_pitch, float* __restrict__ dt, int32_t* __restrict__ ds) {
  const bool vec = (host_pitch % 4 == 0) && (capacity % 4 == 0);
  for (int32_t b = blockIdx.x; b < batch; b += gridDim.x) {
    const int32_t nr = n_real[b];
    const int32_t n = nr < 0 ? 0 : (nr < capacity ? nr : capacity);
    const float* trow = ht + (int64_t)b * host_pitch;
    const int32_t* srow = hs + (int64_t)b * host_pitch;
    float* drow_t = dt + (int64_t)b * capacity;
    int32_t* drow_s = ds + (int64_t)b * capacity;
    int32_t done = 0;
    if (vec) {
      const int32_t n4 = n >> 2;
      for (int32_t i = threadIdx.x; i < n4; i += blockDim.x) {
        reinterpret_cast<float4*>(drow_t)[i] = reinterpret_cast<const float4*>(trow)[i];
        reinterpret_cast<int4*>(drow_s)[i] = reinterpret_cast<const int4*>(srow)[i];
      }
      done = n4 << 2;
    }
    for (int32_t i = done + threadIdx.x; i < n; i += blockDim.x) {
      drow_t[i] = trow[i];
      drow_s[i] = srow[i];
    }
  }
}

cudaError_t gather_rows_launch(const float* ht, const int32_t* hs, const int32_t* n_real_dev,
                               int32_t batch, int32_t capacity, int64_t host_pitch, float* dt,
                               int32_t* ds, cudaStream_t st) {
  const int blocks = std::max(1, std::min(batch, kGatherBlocks));
  gather_rows_kernel<<<blocks, kGatherThreads, 0, st>>>(ht, hs, n_real_dev, batch, capacity,
                                                       host_pitch, dt, ds);
  return cudaGetLastError();
}

}  // namespace salt
