// Host-side dispatch of the queue-form conv kernel (conv_queue.cuh), split over two translation
// units so that they compile in parallel: this one holds the kernels that read 2x2 windows from the layer's address table.
#include "conv_queue.cuh"

namespace salt {

// Host-side dispatch over the (weight width, lanes per channel group, overflow mode, step form)
// instantiations; the no-fit form ignores the overflow mode.
// 16- and 32-lane groups run 512-thread blocks, narrower ones 256 (conv_queue_threads); a
// block size other than that one has no kernel.
template <typename WT, bool SAT, int FORM, bool WIN>
static void* queue_for_lpu(int lpu, int threads) {
  if (threads != conv_queue_threads(lpu)) return nullptr;
  switch (lpu) {
    case 1: return (void*)conv_queue<WT, 1, SAT, FORM, WIN, 256>;
    case 2: return (void*)conv_queue<WT, 2, SAT, FORM, WIN, 256>;
    case 4: return (void*)conv_queue<WT, 4, SAT, FORM, WIN, 256>;
    case 8: return (void*)conv_queue<WT, 8, SAT, FORM, WIN, 256>;
    case 16: return (void*)conv_queue<WT, 16, SAT, FORM, WIN, 512>;
    default: return (void*)conv_queue<WT, 32, SAT, FORM, WIN, 512>;
  }
}

template <bool SAT, int FORM, bool WIN>
static void* queue_for_wt(int wt_bytes, int lpu, int threads) {
  if (wt_bytes == 1) return queue_for_lpu<int8_t, SAT, FORM, WIN>(lpu, threads);
  if (wt_bytes == 2) return queue_for_lpu<int16_t, SAT, FORM, WIN>(lpu, threads);
  return queue_for_lpu<int32_t, SAT, FORM, WIN>(lpu, threads);
}

template <bool WIN>
static void* queue_kernel(int wt_bytes, int lpu, bool saturate, int form, int threads) {
  if (form == kStepWideNoFit)
    return queue_for_wt<false, kStepWideNoFit, WIN>(wt_bytes, lpu, threads);
  if (form != kStepWide) return nullptr;
  return saturate ? queue_for_wt<true, kStepWide, WIN>(wt_bytes, lpu, threads)
                  : queue_for_wt<false, kStepWide, WIN>(wt_bytes, lpu, threads);
}

// The address table of a layer with 2x2 windows: per input address (channel, y, x) its
// window's origin + 1 (bits 4-11 and 12-19), the slots valid in the output plane (bits 0-3)
// and the tap of slot (0, 0) (bits 20-31); the host checks that the fields fit.
__global__ void conv_addr_table(ConvLaunch P, uint32_t* __restrict__ table) {
  const int32_t a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= P.n_addr) return;
  int32_t c, y, x;
  const EvCand k = event_cand(P, a, c, y, x);
  const int32_t tap0 =
      c * P.k * P.k + (y + P.p - k.oy_min * P.s) * P.k + (x + P.p - k.ox_min * P.s);
  table[a] = window_bits(k) | ((uint32_t)(k.oy_min + 1) << 4) |
             ((uint32_t)(k.ox_min + 1) << 12) | ((uint32_t)tap0 << 20);
}

void* conv_queue_kernel_win(int wt_bytes, int lpu, bool saturate, int form, int threads) {
  return queue_kernel<true>(wt_bytes, lpu, saturate, form, threads);
}

}  // namespace salt
