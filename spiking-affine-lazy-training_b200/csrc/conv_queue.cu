// Host-side dispatch of the queue-form conv kernel (conv_queue.cuh), split over two translation
// units so that they compile in parallel: this one holds the kernels that decode every source index.
#include "conv_queue.cuh"

namespace salt {

// Host-side dispatch over the (weight width, lanes per channel group, overflow mode, step form)
// instantiations; the no-fit form ignores the overflow mode.
template <typename WT, bool SAT, int FORM, bool WIN>
static void* queue_for_lpu(int lpu) {
  switch (lpu) {
    case 1: return (void*)conv_queue<WT, 1, SAT, FORM, WIN>;
    case 2: return (void*)conv_queue<WT, 2, SAT, FORM, WIN>;
    case 4: return (void*)conv_queue<WT, 4, SAT, FORM, WIN>;
    case 8: return (void*)conv_queue<WT, 8, SAT, FORM, WIN>;
    case 16: return (void*)conv_queue<WT, 16, SAT, FORM, WIN>;
    default: return (void*)conv_queue<WT, 32, SAT, FORM, WIN>;
  }
}

template <bool SAT, int FORM, bool WIN>
static void* queue_for_wt(int wt_bytes, int lpu) {
  if (wt_bytes == 1) return queue_for_lpu<int8_t, SAT, FORM, WIN>(lpu);
  if (wt_bytes == 2) return queue_for_lpu<int16_t, SAT, FORM, WIN>(lpu);
  return queue_for_lpu<int32_t, SAT, FORM, WIN>(lpu);
}

template <bool WIN>
static void* queue_kernel(int wt_bytes, int lpu, bool saturate, int form) {
  if (form == kStepWideNoFit) return queue_for_wt<false, kStepWideNoFit, WIN>(wt_bytes, lpu);
  if (form != kStepWide) return nullptr;
  return saturate ? queue_for_wt<true, kStepWide, WIN>(wt_bytes, lpu)
                  : queue_for_wt<false, kStepWide, WIN>(wt_bytes, lpu);
}

size_t conv_queue_smem_bytes(const ConvLaunch& P, int wt_bytes) {
  return QueueSmem(P, wt_bytes).total;
}

void* conv_queue_kernel(int wt_bytes, int lpu, bool saturate, int form, bool win) {
  return win ? conv_queue_kernel_win(wt_bytes, lpu, saturate, form)
             : queue_kernel<false>(wt_bytes, lpu, saturate, form);
}

}  // namespace salt
