// Host-side dispatch of the queue-form conv kernel (conv_queue.cuh), split over two translation
// units so that they compile in parallel: this one holds the kernels that decode every source index.
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

size_t conv_queue_smem_bytes(const ConvLaunch& P, int wt_bytes) {
  return QueueSmem(P, wt_bytes, P.q_threads).total;
}

void* conv_queue_kernel(int wt_bytes, int lpu, bool saturate, int form, bool win, int threads) {
  return win ? conv_queue_kernel_win(wt_bytes, lpu, saturate, form, threads)
             : queue_kernel<false>(wt_bytes, lpu, saturate, form, threads);
}

int conv_queue_threads(int lpu) { return (lpu == 16 || lpu == 32) ? 512 : 256; }

}  // namespace salt
