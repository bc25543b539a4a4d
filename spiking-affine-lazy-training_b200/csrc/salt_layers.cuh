// Launch parameter blocks and block-level helpers shared by the layer kernels.
#pragma once
#include "../../include/salt_b200.h"
#include "salt_common.cuh"

namespace salt {

constexpr int kFusedThreads = 256;   // conv_fused block size (8 warps)
constexpr int kFusedChunk = 512;     // events bucketed per shared-memory chunk
constexpr int kPartChunk = 1024;     // events per tile-partition block
constexpr int kConvFillBlocks = 148 * 16;  // conv_fused blocks a launch should reach (tiling)
constexpr int kQueueFillBlocks = 2048;     // the same for conv_queue
constexpr int kQueueNoPartTiles = 4;       // conv_queue tiles per sample read without a partition
constexpr int kPartThreads = 256;    // tile-partition block size
constexpr int kPartPer = kPartChunk / kPartThreads;  // events per partition thread
constexpr int kCompactThreads = 256; // compaction block size == events per spike chunk
constexpr int kSpkChunkShift = 8;
constexpr int kSpkChunk = 1 << kSpkChunkShift;
static_assert(kSpkChunk == kCompactThreads, "one compaction block per spike chunk");
// Conv layers count spikes per group of 32 input events (one compaction warp per group).
constexpr int kConvGroupShift = 5;
constexpr int kConvGroup = 1 << kConvGroupShift;
constexpr int kLutSmemMax = 4096;    // decay tables longer than this are read from global
constexpr int kCompactBlocksPerSample = 8;  // compaction blocks per sample (grid-stride)
// conv_truncated: one block per truncated sample walks all its events several times, so it runs
// as wide as a block goes (each pass is latency-bound, 4x fewer rounds than 256 threads)
constexpr int kTruncThreads = 1024;
constexpr int kScanSmem = 33;        // ints of shared memory block_exclusive_scan needs

__host__ __device__ __forceinline__ size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

struct ConvLaunch {
  // geometry (salt_core/layers/conv.py:23-91)
  int32_t ic, h_in, w_in, hw_in, oc, k, s, p, h_out, w_out, n_sp;
  int64_t n_neurons;
  int32_t ncand, nslots;      // candidates per axis (k-1)//s+1 and per event (ncand^2)
  int32_t L, M, max_extra;    // max_queue_len, max_out_spikes, max_extra_steps
  int32_t lpu, G, ocp;        // lanes per channel group, channel groups, padded channel stride
  // host-built divisors: h_in*w_in, w_in, stride, channel groups, tile width
  FastDiv fd_hw, fd_w, fd_s, fd_G, fd_tw, fd_th;
  // tiling of the output plane
  int32_t tile_h, tile_w, tiles_x, T;
  int32_t n_part_chunks;
  int64_t list_stride;        // per-sample stride of the tile event lists
  // input stream
  StreamView in;
  const int32_t* in_nreal;
  int32_t batch;
  // parameters
  const int32_t* q;
  const int32_t* lut;
  int32_t lut_in_smem;
  const int32_t* vth;
  int32_t has_vth;
  QuantCfg qc;
  // outputs
  int32_t* v_final;
  // scratch (workspace)
  uint32_t* sw;               // spike words [B][E][nslots][G]
  int64_t sw_stride;
  int32_t* chunk_spikes;      // [B][n_spk_chunks]; scanned in place into offsets
  const int32_t* chunk_off;
  int32_t n_spk_chunks;
  int32_t *s_total, *oc_total, *needed, *vmin, *vmax, *ovf, *tail_total;
  int32_t tail_mode;
  int32_t* tail_cnt;          // [B][n_neurons] (tail mode only)
  const int32_t* order;       // [B] samples heaviest first (block y -> sample), or null
  const int32_t* tile_len;    // [B][T] events per tile
  const int32_t* tile_off;    // [B][T] start of each tile's list in the sample's region
  const int32_t* tile_lists;  // [B][list_stride] event indices, tile-major, arrival order
  // queue form (conv_queue): per (sample, tile) the kept candidates of every position, position
  // by position in arrival order, as (event time bits, weight row << q_shift | spike-word index)
  int2* queues;               // [B][queue_stride]
  int64_t queue_stride;
  int32_t q_shift;            // bits of the spike-word index in a queue entry
  const uint32_t* addr_table; // 2x2-window layers: per input address its window (conv_addr_table)
  int32_t n_addr;             // input addresses ic * h_in * w_in
  int32_t q_threads;          // conv_queue block size = events per chunk
  FastDiv fd_sww;             // spike words per event (nslots * G)
  int32_t grp_in_smem;        // per-group spike counts gathered in shared memory

  __device__ __forceinline__ int32_t n_eff(int b) const {
    int32_t n = in_nreal[b];
    return n < 0 ? 0 : (n < in.capacity ? n : in.capacity);
  }

  // Flat source index -> (clamped channel, y, x) with JAX's floor division / modulo
  // (connectivity/conv.py:32-43) and the channel gather clamp of q[oc][c] (conv.py:175-178).
  __device__ __forceinline__ void decode(int32_t src, int32_t& c, int32_t& y, int32_t& x) const {
    int32_t rem;
    if (src >= 0) {
      c = (int32_t)fd_hw.div((uint32_t)src);
      rem = src - c * hw_in;
    } else {
      c = floordiv(src, hw_in);
      rem = floormod(src, hw_in);
    }
    y = (int32_t)fd_w.div((uint32_t)rem);
    x = rem - y * w_in;
    c = (int32_t)jax_index(c, ic);
  }
  // Receptive-field candidates of coordinate i along one axis (conv.py:15-29): the first
  // candidate o_min = ceil((i+p-k+1)/s) and the valid range [lo, hi].
  __device__ __forceinline__ void axis(int32_t i, int32_t O, int32_t& o_min, int32_t& lo,
                                       int32_t& hi) const {
    // i + p - k + s >= 1 - k, so adding k*s keeps the dividend non-negative
    o_min = (int32_t)fd_s.div((uint32_t)(i + p - k + s + k * s)) - k;
    const int32_t upper = (int32_t)fd_s.div((uint32_t)(i + p));
    lo = max(o_min, 0);
    hi = min(min(upper, o_min + ncand - 1), O - 1);
  }
};

// Valid candidate ranges of one event (both axes).
struct EvCand {
  int32_t oy_min, oy_lo, oy_hi, ox_min, ox_lo, ox_hi;
  __device__ __forceinline__ bool empty() const { return oy_lo > oy_hi || ox_lo > ox_hi; }
};

__device__ __forceinline__ EvCand event_cand(const ConvLaunch& P, int32_t src, int32_t& c,
                                             int32_t& y, int32_t& x) {
  EvCand r;
  P.decode(src, c, y, x);
  P.axis(y, P.h_out, r.oy_min, r.oy_lo, r.oy_hi);
  P.axis(x, P.w_out, r.ox_min, r.ox_lo, r.ox_hi);
  return r;
}

struct FCLaunch {
  int32_t n_in, n_out, G;
  int32_t M, max_extra;
  StreamView in;
  const int32_t* in_nreal;
  int32_t batch;
  const int32_t* order;       // [B] samples heaviest first (unit -> sample), or null
  const int32_t* qT;          // (n_in, n_out) int32, transposed weight codes
  const int32_t* lut;
  const int32_t* vth;
  int32_t has_vth;
  QuantCfg qc;
  int32_t* v_final;
  uint32_t* sw;               // spike words [B][E][G] (firing layers only)
  int64_t sw_stride;
  int32_t* chunk_spikes;
  const int32_t* chunk_off;
  int32_t n_spk_chunks;
  int32_t *s_total, *vmin, *vmax, *ovf;
  int32_t* n_spk;             // [B][n_out] spikes per neuron
  int32_t tail_mode;          // process pad columns too (some v_th_int <= 0)

  __device__ __forceinline__ int32_t n_eff(int b) const {
    int32_t n = in_nreal[b];
    return n < 0 ? 0 : (n < in.capacity ? n : in.capacity);
  }
};

// Float FC layer (float chunked affine scan).  Per-(sample, segment, neuron) records of the
// speculative pass are laid out [b][s][neuron] so that a warp's 32 lanes touch 128 B.
constexpr int kFloatLut = 32;  // decay table rows: powf(base, d) for whole d in [0, 32)
constexpr int kFloatSegBlocksPerSM = 16;  // one-warp blocks resident per SM (128 registers)
constexpr int kFloatWarmMax = 16384;  // longest warm-up run before a segment

struct FloatLaunch {
  int32_t n_in, n_out, G, S;  // S time segments per sample
  int32_t C;                  // chunk_size
  int32_t max_steps;          // ceil(L / C) + max_extra_steps
  int32_t base_steps;         // ceil(L / C)
  float vth, margin;
  StreamView in;
  const int32_t* in_nreal;
  int32_t batch;
  const float* gain;          // (B, L) event gains or nullptr (all ones)
  const float* w;             // (n_out, n_in) as the caller holds it
  float* wT;                  // (n_in, n_out) transposed copy
  const float* decay_base;    // (n_out) float32(1 - 1/tau_i)
  float* lut;                 // [kFloatLut][n_out]
  float* v_final;             // (B, n_out)
  uint32_t* sw;               // spike words [B][L][G]
  int64_t sw_stride;
  int32_t* chunk_spikes;      // [B][n_spk_chunks]
  int32_t n_spk_chunks;
  int32_t *s_total, *needed;  // (B)
  int32_t* n_spk;             // (B, n_out)
  int32_t* exact;             // (B, G) groups that the step limit may cut
  int32_t* hist;              // (B, n_in) real events per source (gain == nullptr only)
  double* bsum;               // (B, n_out) Σ of positive b (gain == nullptr only)
  int32_t* bcnt;              // (B, n_out) count of positive b (gain == nullptr only)
  int32_t warm_max;           // longest warm-up run before a segment
  float *r_vstart, *r_vend, *r_u1, *r_A1, *r_M, *r_Aseg, *r_sum;
  int32_t *r_k1, *r_nspk, *r_cnt, *r_mono;

  __device__ __forceinline__ int32_t n_eff(int b) const {
    int32_t n = in_nreal[b];
    return n < 0 ? 0 : (n < in.capacity ? n : in.capacity);
  }
  // events per segment: a multiple of 32 so that 32-event batches never straddle segments or
  // 256-event spike chunks
  __device__ __forceinline__ int32_t seg_len(int32_t n_eff) const {
    const int32_t l = (n_eff + S - 1) / S;
    return max(32, (l + 31) & ~31);
  }
};

// ---------------------------------------------------------------- warp / block helpers
__device__ __forceinline__ int32_t warp_sum(int32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int32_t warp_min(int32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int32_t warp_max(int32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int32_t warp_or(int32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v |= __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide exclusive scan; every thread of the block must call it.  `s` must hold 33 ints
// (kScanSmem).  Returns the exclusive prefix and writes the block total to `total`.
__device__ __forceinline__ int32_t block_exclusive_scan(int32_t v, int32_t* s, int32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  __syncthreads();
  if (lane == 31) s[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int32_t x = lane < nw ? s[lane] : 0, xi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int32_t n = __shfl_up_sync(0xffffffffu, xi, o);
      if (lane >= o) xi += n;
    }
    if (lane < nw) s[lane] = xi - x;
    if (lane == nw - 1) s[32] = xi;
  }
  __syncthreads();
  total = s[32];
  const int32_t r = s[warp] + incl - v;
  __syncthreads();
  return r;
}

// Kernel declarations (definitions in conv_layer.cu / fc_layer.cu).
__global__ void conv_tile_count(ConvLaunch P, int32_t* counts);
__global__ void conv_tile_scan_offsets(ConvLaunch P, int32_t* counts, int32_t* tile_len,
                                       int32_t* tile_off);
__global__ void conv_tile_scatter(ConvLaunch P, const int32_t* counts, int32_t* lists);
// order[0..B) = samples by decreasing min(n_real, capacity) (counting sort, one block).
__global__ void sample_order_desc(const int32_t* __restrict__ n_real, int32_t capacity,
                                  int32_t batch, int32_t* __restrict__ order);
constexpr int kOrderThreads = 1024;
constexpr int kOrderMinBatch = 128;  // below this the sort costs more than the schedule gains
// conv_compact specialised for the geometry (ncand <= 2 and one channel group, or the rest).
// table: the layer's address table is filled (conv_addr_table) and L.addr_table points at it.
void* conv_compact_kernel(int ncand, int G, bool table);
__global__ void conv_tail_append(ConvLaunch P, salt_stream_out out);
__global__ void conv_truncated(ConvLaunch P, salt_stream_out out, int32_t* scratch_hist);
__global__ void fc_compact(FCLaunch P, salt_stream_out out);
__global__ void fc_truncated(FCLaunch P, salt_stream_out out);
// Kernel entry points of the templated kernels, for cudaLaunchKernel.  form: kStepSplit,
// kStepWide or kStepWideNoFit (salt_common.cuh), as step_form chooses it for the layer.
void* conv_fused_kernel(int wt_bytes, int lpu, bool saturate, int form);
// Dynamic shared memory of conv_tile_scatter: per tile a mask and a word prefix per
// 1024-event chunk, plus the chunk's list base.
inline size_t conv_scatter_smem(int T) {
  return (size_t)T * (2 * (kPartChunk / 32) * sizeof(uint32_t) + sizeof(int32_t));
}
// Dynamic shared memory conv_fused needs for a launch configuration (same layout as the kernel).
size_t conv_fused_smem_bytes(const ConvLaunch& P, int wt_bytes);
// The queue form of the fused kernel (conv_queue.cu), for layers without needs_tail: form
// kStepWide or kStepWideNoFit (null otherwise); its dynamic shared memory.
// win: the variant that reads 2x2 windows from the layer's address table (conv_addr_table).
// threads: the block size, conv_queue_threads(lpu): 512 for 16- and 32-lane groups, else 256.
void* conv_queue_kernel(int wt_bytes, int lpu, bool saturate, int form, bool win, int threads);
void* conv_queue_kernel_win(int wt_bytes, int lpu, bool saturate, int form, int threads);
int conv_queue_threads(int lpu);
// Fills the address table of a layer with 2x2 windows (one thread per input address).
__global__ void conv_addr_table(ConvLaunch P, uint32_t* table);
size_t conv_queue_smem_bytes(const ConvLaunch& P, int wt_bytes);
// lpu: lanes per (sample, neuron group) unit, 8 / 16 for layers of at most that many neurons;
// wt: bytes per weight code staged in shared memory (1, 2, 4), 0 to read them from global.
void* fc_scan_kernel(bool fires, bool saturate, int lpu, int wt, int form);
// Dynamic shared memory of fc_scan for these sizes.
size_t fc_scan_smem(int32_t n_in, int32_t n_out, int32_t lut_len, int wt, int lpu);
// Bytes of the weight table fc_scan stages in shared memory (0 when wt == 0).
size_t fc_scan_q_bytes(int32_t n_in, int32_t n_out, int wt, int lpu);

// Device address of the fixed scratch behind salt_conv_layer_forward_noalloc (fixed_scratch.cu).
cudaError_t fixed_scratch_address(void** ptr);

// Real-event rows of pinned host streams into device streams (stream_io.cu).
constexpr int kGatherBlocks = 16, kGatherThreads = 256;
cudaError_t gather_rows_launch(const float* ht, const int32_t* hs, const int32_t* n_real_dev,
                               int32_t batch, int32_t capacity, int64_t host_pitch, float* dt,
                               int32_t* ds, cudaStream_t st);

// Per-column traces of the integer scan (trace.cu).
cudaError_t conv_trace_launch(const ConvLaunch& P, const salt_neuron_trace* rec, int32_t* v_steps,
                              uint8_t* spike_mask, float* event_ms, cudaStream_t st);
cudaError_t fc_trace_launch(const FCLaunch& P, const salt_neuron_trace* rec, int32_t* v_steps,
                            uint8_t* spike_mask, float* event_ms, cudaStream_t st);

// Enqueues the float FC layer's kernels up to the final spike words (float_scan.cu); adds the
// number of launches to *launches.  When given, seg_start/seg_stop are recorded around the
// speculative segment kernel.
cudaError_t float_fc_launch(const FloatLaunch& P, cudaStream_t st, int64_t* launches,
                            cudaEvent_t seg_start = nullptr, cudaEvent_t seg_stop = nullptr);
// Float conv layer (float_conv.cu): per-warp arguments beyond the shared ConvLaunch geometry,
// stream and spike-word scratch.
constexpr int kFConvThreads = 128;
struct FConvArgs {
  const float* wT;            // (ic*k*k, ocp) weights, channels zero-padded
  const float* gain;          // (B, E) event gains or null (ones)
  float base, v_th;           // float32(1 - 1/tau), ConvLayer.v_th
  int32_t C, max_steps, base_steps;
  float* v_final;             // (B, n_neurons)
  int32_t* needed_extra;      // (B)
  int32_t *vkey_max, *vkey_min;  // (B, oc) order-preserving keys of the potential extremes
  float* v_steps;             // (B, n_neurons, max_steps) traces, or null
  float* event_ms;
  uint8_t* spike_mask;
};
cudaError_t float_conv_launch(const ConvLaunch& P, const FConvArgs& X, const float* w, float* wT,
                              int32_t* out_nreal, const salt_float_conv_stats* st, float* v_max,
                              float* v_min, cudaStream_t stream);

// Float FC per-step traces and potential ranges (float_conv.cu).
struct FTraceArgs {
  int32_t n_in, n_out, C, max_steps, batch;
  float v_th;
  StreamView in;
  const int32_t* in_nreal;
  const float* w;             // (n_out, n_in)
  const float* decay_base;    // (n_out)
  const float* gain;          // (B, E) or null
  float* v_final;             // (B, n_out) or null
  float *v_max, *v_min;       // (B, n_out) or null
  float* v_steps;             // (B, n_out, max_steps) or null
  float* event_ms;
  uint8_t* spike_mask;
};
cudaError_t float_fc_trace_launch(const FTraceArgs& T, cudaStream_t stream);

constexpr int kFcThreads = 128;
constexpr int kFcRing = 4;            // events per lane per fc_scan super-batch (smem codes)
constexpr int kFcStepBlock = 8;       // fc_scan steps whose loads are issued together
constexpr int kStageLoads = 8;        // weight-table staging: global loads in flight per thread
constexpr int kConvStageLoads = 4;    // the same for conv_fused (held to its register budget)
constexpr size_t kFcQSmemMax = 96 * 1024;  // largest staged weight table of fc_scan

}  // namespace salt
