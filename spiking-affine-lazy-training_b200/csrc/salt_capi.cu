// Host side of libsalt_b200: argument checks, launch planning, workspace layout, the C ABI of
// include/salt_b200.h and the native network plan.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "salt_layers.cuh"

namespace salt {


static thread_local std::string g_err;
static thread_local int64_t g_launches = 0;

static salt_status fail(salt_status s, const std::string& msg) {
  g_err = msg;
  return s;
}

#define SALT_CUDA(call)                                                                \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return fail(SALT_CUDA_ERROR, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

#define SALT_LAUNCHED(name)                                                             \
  do {                                                                                  \
    ++g_launches;                                                                       \
    cudaError_t e_ = cudaGetLastError();                                                \
    if (e_ != cudaSuccess)                                                              \
      return fail(SALT_CUDA_ERROR, std::string("launch ") + name + ": " + cudaGetErrorString(e_)); \
  } while (0)

static inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Compaction blocks per sample: the per-sample minimum, or enough to fill the GPU when the
// batch is small.
// Blocks per sample for conv_compact (8 warps each, one 32-event group per warp at a time):
// about 16 K warps over the batch, no more than the groups need.
static int conv_compact_blocks(int32_t n_groups, int32_t B) {
  const int want = (2048 + B - 1) / std::max(B, 1);
  return std::max(1, std::min((n_groups + 7) / 8, std::max(2, want)));
}

static int compact_blocks(int32_t B) {
  return std::max(kCompactBlocksPerSample, (1184 + B - 1) / std::max(B, 1));
}

// Sequential carving of a workspace; with base == nullptr it only measures.
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t n) {
    off = align256(off);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
  size_t size() const { return align256(off); }
};

// ---------------------------------------------------------------- small kernels

// One warp per sample: exclusive scan in place of the spike counts per event chunk; with
// total_add, the sample's total is also added to total_add[sample].
__global__ void spike_chunk_scan(int32_t* __restrict__ chunk, int32_t n_chunks, int32_t batch,
                                 int32_t* __restrict__ total_add) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= batch) return;
  int32_t* c = chunk + (int64_t)warp * n_chunks;
  int32_t carry = 0;
  for (int base = 0; base < n_chunks; base += 32) {
    const int i = base + lane;
    const int32_t v = i < n_chunks ? c[i] : 0;
    int32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (i < n_chunks) c[i] = carry + incl - v;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (total_add && lane == 0 && carry) total_add[warp] += carry;
}

struct FinishArgs {
  const int32_t *s_total, *needed, *vmin, *vmax, *ovf;
  int32_t L, M, max_extra, is_conv, batch;
  int32_t half;  // 2^(i_V + f_V - 1): the register range is [-half, half)
};

// Per-sample diagnostics and Capacity.fits (salt_core/capacity.py:60-63; layers/conv.py:137-141,
// layers/fc.py:92-94).
__global__ void layer_finish(FinishArgs A, int32_t* out_nreal, salt_layer_stats st) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= A.batch) return;
  const int32_t S = A.s_total[b];
  const int32_t nq = A.is_conv ? A.needed[b] : 0;
  if (out_nreal) out_nreal[b] = S;
  if (st.spike_count) st.spike_count[b] = S;
  if (st.needed_queue) st.needed_queue[b] = nq;
  // the hot scans track only the unfitted range; an update overflowed iff it left the register
  // range, so the sample overflowed iff its unfitted range did
  if (st.overflowed)
    st.overflowed[b] = A.ovf[b] != 0 || A.vmin[b] < -A.half || A.vmax[b] >= A.half;
  if (st.vmin) st.vmin[b] = A.vmin[b];
  if (st.vmax) st.vmax[b] = A.vmax[b];
  if (st.fits)
    st.fits[b] = (A.is_conv ? nq <= A.L : 1) && S <= A.M && 0 <= A.max_extra;
}

__global__ void transpose_i32(const int32_t* __restrict__ q, int32_t* __restrict__ qT, int rows,
                              int cols) {  // qT[c][r] = q[r][c]
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)rows * cols) return;
  const int r = (int)(i / cols), c = (int)(i % cols);
  qT[(int64_t)c * rows + r] = q[i];
}

// fits of layer l for sample b lives at per_layer[l * layer_stride + b].
__global__ void fits_and(const int32_t* __restrict__ per_layer, int n_layers, int64_t layer_stride,
                         int batch, int32_t* __restrict__ fits) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  int32_t f = 1;
  for (int l = 0; l < n_layers; ++l) f &= per_layer[(int64_t)l * layer_stride + b] != 0;
  fits[b] = f;
}

// quant/scan.py:97-132 on materialised (n, L) inputs: one thread per neuron, every column.
// v_steps (optional): the register after each column (run_layer_traced, quant/scan.py:83-94).
__global__ void dense_scan(QuantCfg qc, int32_t n, int32_t L, const int32_t* __restrict__ a_int,
                           const uint8_t* __restrict__ is_id, const int32_t* __restrict__ q_int,
                           const int32_t* __restrict__ vth, uint8_t* __restrict__ mask,
                           uint8_t* __restrict__ ovf_out, int32_t* __restrict__ v_final,
                           int32_t* __restrict__ vmin, int32_t* __restrict__ vmax,
                           int32_t* __restrict__ v_steps) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int32_t v = 0, lo = 0, hi = 0;
  const int32_t th = vth ? vth[i] : 0;
  for (int32_t t = 0; t < L; ++t) {
    const int64_t e = i * L + t;
    int32_t u;
    bool ovf;
    const int32_t w = quant_step(v, a_int[e], is_id[e] != 0, q_int[e], qc, u, ovf);
    const bool spike = vth != nullptr && w >= th;
    v = spike ? 0 : w;
    lo = min(lo, u);
    hi = max(hi, u);
    if (mask) mask[e] = spike;
    if (ovf_out) ovf_out[e] = ovf;
    if (v_steps) v_steps[e] = v;
  }
  v_final[i] = v;
  vmin[i] = lo;
  vmax[i] = hi;
}

// ---------------------------------------------------------------- checks

static salt_status check_quant(const salt_quant_desc* q) {
  if (!q) return fail(SALT_BAD_ARG, "quant descriptor is NULL");
  if (q->f_a < 0 || q->f_a > 15)
    return fail(SALT_BAD_ARG, "f_a must be in [0, 15] (fixed_point.MAX_SHIFT_BITS)");
  if (q->f_V < 0 || q->i_V < 1 || q->i_V + q->f_V > 30)
    return fail(SALT_BAD_ARG, "need f_V >= 0, i_V >= 1, i_V + f_V <= 30 (MAX_REGISTER_BITS)");
  if (q->round_mode != SALT_ROUND && q->round_mode != SALT_TRUNCATE)
    return fail(SALT_BAD_ARG, "round_mode must be SALT_ROUND or SALT_TRUNCATE");
  if (q->overflow_mode != SALT_WRAP && q->overflow_mode != SALT_SATURATE)
    return fail(SALT_BAD_ARG, "overflow_mode must be SALT_WRAP or SALT_SATURATE");
  if (q->lut_len < 0) return fail(SALT_BAD_ARG, "lut_len must be >= 0");
  return SALT_OK;
}

static QuantCfg make_qc(const salt_quant_desc* q) {
  QuantCfg c;
  c.f_a = q->f_a;
  c.f_V = q->f_V;
  c.total_bits = q->i_V + q->f_V;
  c.round_half = (q->round_mode == SALT_ROUND && q->f_a > 0) ? (1 << (q->f_a - 1)) : 0;
  c.saturate = q->overflow_mode == SALT_SATURATE;
  c.lut_len = q->lut_len;
  return c;
}

static salt_status check_stream_in(const salt_stream_in* in, int32_t batch) {
  if (!in || !in->times || !in->src || !in->n_real)
    return fail(SALT_BAD_ARG, "input stream pointers must be non-NULL");
  if (in->capacity < 1) return fail(SALT_BAD_ARG, "input stream capacity must be >= 1");
  if (batch < 1 || batch > 65535) return fail(SALT_BAD_ARG, "batch must be in [1, 65535]");
  return SALT_OK;
}

// ---------------------------------------------------------------- conv planning

struct ConvPlan {
  int32_t h_out, w_out, n_sp, ncand, nslots, lpu, G, ocp, wt_bytes;
  int64_t n_neurons;
  int32_t tile_h, tile_w, tiles_x, tiles_y, T, n_part_chunks, n_spk_chunks, tail_mode;
  int64_t list_stride;
  size_t smem;
  // queue form (conv_queue): whole-sample position queues instead of per-chunk walks
  bool queue;
  bool win;                   // 2x2 windows read from an address table (conv_addr_table)
  bool part;                  // tiles get event lists from the partition kernels
  int32_t q_threads;          // conv_queue block size
  int32_t grp_in_smem;
  int64_t queue_stride;       // queue entries per sample
};

// A launch block carrying only what the shared-memory layout depends on.
static size_t fused_smem(const salt_conv_desc* d, const salt_quant_desc* q, const ConvPlan& p,
                         int tile_h, int tile_w, int T) {
  ConvLaunch L;
  memset(&L, 0, sizeof(L));
  L.ic = d->ic;
  L.k = d->k;
  L.ocp = p.ocp;
  L.lpu = p.lpu;
  L.G = p.G;
  L.nslots = p.nslots;
  L.tile_h = tile_h;
  L.tile_w = tile_w;
  L.T = T;
  L.lut_in_smem = q->lut_len <= kLutSmemMax;
  L.qc.lut_len = q->lut_len;
  L.n_spk_chunks = p.n_spk_chunks;
  L.grp_in_smem = p.grp_in_smem;
  L.q_threads = p.q_threads;
  return p.queue ? conv_queue_smem_bytes(L, p.wt_bytes) : conv_fused_smem_bytes(L, p.wt_bytes);
}

// Bits of a conv_queue entry's spike-word index: enough for every (event, slot, group) word of a
// sample.
static int queue_shift(int64_t words_per_sample) {
  int b = 1;
  while ((int64_t(1) << b) < words_per_sample) ++b;
  return b;
}

// The queue form serves layers whose catch-up/identity columns cannot fire (no needs_tail) and
// whose queue entries can pack a tap's weight row beside the spike-word index in 32 bits.
// SALT_CONV_FORM=chunked in the environment selects conv_fused for every layer (a comparison
// switch; both forms give identical results).
static bool queue_form(const salt_conv_desc* d, const salt_quant_desc* q, int ocp, int nslots,
                       int G, int32_t E) {
  static const bool chunked = [] {
    const char* v = getenv("SALT_CONV_FORM");
    return v && strcmp(v, "chunked") == 0;
  }();
  if (chunked || q->needs_tail) return false;
  const int shift = queue_shift((int64_t)E * nslots * G);
  const int64_t max_row = (int64_t)(d->ic * d->k * d->k - 1) * ocp;
  return shift < 32 && max_row < (int64_t(1) << (32 - shift));
}

// Step form of a layer's hot loop (salt_common.cuh).  Without needs_tail every decay code lies
// in [0, 2^f_a]: the one-multiply product is exact, and a decay never grows |v|, so a neuron that
// sees at most max_steps weighted steps with |q| <= 2^(q_bits - 1) stays inside its register
// range when max_steps < 2^(i_V - q_bits), and the fit can be left out.
static int step_form(const salt_quant_desc* q, int64_t max_steps) {
  if (q->needs_tail) return kStepSplit;
  const int headroom = q->i_V - q->q_bits;
  if (headroom > 0 && headroom < 62 && max_steps < (int64_t(1) << headroom)) return kStepWideNoFit;
  return kStepWide;
}

static salt_status plan_conv(const salt_conv_desc* d, const salt_quant_desc* q, int32_t batch,
                             int32_t E, ConvPlan& p) {
  if (!d) return fail(SALT_BAD_ARG, "conv descriptor is NULL");
  if (d->ic < 1 || d->h_in < 1 || d->w_in < 1 || d->oc < 1 || d->k < 1 || d->s < 1 || d->p < 0)
    return fail(SALT_BAD_ARG, "conv geometry: ic,h_in,w_in,oc,k,s must be >= 1 and p >= 0");
  if (d->h_in + d->p > 32000 || d->w_in + d->p > 32000)
    return fail(SALT_BAD_ARG, "conv input plane too large (h_in + p and w_in + p <= 32000)");
  p.h_out = (d->h_in + 2 * d->p - d->k) / d->s + 1;
  p.w_out = (d->w_in + 2 * d->p - d->k) / d->s + 1;
  if (d->h_in + 2 * d->p - d->k < 0 || p.h_out < 1 || p.w_out < 1)
    return fail(SALT_BAD_ARG, "conv geometry degenerates to an empty output plane");
  if (d->max_queue_len < 1) return fail(SALT_BAD_ARG, "max_queue_len must be >= 1");
  if (d->max_out_spikes < 1) return fail(SALT_BAD_ARG, "max_out_spikes must be >= 1");
  p.n_sp = p.h_out * p.w_out;
  p.n_neurons = (int64_t)d->oc * p.n_sp;
  if (p.n_neurons > 0x7fffffffLL) return fail(SALT_BAD_ARG, "too many neurons");
  p.ncand = (d->k - 1) / d->s + 1;
  p.nslots = p.ncand * p.ncand;
  if (p.ncand > 16) return fail(SALT_BAD_ARG, "k / s too large (at most 16 candidates per axis)");
  int lpu = 1;
  while (lpu < d->oc && lpu < 32) lpu <<= 1;
  p.lpu = lpu;
  p.G = (d->oc + lpu - 1) / lpu;
  p.ocp = p.G * lpu;
  p.wt_bytes = q->q_bits <= 8 ? 1 : (q->q_bits <= 16 ? 2 : 4);
  p.tail_mode = q->needs_tail ? 1 : 0;
  p.n_spk_chunks = (E + kConvGroup - 1) / kConvGroup;  // conv: per 32-event group
  p.queue = queue_form(d, q, p.ocp, p.nslots, p.G, E);
  // the address table packs the window origin + 1 into 8 bits per axis and the tap into 12
  p.win = p.queue && p.ncand == 2 && p.h_out <= 254 && p.w_out <= 254 &&
          d->ic * d->k * d->k <= 4096;
  p.grp_in_smem = (int64_t)p.n_spk_chunks * 4 <= 32 * 1024;
  p.q_threads = p.queue ? conv_queue_threads(p.lpu) : kFusedThreads;
  // Positions per block: at most 64 (fewer positions per block means more of each position's
  // events per 512-event chunk, so the per-position setup of the recurrence is shared by more
  // events, and more, smaller blocks), within a ~100 KB shared-memory budget, never fewer than
  // one candidate window.  Measured against 256: configuration 3 1.07x, 2 1.86x, 4 1.48x; 32
  // and 128 were slower on configuration 3 too.  A layer whose input capacity is below its
  // position count has few events per position whatever the tiling, and its blocks' fixed work
  // (weight staging, register init, catch-up) dominates: it takes tiles of up to 256 positions
  // (configuration 4's conv2, 36 events over 1024 positions: 0.50 -> 0.36 ms at 128).
  //
  // A small batch would leave SMs idle behind a few long blocks (one heavy sample's whole plane
  // in one block): while batch x tiles stays below kConvFillBlocks, the tiles shrink (to no
  // fewer than 8 positions), so each sample is spread over more blocks.  The workspace sizes
  // take the finest tiling into account (conv_scratch_bytes), so a plan made for a batch also
  // serves its row slices.
  //
  // The queue form has no per-chunk walk to amortise: its blocks take up to 256 positions (one
  // thread per position in its count and scan phases), and a whole plane needs no partition.
  // Its tiles shrink while batch x tiles stays below kQueueFillBlocks, and up to
  // kQueueNoPartTiles tiles each block reads the sample's whole stream and keeps its own
  // candidates instead of waiting for the partition kernels (configuration 3, G events/s:
  // 2048 samples 6.03 partitioned in two tiles, 6.93 in one block; 1024 samples 5.25 in four
  // partitioned tiles, 5.71 in two unpartitioned; 512 samples 4.23 and 4.25 in four).
  const size_t budget = 100 * 1024;
  int npm_cap = (p.queue || E < p.n_sp) ? 256 : 64;
  while (npm_cap > 1 && fused_smem(d, q, p, 1, npm_cap, 2) > budget) npm_cap >>= 1;
  auto tile_for = [&](int cap) {
    if (p.n_sp <= cap) {
      p.tile_h = p.h_out;
      p.tile_w = p.w_out;
    } else {
      // 16 positions wide (8 below a 32-position cap, 4 below 16), never narrower than one
      // candidate window
      p.tile_w = std::min(p.w_out, std::max(p.ncand, std::min(16, cap / 2)));
      p.tile_h = std::max(1, cap / p.tile_w);
      p.tile_h = std::min(p.h_out, std::max(p.tile_h, std::min(p.ncand, p.h_out)));
      if (p.tile_w < p.w_out && p.tile_w < p.ncand) p.tile_w = std::min(p.w_out, p.ncand);
    }
    p.tiles_x = (p.w_out + p.tile_w - 1) / p.tile_w;
    p.tiles_y = (p.h_out + p.tile_h - 1) / p.tile_h;
    p.T = p.tiles_x * p.tiles_y;
  };
  tile_for(npm_cap);
  const int fill = p.queue ? kQueueFillBlocks * 256 / p.q_threads : kConvFillBlocks;
  while ((int64_t)std::max(batch, 1) * p.T < fill && npm_cap > 8) {
    const int prev = npm_cap;
    npm_cap >>= 1;
    tile_for(npm_cap);
    if (p.T > 1 && conv_scatter_smem(p.T) > 227 * 1024) {  // past the partition's tile limit
      tile_for(prev);
      break;
    }
  }
  const int per_y = p.tiles_y > 1 ? (p.ncand - 1 + p.tile_h - 1) / p.tile_h + 1 : 1;
  const int per_x = p.tiles_x > 1 ? (p.ncand - 1 + p.tile_w - 1) / p.tile_w + 1 : 1;
  p.list_stride = (int64_t)E * std::min(per_y * per_x, p.T);
  p.n_part_chunks = (E + kPartChunk - 1) / kPartChunk;
  // a tile's queues hold at most nslots entries per tile event
  p.part = p.T > 1 && !(p.queue && p.T <= kQueueNoPartTiles);
  // an unpartitioned tile's queues hold at most nslots entries per sample event
  p.queue_stride = p.queue ? (int64_t)p.nslots * (p.part ? p.list_stride : (int64_t)p.T * E) : 0;
  if (p.queue && p.tile_h * p.tile_w > p.q_threads)
    return fail(SALT_BAD_ARG, "queue form: tile larger than a block");
  if (p.T > 1 && conv_scatter_smem(p.T) > 227 * 1024)
    return fail(SALT_BAD_ARG, "conv output plane too large: its tile partition needs more shared "
                              "memory than a block has (at most 894 tiles)");
  p.smem = fused_smem(d, q, p, p.tile_h, p.tile_w, p.T);
  if (p.smem > 227 * 1024)
    return fail(SALT_BAD_ARG, "conv layer weights do not fit in shared memory (ic*k*k*oc too "
                              "large for the chosen weight width)");
  return SALT_OK;
}

struct ConvScratch {
  int32_t *stats, *s_total, *needed, *vmin, *vmax, *ovf, *tail_total, *oc_total, *chunk;
  size_t stats_bytes;
  uint32_t* sw;
  int32_t *tail_cnt, *counts, *tile_len, *tile_off, *lists, *hist, *order;
  int2* queues;
  uint32_t* addr_table;
};

static size_t conv_carve(const salt_conv_desc* d, const ConvPlan& p, int32_t B, int32_t E,
                         void* ws, ConvScratch& s) {
  Carver c(ws);
  const size_t nstat = (size_t)B * 6 + (size_t)B * d->oc + (size_t)B * p.n_spk_chunks;
  s.stats = c.take<int32_t>(nstat);
  s.stats_bytes = nstat * 4;
  if (s.stats) {
    s.s_total = s.stats;
    s.needed = s.stats + B;
    s.vmin = s.stats + 2 * B;
    s.vmax = s.stats + 3 * B;
    s.ovf = s.stats + 4 * B;
    s.tail_total = s.stats + 5 * B;
    s.oc_total = s.stats + 6 * B;
    s.chunk = s.oc_total + (size_t)B * d->oc;
  }
  s.sw = c.take<uint32_t>((size_t)B * E * p.nslots * p.G);
  s.tail_cnt = p.tail_mode ? c.take<int32_t>((size_t)B * p.n_neurons) : nullptr;
  if (p.part) {
    s.counts = c.take<int32_t>((size_t)B * p.n_part_chunks * p.T);
    s.tile_len = c.take<int32_t>((size_t)B * p.T);
    s.tile_off = c.take<int32_t>((size_t)B * p.T);
    s.lists = c.take<int32_t>((size_t)B * p.list_stride);
  } else {
    s.counts = s.tile_len = s.tile_off = s.lists = nullptr;
  }
  s.hist = c.take<int32_t>((size_t)B * 2 * p.n_sp);
  s.order = c.take<int32_t>((size_t)B);
  s.queues = p.queue ? c.take<int2>((size_t)B * p.queue_stride) : nullptr;
  s.addr_table = p.win ? c.take<uint32_t>((size_t)d->ic * d->h_in * d->w_in) : nullptr;
  return c.size();
}

// Scratch bytes of a conv layer on B samples: enough for the batch's own tiling and for the
// finest one a slice of the batch may take (plan_conv shrinks tiles for small batches; every
// scratch term grows with the tile count and the batch).
static salt_status conv_scratch_bytes(const salt_conv_desc* d, const salt_quant_desc* q, int32_t B,
                                      int32_t E, size_t& bytes) {
  ConvPlan p, fine;
  salt_status rc = plan_conv(d, q, B, E, p);
  if (rc) return rc;
  if ((rc = plan_conv(d, q, 1, E, fine))) return rc;
  ConvScratch s;
  bytes = std::max(conv_carve(d, p, B, E, nullptr, s), conv_carve(d, fine, B, E, nullptr, s));
  if (p.queue) {  // the widest unpartitioned tiling a row slice of the queue form may take
    ConvPlan wide = p;
    wide.T = kQueueNoPartTiles;
    wide.part = false;
    wide.queue_stride = (int64_t)p.nslots * kQueueNoPartTiles * E;
    bytes = std::max(bytes, conv_carve(d, wide, B, E, nullptr, s));
  }
  return SALT_OK;
}

// Optional CUDA-event pair recorded around the fused kernel (network profiling).
struct KernelTimer {
  cudaEvent_t start = nullptr, stop = nullptr;
};

static salt_status conv_forward_impl(const salt_conv_desc* d, const salt_quant_desc* q,
                                     const int32_t* qw, const int32_t* lut, const int32_t* vth,
                                     int32_t B, const salt_stream_in* in, salt_stream_out* out,
                                     int32_t* v_final, const salt_layer_stats* stats, void* ws,
                                     size_t ws_bytes, cudaStream_t st,
                                     const KernelTimer* timer = nullptr) {
  salt_status rc = check_quant(q);
  if (rc) return rc;
  if ((rc = check_stream_in(in, B))) return rc;
  if (!qw || (q->lut_len > 0 && !lut) || (q->has_vth && !vth) || !out || !out->times ||
      !out->src || !out->n_real || !v_final)
    return fail(SALT_BAD_ARG, "conv layer: NULL parameter or output pointer");
  const int32_t E = in->capacity;
  ConvPlan p;
  if ((rc = plan_conv(d, q, B, E, p))) return rc;
  ConvScratch s;
  const size_t need = conv_carve(d, p, B, E, nullptr, s);
  if (!ws || ws_bytes < need) return fail(SALT_WORKSPACE_TOO_SMALL, "conv workspace too small");
  if (reinterpret_cast<uintptr_t>(ws) & 255) return fail(SALT_BAD_ARG, "workspace not 256-byte aligned");
  conv_carve(d, p, B, E, ws, s);

  ConvLaunch L;
  memset(&L, 0, sizeof(L));
  L.ic = d->ic; L.h_in = d->h_in; L.w_in = d->w_in; L.hw_in = d->h_in * d->w_in;
  L.oc = d->oc; L.k = d->k; L.s = d->s; L.p = d->p;
  L.h_out = p.h_out; L.w_out = p.w_out; L.n_sp = p.n_sp; L.n_neurons = p.n_neurons;
  L.ncand = p.ncand; L.nslots = p.nslots;
  L.L = d->max_queue_len; L.M = d->max_out_spikes; L.max_extra = d->max_extra_steps;
  L.lpu = p.lpu; L.G = p.G; L.ocp = p.ocp;
  L.tile_h = p.tile_h; L.tile_w = p.tile_w; L.tiles_x = p.tiles_x; L.T = p.T;
  L.fd_hw = FastDiv((uint32_t)(d->h_in * d->w_in));
  L.fd_w = FastDiv((uint32_t)d->w_in);
  L.fd_s = FastDiv((uint32_t)d->s);
  L.fd_G = FastDiv((uint32_t)p.G);
  L.fd_tw = FastDiv((uint32_t)p.tile_w);
  L.fd_th = FastDiv((uint32_t)p.tile_h);
  L.n_part_chunks = p.n_part_chunks; L.list_stride = p.list_stride;
  L.in.times = in->times; L.in.src = in->src; L.in.capacity = E; L.in.virtual_pads = in->virtual_pads;
  L.in_nreal = in->n_real; L.batch = B;
  L.q = qw; L.lut = lut; L.lut_in_smem = q->lut_len <= kLutSmemMax; L.vth = vth;
  L.has_vth = q->has_vth != 0; L.qc = make_qc(q);
  L.v_final = v_final;
  L.sw = s.sw; L.sw_stride = (int64_t)E * p.nslots * p.G;
  L.chunk_spikes = s.chunk; L.chunk_off = s.chunk; L.n_spk_chunks = p.n_spk_chunks;
  L.s_total = s.s_total; L.oc_total = s.oc_total; L.needed = s.needed; L.vmin = s.vmin;
  L.vmax = s.vmax; L.ovf = s.ovf; L.tail_total = s.tail_total;
  L.tail_mode = p.tail_mode; L.tail_cnt = s.tail_cnt;
  L.tile_len = s.tile_len; L.tile_off = s.tile_off; L.tile_lists = s.lists;
  L.order = B >= kOrderMinBatch ? s.order : nullptr;  // small batches: launch-bound anyway
  L.queues = s.queues;
  L.queue_stride = p.queue_stride;
  L.fd_sww = FastDiv((uint32_t)(p.nslots * p.G));
  L.q_shift = queue_shift((int64_t)E * p.nslots * p.G);
  L.q_threads = p.q_threads;
  L.addr_table = s.addr_table;
  L.n_addr = d->ic * d->h_in * d->w_in;
  L.grp_in_smem = p.grp_in_smem;

  SALT_CUDA(cudaMemsetAsync(s.stats, 0, s.stats_bytes, st));
  if (L.order) {
    sample_order_desc<<<1, kOrderThreads, 0, st>>>(in->n_real, E, B, s.order);
    SALT_LAUNCHED("sample_order_desc");
  }
  if (p.part) {
    // a few blocks per sample loop over its chunks (chunks past its events are skipped)
    dim3 gp(std::min(p.n_part_chunks, std::max(2, (4 * 1184 + B - 1) / B)), B);
    conv_tile_count<<<gp, kPartThreads, p.T * sizeof(int32_t), st>>>(L, s.counts);
    SALT_LAUNCHED("conv_tile_count");
    conv_tile_scan_offsets<<<(B * 32 + 255) / 256, 256, 0, st>>>(L, s.counts, s.tile_len,
                                                                 s.tile_off);
    SALT_LAUNCHED("conv_tile_scan_offsets");
    const size_t scatter_smem = conv_scatter_smem(p.T);
    if (scatter_smem > 48 * 1024)
      SALT_CUDA(cudaFuncSetAttribute((const void*)conv_tile_scatter,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)scatter_smem));
    conv_tile_scatter<<<gp, kPartThreads, scatter_smem, st>>>(L, s.counts, s.lists);
    SALT_LAUNCHED("conv_tile_scatter");
  }
  // a neuron sees at most max_queue_len weighted steps
  if (p.win) {
    conv_addr_table<<<(L.n_addr + 255) / 256, 256, 0, st>>>(L, s.addr_table);
    SALT_LAUNCHED("conv_addr_table");
  }
  const int form = step_form(q, d->max_queue_len);
  void* fn = p.queue ? conv_queue_kernel(p.wt_bytes, p.lpu, q->overflow_mode == SALT_SATURATE, form,
                                         p.win, p.q_threads)
                     : conv_fused_kernel(p.wt_bytes, p.lpu, q->overflow_mode == SALT_SATURATE, form);
  if (!fn) return fail(SALT_BAD_ARG, "conv layer: no kernel for this step form");
  SALT_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem));
  void* args[] = {&L};
  if (timer) SALT_CUDA(cudaEventRecord(timer->start, st));
  SALT_CUDA(cudaLaunchKernel(fn, dim3(p.T, B), dim3(p.q_threads), args, p.smem, st));
  SALT_LAUNCHED("conv_fused");
  if (timer) SALT_CUDA(cudaEventRecord(timer->stop, st));
  // conv_fused counts only catch-up/identity spikes into s_total: the spike words' count is the
  // scan's total
  spike_chunk_scan<<<(B * 32 + 255) / 256, 256, 0, st>>>(s.chunk, p.n_spk_chunks, B, s.s_total);
  SALT_LAUNCHED("spike_chunk_scan");
  {
    salt_stream_out so = *out;
    void* cargs[] = {&L, &so};
    SALT_CUDA(cudaLaunchKernel(conv_compact_kernel(p.ncand, p.G, L.addr_table != nullptr),
                               dim3(conv_compact_blocks(p.n_spk_chunks, B), B),
                               dim3(kCompactThreads), cargs, 0, st));
  }
  SALT_LAUNCHED("conv_compact");
  if (p.tail_mode) {
    conv_tail_append<<<B, kCompactThreads, 0, st>>>(L, *out);
    SALT_LAUNCHED("conv_tail_append");
  }
  conv_truncated<<<B, kTruncThreads, 0, st>>>(L, *out, s.hist);
  SALT_LAUNCHED("conv_truncated");
  FinishArgs fa{s.s_total, s.needed, s.vmin, s.vmax, s.ovf, d->max_queue_len, d->max_out_spikes,
                d->max_extra_steps, 1, B, 1 << (q->i_V + q->f_V - 1)};
  salt_layer_stats none{};
  layer_finish<<<(B + 255) / 256, 256, 0, st>>>(fa, out->n_real, stats ? *stats : none);
  SALT_LAUNCHED("layer_finish");
  return SALT_OK;
}

// ---------------------------------------------------------------- fc

struct FCScratch {
  int32_t *stats, *s_total, *vmin, *vmax, *ovf, *chunk, *n_spk, *qT, *order;
  size_t stats_bytes;
  uint32_t* sw;
};

static size_t fc_carve(const salt_fc_desc* d, const salt_quant_desc* q, int32_t B, int32_t E,
                       bool need_qT, void* ws, FCScratch& s) {
  Carver c(ws);
  const int G = (d->n_out + 31) / 32;
  const int nsc = (E + kSpkChunk - 1) / kSpkChunk;
  const size_t nstat = (size_t)B * 4 + (q->has_vth ? (size_t)B * nsc : 0);
  s.stats = c.take<int32_t>(nstat);
  s.stats_bytes = nstat * 4;
  if (s.stats) {
    s.s_total = s.stats;
    s.vmin = s.stats + B;
    s.vmax = s.stats + 2 * B;
    s.ovf = s.stats + 3 * B;
    s.chunk = q->has_vth ? s.stats + 4 * B : nullptr;
  }
  s.sw = q->has_vth ? c.take<uint32_t>((size_t)B * E * G) : nullptr;
  s.n_spk = q->has_vth ? c.take<int32_t>((size_t)B * d->n_out) : nullptr;
  s.qT = need_qT ? c.take<int32_t>((size_t)d->n_in * d->n_out) : nullptr;
  s.order = c.take<int32_t>((size_t)B);
  return c.size();
}

static salt_status check_fc(const salt_fc_desc* d) {
  if (!d) return fail(SALT_BAD_ARG, "fc descriptor is NULL");
  if (d->n_in < 1 || d->n_out < 1) return fail(SALT_BAD_ARG, "fc: n_in and n_out must be >= 1");
  if (d->max_out_spikes < 1) return fail(SALT_BAD_ARG, "max_out_spikes must be >= 1");
  return SALT_OK;
}

static salt_status fc_forward_impl(const salt_fc_desc* d, const salt_quant_desc* q,
                                   const int32_t* qw, bool q_is_transposed, const int32_t* lut,
                                   const int32_t* vth, int32_t B, const salt_stream_in* in,
                                   salt_stream_out* out, int32_t* v_final,
                                   const salt_layer_stats* stats, void* ws, size_t ws_bytes,
                                   cudaStream_t st) {
  salt_status rc = check_quant(q);
  if (rc) return rc;
  if ((rc = check_stream_in(in, B))) return rc;
  if ((rc = check_fc(d))) return rc;
  if (!qw || (q->lut_len > 0 && !lut) || (q->has_vth && !vth) || !out || !out->n_real ||
      !v_final || (q->has_vth && (!out->times || !out->src)))
    return fail(SALT_BAD_ARG, "fc layer: NULL parameter or output pointer");
  const int32_t E = in->capacity;
  FCScratch s;
  const size_t need = fc_carve(d, q, B, E, !q_is_transposed, nullptr, s);
  if (!ws || ws_bytes < need) return fail(SALT_WORKSPACE_TOO_SMALL, "fc workspace too small");
  if (reinterpret_cast<uintptr_t>(ws) & 255) return fail(SALT_BAD_ARG, "workspace not 256-byte aligned");
  fc_carve(d, q, B, E, !q_is_transposed, ws, s);
  const int32_t* qT = qw;
  if (!q_is_transposed) {
    const int64_t n = (int64_t)d->n_in * d->n_out;
    transpose_i32<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(qw, s.qT, d->n_out, d->n_in);
    SALT_LAUNCHED("transpose_i32");
    qT = s.qT;
  }
  FCLaunch L;
  memset(&L, 0, sizeof(L));
  L.n_in = d->n_in; L.n_out = d->n_out; L.G = (d->n_out + 31) / 32;
  L.M = d->max_out_spikes; L.max_extra = d->max_extra_steps;
  L.in.times = in->times; L.in.src = in->src; L.in.capacity = E; L.in.virtual_pads = in->virtual_pads;
  L.in_nreal = in->n_real; L.batch = B;
  L.qT = qT; L.lut = lut; L.vth = vth; L.has_vth = q->has_vth != 0; L.qc = make_qc(q);
  L.v_final = v_final;
  L.sw = s.sw; L.sw_stride = (int64_t)E * L.G;
  L.chunk_spikes = s.chunk; L.chunk_off = s.chunk; L.n_spk_chunks = (E + kSpkChunk - 1) / kSpkChunk;
  L.s_total = s.s_total; L.vmin = s.vmin; L.vmax = s.vmax; L.ovf = s.ovf; L.n_spk = s.n_spk;
  L.tail_mode = q->has_vth && q->needs_tail;
  SALT_CUDA(cudaMemsetAsync(s.stats, 0, s.stats_bytes, st));
  L.order = B >= kOrderMinBatch ? s.order : nullptr;  // small batches: launch-bound anyway
  if (L.order) {
    sample_order_desc<<<1, kOrderThreads, 0, st>>>(in->n_real, E, B, s.order);
    SALT_LAUNCHED("sample_order_desc");
  }
  // narrow layers (the membrane readouts) pack several samples into a warp; weight tables that
  // fit are staged in shared memory at the width of their codes
  const int lpu = d->n_out <= 8 ? 8 : (d->n_out <= 16 ? 16 : 32);
  // every block serves one neuron group (grid y) for 4 warps of samples (grid x) and stages
  // that group's weight columns
  int wt = q->q_bits <= 8 ? 1 : (q->q_bits <= 16 ? 2 : 4);
  if (fc_scan_q_bytes(d->n_in, d->n_out, wt, lpu) > kFcQSmemMax) wt = 0;
  const size_t smem = fc_scan_smem(d->n_in, d->n_out, q->lut_len, wt, lpu);
  const int64_t warps = ((int64_t)B + 32 / lpu - 1) / (32 / lpu);
  const int wpb = kFcThreads / 32;
  const dim3 grid((unsigned)((warps + wpb - 1) / wpb), (unsigned)L.G);
  // a neuron sees at most one weighted step per input entry
  void* scan_fn = fc_scan_kernel(q->has_vth != 0, q->overflow_mode == SALT_SATURATE, lpu, wt,
                                 step_form(q, E));
  if (smem > 48 * 1024)
    SALT_CUDA(cudaFuncSetAttribute(scan_fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  void* scan_args[] = {&L};
  SALT_CUDA(cudaLaunchKernel(scan_fn, dim3(grid), dim3(kFcThreads), scan_args, smem, st));
  SALT_LAUNCHED("fc_scan");
  if (q->has_vth) {
    spike_chunk_scan<<<(B * 32 + 255) / 256, 256, 0, st>>>(s.chunk, L.n_spk_chunks, B, nullptr);
    SALT_LAUNCHED("spike_chunk_scan");
    fc_compact<<<dim3(std::min(L.n_spk_chunks, compact_blocks(B)), B), kCompactThreads, 0,
                 st>>>(L, *out);
    SALT_LAUNCHED("fc_compact");
    fc_truncated<<<B, kCompactThreads, 0, st>>>(L, *out);
    SALT_LAUNCHED("fc_truncated");
  }
  FinishArgs fa{s.s_total, nullptr, s.vmin, s.vmax, s.ovf, 0, d->max_out_spikes,
                d->max_extra_steps, 0, B, 1 << (q->i_V + q->f_V - 1)};
  salt_layer_stats none{};
  layer_finish<<<(B + 255) / 256, 256, 0, st>>>(fa, out->n_real, stats ? *stats : none);
  SALT_LAUNCHED("layer_finish");
  return SALT_OK;
}

// ---------------------------------------------------------------- float fc

struct FloatScratch {
  int32_t *stats, *s_total, *needed, *exact, *chunk, *hist, *bcnt, *n_spk;
  double* bsum;
  size_t stats_bytes;
  float *wT, *lut;
  uint32_t* sw;
  float *r_vstart, *r_vend, *r_u1, *r_A1, *r_M, *r_Aseg, *r_sum;
  int32_t *r_k1, *r_nspk, *r_cnt, *r_mono;
};

// Time segments per sample: as many (segment, group) warps as fit on the GPU in one wave (148
// SMs x kFloatSegBlocksPerSM); one segment — a plain in-order scan, no guessing — when neurons x
// samples already fill it.  Segments hold at least 4096 events so that the warm-up guess stays
// affordable.
static int32_t float_segments(int32_t G, int32_t B, int32_t E) {
  const int64_t wave = 148LL * kFloatSegBlocksPerSM;
  const int64_t per = (int64_t)G * B;
  return (int32_t)std::max<int64_t>(1, std::min<int64_t>(wave / per, std::max(1, E / 4096)));
}

static size_t float_carve(const salt_float_fc_desc* d, int32_t B, int32_t E, bool gain, void* ws,
                          FloatScratch& s) {
  Carver c(ws);
  const int G = (d->n_out + 31) / 32, S = float_segments(G, B, E);
  const int nsc = (E + kSpkChunk - 1) / kSpkChunk;
  // one zeroed block: per-sample counters, flags, chunk counts and (unit gains) the bound's
  // histogram and per-neuron sums
  const size_t nb = gain ? 0 : (size_t)B * d->n_out;
  const size_t nstat = (size_t)B * 2 + (size_t)B * G + (size_t)B * nsc +
                       (gain ? 0 : (size_t)B * d->n_in) + nb + 2 * nb + 1;
  s.stats = c.take<int32_t>(nstat);
  s.stats_bytes = nstat * 4;
  if (s.stats) {
    s.s_total = s.stats;
    s.needed = s.stats + B;
    s.exact = s.stats + 2 * B;
    s.chunk = s.exact + (size_t)B * G;
    s.hist = gain ? nullptr : s.chunk + (size_t)B * nsc;
    s.bcnt = gain ? nullptr : s.hist + (size_t)B * d->n_in;
    // 8-byte aligned: the block starts 256-aligned and everything before it is 4-byte counts
    int32_t* dbl = gain ? nullptr : s.bcnt + nb;
    if (dbl && (reinterpret_cast<uintptr_t>(dbl) & 7)) ++dbl;
    s.bsum = reinterpret_cast<double*>(dbl);
  } else {
    s.hist = s.bcnt = nullptr;
    s.bsum = nullptr;
  }
  s.wT = c.take<float>((size_t)d->n_in * d->n_out);
  s.lut = c.take<float>((size_t)kFloatLut * d->n_out);
  s.sw = c.take<uint32_t>((size_t)B * E * G);
  s.n_spk = c.take<int32_t>((size_t)B * d->n_out);
  const size_t nr = (size_t)B * S * d->n_out;
  s.r_vstart = c.take<float>(nr);
  s.r_vend = c.take<float>(nr);
  s.r_u1 = c.take<float>(nr);
  s.r_A1 = c.take<float>(nr);
  s.r_M = c.take<float>(nr);
  s.r_Aseg = c.take<float>(nr);
  s.r_k1 = c.take<int32_t>(nr);
  s.r_nspk = c.take<int32_t>(nr);
  s.r_sum = gain ? c.take<float>(nr) : nullptr;
  s.r_cnt = gain ? c.take<int32_t>(nr) : nullptr;
  s.r_mono = c.take<int32_t>((size_t)B * S);
  return c.size();
}

static salt_status check_float(const salt_float_fc_desc* d) {
  if (!d) return fail(SALT_BAD_ARG, "float fc descriptor is NULL");
  if (d->n_in < 1 || d->n_out < 1) return fail(SALT_BAD_ARG, "float fc: n_in and n_out must be >= 1");
  if (d->chunk_size < 1) return fail(SALT_BAD_ARG, "float fc: chunk_size must be >= 1");
  if (d->max_out_spikes < 1) return fail(SALT_BAD_ARG, "max_out_spikes must be >= 1");
  if (d->max_extra_steps < 0) return fail(SALT_BAD_ARG, "max_extra_steps must be >= 0");
  if (!(d->v_th > 0.0f) || d->v_th == INFINITY)
    return fail(SALT_BAD_ARG, "float fc: v_th must be a finite value > 0 (a threshold <= 0 "
                              "fires on pad entries)");
  return SALT_OK;
}

__global__ void float_finish(const int32_t* __restrict__ s_total,
                             const int32_t* __restrict__ needed, int32_t M, int32_t max_extra,
                             int32_t batch, int32_t* out_nreal, salt_float_layer_stats st) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int32_t S = s_total[b], need = needed[b];
  if (out_nreal) out_nreal[b] = S;
  if (st.spike_count) st.spike_count[b] = S;
  if (st.needed_extra_steps) st.needed_extra_steps[b] = need;
  if (st.fits) st.fits[b] = S <= M && need <= max_extra;  // capacity.py:60-63
}

// Optional per-thread timing of float FC layers: CUDA events around the speculative segment
// kernel and around the whole layer, summed when read.
struct FloatProfile {
  bool on = false;
  std::vector<cudaEvent_t> seg, layer;  // start/stop pairs, in order
  double seg_ms = 0, layer_ms = 0;
  int32_t n = 0;
};
static thread_local FloatProfile g_fprof;

static cudaEvent_t timing_event() {
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

static salt_status float_forward_impl(const salt_float_fc_desc* d, const float* w,
                                      const float* decay_base, int32_t B,
                                      const salt_stream_in* in, const float* gain,
                                      salt_stream_out* out, float* v_final,
                                      const salt_float_layer_stats* stats, void* ws,
                                      size_t ws_bytes, cudaStream_t st) {
  salt_status rc = check_float(d);
  if (rc) return rc;
  if ((rc = check_stream_in(in, B))) return rc;
  if (!w || !decay_base || !out || !out->times || !out->src || !out->n_real || !v_final)
    return fail(SALT_BAD_ARG, "float fc layer: NULL parameter or output pointer");
  const int32_t E = in->capacity;
  const int64_t base_steps = ((int64_t)E + d->chunk_size - 1) / d->chunk_size;
  if (base_steps + d->max_extra_steps > INT32_MAX)
    return fail(SALT_BAD_ARG, "float fc: ceil(capacity / chunk_size) + max_extra_steps overflows");
  FloatScratch s;
  const size_t need = float_carve(d, B, E, gain != nullptr, nullptr, s);
  if (!ws || ws_bytes < need) return fail(SALT_WORKSPACE_TOO_SMALL, "float fc workspace too small");
  if (reinterpret_cast<uintptr_t>(ws) & 255) return fail(SALT_BAD_ARG, "workspace not 256-byte aligned");
  float_carve(d, B, E, gain != nullptr, ws, s);

  FloatLaunch P;
  memset(&P, 0, sizeof(P));
  P.n_in = d->n_in; P.n_out = d->n_out; P.G = (d->n_out + 31) / 32;
  P.S = float_segments(P.G, B, E);
  P.C = d->chunk_size; P.base_steps = (int32_t)base_steps;
  P.max_steps = (int32_t)(base_steps + d->max_extra_steps);
  P.vth = d->v_th; P.margin = d->v_th * 1.5e-5f;
  P.in.times = in->times; P.in.src = in->src; P.in.capacity = E; P.in.virtual_pads = in->virtual_pads;
  P.in_nreal = in->n_real; P.batch = B; P.gain = gain;
  P.w = w; P.wT = s.wT; P.decay_base = decay_base; P.lut = s.lut; P.v_final = v_final;
  P.sw = s.sw; P.sw_stride = (int64_t)E * P.G;
  P.chunk_spikes = s.chunk; P.n_spk_chunks = (E + kSpkChunk - 1) / kSpkChunk;
  P.s_total = s.s_total; P.needed = s.needed; P.n_spk = s.n_spk; P.exact = s.exact; P.hist = s.hist;
  P.bcnt = s.bcnt; P.bsum = s.bsum; P.warm_max = kFloatWarmMax;
  P.r_vstart = s.r_vstart; P.r_vend = s.r_vend; P.r_u1 = s.r_u1; P.r_A1 = s.r_A1; P.r_M = s.r_M; P.r_Aseg = s.r_Aseg;
  P.r_sum = s.r_sum; P.r_k1 = s.r_k1; P.r_nspk = s.r_nspk; P.r_cnt = s.r_cnt; P.r_mono = s.r_mono;
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};  // layer start/stop, segment start/stop
  if (g_fprof.on) {
    for (auto& e : ev)
      if (!(e = timing_event())) return fail(SALT_CUDA_ERROR, "cudaEventCreate failed");
    g_fprof.layer.push_back(ev[0]);
    g_fprof.layer.push_back(ev[1]);
    g_fprof.seg.push_back(ev[2]);
    g_fprof.seg.push_back(ev[3]);
    SALT_CUDA(cudaEventRecord(ev[0], st));
  }
  SALT_CUDA(cudaMemsetAsync(s.stats, 0, s.stats_bytes, st));
  SALT_CUDA(float_fc_launch(P, st, &g_launches, ev[2], ev[3]));

  // the FC compaction reads the spike words and per-neuron counts in the integer layer's form
  FCLaunch L;
  memset(&L, 0, sizeof(L));
  L.n_in = d->n_in; L.n_out = d->n_out; L.G = P.G; L.M = d->max_out_spikes;
  L.in = P.in; L.in_nreal = in->n_real; L.batch = B;
  L.sw = s.sw; L.sw_stride = P.sw_stride;
  L.chunk_spikes = s.chunk; L.chunk_off = s.chunk; L.n_spk_chunks = P.n_spk_chunks;
  L.s_total = s.s_total; L.n_spk = s.n_spk; L.tail_mode = 0;
  spike_chunk_scan<<<(B * 32 + 255) / 256, 256, 0, st>>>(s.chunk, L.n_spk_chunks, B, nullptr);
  SALT_LAUNCHED("spike_chunk_scan");
  fc_compact<<<dim3(std::min(L.n_spk_chunks, compact_blocks(B)), B), kCompactThreads, 0, st>>>(
      L, *out);
  SALT_LAUNCHED("fc_compact");
  fc_truncated<<<B, kCompactThreads, 0, st>>>(L, *out);
  SALT_LAUNCHED("fc_truncated");
  salt_float_layer_stats none{};
  float_finish<<<(B + 255) / 256, 256, 0, st>>>(s.s_total, s.needed, d->max_out_spikes,
                                                d->max_extra_steps, B, out->n_real,
                                                stats ? *stats : none);
  SALT_LAUNCHED("float_finish");
  if (ev[1]) SALT_CUDA(cudaEventRecord(ev[1], st));
  return SALT_OK;
}

}  // namespace salt

// ==================================================================== C ABI
using namespace salt;

struct LayerRec {
  salt_layer_spec spec;
  int32_t *d_q = nullptr, *d_lut = nullptr, *d_vth = nullptr;
  int64_t n_neurons = 0;
  int32_t M = 0;
};

struct TimedLaunch {
  int32_t layer;
  int32_t whole_layer;  // 1: events bracket the whole layer, 0: the fused kernel
  KernelTimer ev;
};

struct salt_network {
  std::vector<LayerRec> layers;
  int32_t last_launches = 0;
  bool profiling = false;
  std::vector<TimedLaunch> timed;   // recorded, not yet read
  std::vector<KernelTimer> pool;    // events free for reuse
};

extern "C" {

// ---------------------------------------------------------------- runtime plumbing

// The current device's default memory pool keeps what cudaFreeAsync returns instead of handing
// it back to the driver at the next synchronisation (a per-process pool attribute).
static salt_status keep_pool_cached() {
  int dev = 0;
  SALT_CUDA(cudaGetDevice(&dev));
  static thread_local uint64_t done_mask = 0;
  if (dev < 64 && (done_mask >> dev) & 1u) return SALT_OK;
  cudaMemPool_t pool;
  SALT_CUDA(cudaDeviceGetDefaultMemPool(&pool, dev));
  uint64_t keep = UINT64_MAX;
  SALT_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
  if (dev < 64) done_mask |= uint64_t(1) << dev;
  return SALT_OK;
}

salt_status salt_malloc(size_t bytes, void* stream, void** ptr) {
  if (!ptr) return fail(SALT_BAD_ARG, "salt_malloc: ptr is NULL");
  *ptr = nullptr;
  if (bytes == 0) return SALT_OK;
  salt_status rc = keep_pool_cached();
  if (rc) return rc;
  SALT_CUDA(cudaMallocAsync(ptr, bytes, (cudaStream_t)stream));
  return SALT_OK;
}

salt_status salt_free(void* ptr, void* stream) {
  if (ptr) SALT_CUDA(cudaFreeAsync(ptr, (cudaStream_t)stream));
  return SALT_OK;
}

salt_status salt_host_alloc(size_t bytes, void** ptr) {
  if (!ptr) return fail(SALT_BAD_ARG, "salt_host_alloc: ptr is NULL");
  *ptr = nullptr;
  SALT_CUDA(cudaHostAlloc(ptr, bytes ? bytes : 1, cudaHostAllocPortable | cudaHostAllocMapped));
  return SALT_OK;
}

salt_status salt_host_free(void* ptr) {
  if (ptr) SALT_CUDA(cudaFreeHost(ptr));
  return SALT_OK;
}

salt_status salt_memcpy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return SALT_OK;
  if (!dst || !src) return fail(SALT_BAD_ARG, "salt_memcpy_async: NULL pointer");
  SALT_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, (cudaStream_t)stream));
  return SALT_OK;
}

salt_status salt_memset_async(void* ptr, int32_t value, size_t bytes, void* stream) {
  if (bytes == 0) return SALT_OK;
  if (!ptr) return fail(SALT_BAD_ARG, "salt_memset_async: NULL pointer");
  SALT_CUDA(cudaMemsetAsync(ptr, value, bytes, (cudaStream_t)stream));
  return SALT_OK;
}

salt_status salt_device_count(int32_t* count) {
  if (!count) return fail(SALT_BAD_ARG, "salt_device_count: NULL");
  int n = 0;
  const cudaError_t e = cudaGetDeviceCount(&n);
  *count = e == cudaSuccess ? n : 0;
  if (e != cudaSuccess) cudaGetLastError();  // no driver or no device: report 0 devices
  return SALT_OK;
}

salt_status salt_set_device(int32_t device) {
  SALT_CUDA(cudaSetDevice(device));
  return SALT_OK;
}

salt_status salt_get_device(int32_t* device) {
  int d = 0;
  SALT_CUDA(cudaGetDevice(&d));
  *device = d;
  return SALT_OK;
}

salt_status salt_device_synchronize(void) {
  SALT_CUDA(cudaDeviceSynchronize());
  return SALT_OK;
}

salt_status salt_stream_create(void** stream) {
  cudaStream_t s;
  SALT_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = (void*)s;
  return SALT_OK;
}

salt_status salt_stream_create_high_priority(void** stream) {
  int least = 0, greatest = 0;
  SALT_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest));
  cudaStream_t s;
  SALT_CUDA(cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, greatest));
  *stream = (void*)s;
  return SALT_OK;
}

salt_status salt_stream_destroy(void* stream) {
  if (stream) SALT_CUDA(cudaStreamDestroy((cudaStream_t)stream));
  return SALT_OK;
}

salt_status salt_stream_synchronize(void* stream) {
  SALT_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  return SALT_OK;
}

salt_status salt_stream_wait_event(void* stream, void* event) {
  SALT_CUDA(cudaStreamWaitEvent((cudaStream_t)stream, (cudaEvent_t)event, 0));
  return SALT_OK;
}

salt_status salt_event_create(int32_t timing, void** event) {
  cudaEvent_t e;
  SALT_CUDA(cudaEventCreateWithFlags(&e, timing ? cudaEventDefault : cudaEventDisableTiming));
  *event = (void*)e;
  return SALT_OK;
}

salt_status salt_event_destroy(void* event) {
  if (event) SALT_CUDA(cudaEventDestroy((cudaEvent_t)event));
  return SALT_OK;
}

salt_status salt_event_record(void* event, void* stream) {
  SALT_CUDA(cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream));
  return SALT_OK;
}

salt_status salt_event_synchronize(void* event) {
  SALT_CUDA(cudaEventSynchronize((cudaEvent_t)event));
  return SALT_OK;
}

salt_status salt_event_query(void* event, int32_t* done) {
  if (!done) return fail(SALT_BAD_ARG, "salt_event_query: NULL");
  const cudaError_t e = cudaEventQuery((cudaEvent_t)event);
  if (e == cudaErrorNotReady) {
    *done = 0;
    return SALT_OK;
  }
  SALT_CUDA(e);
  *done = 1;
  return SALT_OK;
}

salt_status salt_event_elapsed_ms(void* start, void* stop, float* ms) {
  SALT_CUDA(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)stop));
  return SALT_OK;
}

salt_status salt_graph_begin_capture(void* stream) {
  if (!stream) return fail(SALT_BAD_ARG, "graph capture needs a non-default stream");
  SALT_CUDA(cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeThreadLocal));
  return SALT_OK;
}

salt_status salt_graph_end_capture(void* stream, void** graph_exec) {
  cudaGraph_t g = nullptr;
  SALT_CUDA(cudaStreamEndCapture((cudaStream_t)stream, &g));
  cudaGraphExec_t ex = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess)
    return fail(SALT_CUDA_ERROR, std::string("cudaGraphInstantiate: ") + cudaGetErrorString(e));
  *graph_exec = (void*)ex;
  return SALT_OK;
}

salt_status salt_graph_launch(void* graph_exec, void* stream) {
  SALT_CUDA(cudaGraphLaunch((cudaGraphExec_t)graph_exec, (cudaStream_t)stream));
  return SALT_OK;
}

salt_status salt_graph_destroy(void* graph_exec) {
  if (graph_exec) SALT_CUDA(cudaGraphExecDestroy((cudaGraphExec_t)graph_exec));
  return SALT_OK;
}

const char* salt_last_error(void) { return g_err.c_str(); }
const char* salt_version(void) { return "salt_b200 0.1 (sm_100a)"; }
int64_t salt_launch_counter(int32_t reset) {
  const int64_t v = g_launches;
  if (reset) g_launches = 0;
  return v;
}

salt_status salt_conv_layer_workspace_size(const salt_conv_desc* layer, const salt_quant_desc* quant,
                                           int32_t batch, int32_t in_capacity, size_t* bytes) {
  salt_status rc = check_quant(quant);
  if (rc) return rc;
  if (!bytes || batch < 1 || in_capacity < 1) return fail(SALT_BAD_ARG, "bad batch/capacity");
  return conv_scratch_bytes(layer, quant, batch, in_capacity, *bytes);
}

salt_status salt_conv_layer_forward(const salt_conv_desc* layer, const salt_quant_desc* quant,
                                    const int32_t* q, const int32_t* lut, const int32_t* vth,
                                    int32_t batch, const salt_stream_in* in, salt_stream_out* out,
                                    int32_t* v_final, const salt_layer_stats* stats,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  return conv_forward_impl(layer, quant, q, lut, vth, batch, in, out, v_final, stats, workspace,
                           workspace_bytes, (cudaStream_t)stream);
}

salt_status salt_conv_layer_forward_noalloc(const salt_conv_desc* layer,
                                            const salt_quant_desc* quant, const int32_t* q,
                                            const int32_t* lut, const int32_t* vth, int32_t batch,
                                            const salt_stream_in* in, salt_stream_out* out,
                                            int32_t* v_final, const salt_layer_stats* stats,
                                            void* stream) {
  size_t need = 0;
  salt_status rc = salt_conv_layer_workspace_size(layer, quant, batch, in ? in->capacity : 0, &need);
  if (rc) return rc;
  if (need > SALT_NOALLOC_SCRATCH_BYTES)
    return fail(SALT_WORKSPACE_TOO_SMALL,
                "conv layer needs " + std::to_string(need) + " bytes of scratch; the fixed scratch "
                "of salt_conv_layer_forward_noalloc holds " +
                std::to_string(SALT_NOALLOC_SCRATCH_BYTES) +
                " (use salt_conv_layer_forward with a workspace, or a smaller batch)");
  void* ws = nullptr;
  SALT_CUDA(fixed_scratch_address(&ws));
  return conv_forward_impl(layer, quant, q, lut, vth, batch, in, out, v_final, stats, ws, need,
                           (cudaStream_t)stream);
}

salt_status salt_conv_layer_trace(const salt_conv_desc* d, const salt_quant_desc* q,
                                  const int32_t* qw, const int32_t* lut, const int32_t* vth,
                                  int32_t B, const salt_stream_in* in, int32_t* v_steps,
                                  uint8_t* spike_mask, float* event_ms,
                                  const salt_neuron_trace* per_neuron, void* stream) {
  salt_status rc = check_quant(q);
  if (rc) return rc;
  if ((rc = check_stream_in(in, B))) return rc;
  if (!d || d->ic < 1 || d->oc < 1 || d->k < 1 || d->s < 1 || d->p < 0 || d->h_in < 1 ||
      d->w_in < 1 || d->max_queue_len < 1)
    return fail(SALT_BAD_ARG, "conv trace: bad geometry or max_queue_len");
  const int32_t h_out = (d->h_in + 2 * d->p - d->k) / d->s + 1;
  const int32_t w_out = (d->w_in + 2 * d->p - d->k) / d->s + 1;
  if (h_out < 1 || w_out < 1) return fail(SALT_BAD_ARG, "conv trace: empty output plane");
  if (!qw || (q->lut_len > 0 && !lut) || (q->has_vth && !vth))
    return fail(SALT_BAD_ARG, "conv trace: NULL parameter pointer");
  ConvLaunch L;
  memset(&L, 0, sizeof(L));
  L.ic = d->ic; L.h_in = d->h_in; L.w_in = d->w_in; L.hw_in = d->h_in * d->w_in;
  L.oc = d->oc; L.k = d->k; L.s = d->s; L.p = d->p;
  L.h_out = h_out; L.w_out = w_out; L.n_sp = h_out * w_out;
  L.n_neurons = (int64_t)d->oc * h_out * w_out;
  L.L = d->max_queue_len;
  L.in.times = in->times; L.in.src = in->src; L.in.capacity = in->capacity;
  L.in.virtual_pads = in->virtual_pads;
  L.in_nreal = in->n_real; L.batch = B;
  L.q = qw; L.lut = lut; L.vth = vth; L.has_vth = q->has_vth != 0; L.qc = make_qc(q);
  SALT_CUDA(conv_trace_launch(L, per_neuron, v_steps, spike_mask, event_ms, (cudaStream_t)stream));
  ++g_launches;
  return SALT_OK;
}

salt_status salt_fc_layer_trace(const salt_fc_desc* d, const salt_quant_desc* q, const int32_t* qw,
                                const int32_t* lut, const int32_t* vth, int32_t B,
                                const salt_stream_in* in, int32_t* v_steps, uint8_t* spike_mask,
                                float* event_ms, const salt_neuron_trace* per_neuron,
                                void* stream) {
  salt_status rc = check_quant(q);
  if (rc) return rc;
  if ((rc = check_stream_in(in, B))) return rc;
  if ((rc = check_fc(d))) return rc;
  if (!qw || (q->lut_len > 0 && !lut) || (q->has_vth && !vth))
    return fail(SALT_BAD_ARG, "fc trace: NULL parameter pointer");
  FCLaunch L;
  memset(&L, 0, sizeof(L));
  L.n_in = d->n_in; L.n_out = d->n_out; L.G = (d->n_out + 31) / 32;
  L.in.times = in->times; L.in.src = in->src; L.in.capacity = in->capacity;
  L.in.virtual_pads = in->virtual_pads;
  L.in_nreal = in->n_real; L.batch = B;
  L.qT = qw;  // the trace kernel reads the caller's (n_out, n_in) layout
  L.lut = lut; L.vth = vth; L.has_vth = q->has_vth != 0; L.qc = make_qc(q);
  SALT_CUDA(fc_trace_launch(L, per_neuron, v_steps, spike_mask, event_ms, (cudaStream_t)stream));
  ++g_launches;
  return SALT_OK;
}

salt_status salt_stream_h2d_real(const float* host_times, const int32_t* host_src,
                                 int64_t host_pitch, const int32_t* n_real, int32_t batch,
                                 int32_t capacity, float* dev_times, int32_t* dev_src,
                                 void* stream) {
  if (!host_times || !host_src || !n_real || !dev_times || !dev_src)
    return fail(SALT_BAD_ARG, "stream transfer: NULL pointer");
  if (batch < 1 || batch > 65535 || capacity < 1 || host_pitch < capacity)
    return fail(SALT_BAD_ARG, "stream transfer: bad batch, capacity or pitch");
  // the host rows must be page-locked and mapped into the device address space
  void* dt = nullptr;
  void* ds = nullptr;
  if (cudaHostGetDevicePointer(&dt, const_cast<float*>(host_times), 0) != cudaSuccess ||
      cudaHostGetDevicePointer(&ds, const_cast<int32_t*>(host_src), 0) != cudaSuccess) {
    cudaGetLastError();
    return fail(SALT_BAD_ARG, "stream transfer: host rows are not pinned, mapped memory");
  }
  SALT_CUDA(gather_rows_launch(static_cast<const float*>(dt), static_cast<const int32_t*>(ds),
                               n_real, batch, capacity, host_pitch, dev_times, dev_src,
                               (cudaStream_t)stream));
  ++g_launches;
  return SALT_OK;
}

salt_status salt_float_fc_layer_workspace_size(const salt_float_fc_desc* layer, int32_t batch,
                                               int32_t in_capacity, int32_t has_gain,
                                               size_t* bytes) {
  salt_status rc = check_float(layer);
  if (rc) return rc;
  if (!bytes || batch < 1 || in_capacity < 1) return fail(SALT_BAD_ARG, "bad batch/capacity");
  FloatScratch s;
  *bytes = float_carve(layer, batch, in_capacity, has_gain != 0, nullptr, s);
  return SALT_OK;
}

salt_status salt_float_fc_layer_forward(const salt_float_fc_desc* layer, const float* w,
                                        const float* decay_base, int32_t batch,
                                        const salt_stream_in* in, const float* in_gain,
                                        salt_stream_out* out, float* v_final,
                                        const salt_float_layer_stats* stats, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  return float_forward_impl(layer, w, decay_base, batch, in, in_gain, out, v_final, stats,
                            workspace, workspace_bytes, (cudaStream_t)stream);
}

// ---------------------------------------------------------------- float conv layer

struct FConvPlan {
  int32_t h_out, w_out, n_sp, ncand, nslots, lpu, G, ocp, taps, n_spk_chunks, max_steps, base;
  int64_t n_neurons;
};

static salt_status plan_float_conv(const salt_float_conv_desc* d, int32_t E, FConvPlan& p) {
  if (!d) return fail(SALT_BAD_ARG, "float conv descriptor is NULL");
  if (d->ic < 1 || d->h_in < 1 || d->w_in < 1 || d->oc < 1 || d->k < 1 || d->s < 1 || d->p < 0)
    return fail(SALT_BAD_ARG, "conv geometry: ic,h_in,w_in,oc,k,s must be >= 1 and p >= 0");
  if (d->h_in + d->p > 32000 || d->w_in + d->p > 32000)
    return fail(SALT_BAD_ARG, "conv input plane too large (h_in + p and w_in + p <= 32000)");
  p.h_out = (d->h_in + 2 * d->p - d->k) / d->s + 1;
  p.w_out = (d->w_in + 2 * d->p - d->k) / d->s + 1;
  if (d->h_in + 2 * d->p - d->k < 0 || p.h_out < 1 || p.w_out < 1)
    return fail(SALT_BAD_ARG, "conv geometry degenerates to an empty output plane");
  if (d->max_queue_len < 1) return fail(SALT_BAD_ARG, "max_queue_len must be >= 1");
  if (d->max_out_spikes < 1) return fail(SALT_BAD_ARG, "max_out_spikes must be >= 1");
  if (d->max_extra_steps < 0) return fail(SALT_BAD_ARG, "max_extra_steps must be >= 0");
  if (d->chunk_size < 1) return fail(SALT_BAD_ARG, "chunk_size must be >= 1");
  if (!(d->v_th > 0.0f) || d->v_th == INFINITY)
    return fail(SALT_BAD_ARG, "float conv: v_th must be a finite value > 0 (a threshold <= 0 "
                              "fires on identity columns)");
  p.n_sp = p.h_out * p.w_out;
  p.n_neurons = (int64_t)d->oc * p.n_sp;
  if (p.n_neurons > 0x7fffffffLL) return fail(SALT_BAD_ARG, "too many neurons");
  p.ncand = (d->k - 1) / d->s + 1;
  if (p.ncand > 16) return fail(SALT_BAD_ARG, "k / s too large (at most 16 candidates per axis)");
  p.nslots = p.ncand * p.ncand;
  int lpu = 1;
  while (lpu < d->oc && lpu < 32) lpu <<= 1;
  p.lpu = lpu;
  p.G = (d->oc + lpu - 1) / lpu;
  p.ocp = p.G * lpu;
  p.taps = d->ic * d->k * d->k;
  p.n_spk_chunks = (E + kConvGroup - 1) / kConvGroup;  // conv: per 32-event group
  p.base = (d->max_queue_len + d->chunk_size - 1) / d->chunk_size;
  const int64_t steps = (int64_t)p.base + d->max_extra_steps;
  if (steps > (1 << 30)) return fail(SALT_BAD_ARG, "too many scan steps");
  p.max_steps = (int32_t)steps;
  return SALT_OK;
}

struct FConvScratch {
  int32_t *stats, *s_total, *needed, *tail_total, *needed_extra, *oc_total, *chunk;
  int32_t *vkey_max, *vkey_min, *tail_cnt, *hist;
  size_t stats_bytes;
  uint32_t* sw;
  float* wT;
};

static size_t float_conv_carve(const salt_float_conv_desc* d, const FConvPlan& p, int32_t B,
                               int32_t E, void* ws, FConvScratch& s) {
  Carver c(ws);
  const size_t nstat = (size_t)B * 4 + (size_t)B * d->oc + (size_t)B * p.n_spk_chunks;
  s.stats = c.take<int32_t>(nstat);
  s.stats_bytes = nstat * 4;
  if (s.stats) {
    s.s_total = s.stats;
    s.needed = s.stats + B;
    s.tail_total = s.stats + 2 * B;
    s.needed_extra = s.stats + 3 * B;
    s.oc_total = s.stats + 4 * B;
    s.chunk = s.oc_total + (size_t)B * d->oc;
  }
  s.vkey_max = c.take<int32_t>((size_t)B * d->oc);
  s.vkey_min = c.take<int32_t>((size_t)B * d->oc);
  s.sw = c.take<uint32_t>((size_t)B * E * p.nslots * p.G);
  s.tail_cnt = c.take<int32_t>((size_t)B * p.n_neurons);
  s.hist = c.take<int32_t>((size_t)B * 2 * p.n_sp);
  s.wT = c.take<float>((size_t)p.taps * p.ocp);
  return c.size();
}

salt_status salt_float_conv_layer_workspace_size(const salt_float_conv_desc* layer, int32_t batch,
                                                 int32_t in_capacity, size_t* bytes) {
  if (!bytes || batch < 1 || in_capacity < 1) return fail(SALT_BAD_ARG, "bad batch/capacity");
  FConvPlan p;
  salt_status rc = plan_float_conv(layer, in_capacity, p);
  if (rc) return rc;
  FConvScratch s;
  *bytes = float_conv_carve(layer, p, batch, in_capacity, nullptr, s);
  return SALT_OK;
}

salt_status salt_float_conv_layer_forward(const salt_float_conv_desc* d, const float* w,
                                          float decay_base, int32_t B, const salt_stream_in* in,
                                          const float* in_gain, salt_stream_out* out,
                                          float* v_final, const salt_float_conv_stats* stats,
                                          const salt_float_trace* trace, void* ws,
                                          size_t ws_bytes, void* stream) {
  salt_status rc = check_stream_in(in, B);
  if (rc) return rc;
  if (!w || !out || !out->times || !out->src || !out->n_real || !v_final)
    return fail(SALT_BAD_ARG, "float conv layer: NULL parameter or output pointer");
  if (!(decay_base > 0.0f) || decay_base > 1.0f)
    return fail(SALT_BAD_ARG, "float conv: decay_base must be in (0, 1] (tau >= 1)");
  if (trace && ((trace->v_max == nullptr) != (trace->v_min == nullptr)))
    return fail(SALT_BAD_ARG, "float conv trace: v_max and v_min go together");
  const int32_t E = in->capacity;
  FConvPlan p;
  if ((rc = plan_float_conv(d, E, p))) return rc;
  FConvScratch s;
  const size_t need = float_conv_carve(d, p, B, E, nullptr, s);
  if (!ws || ws_bytes < need) return fail(SALT_WORKSPACE_TOO_SMALL, "float conv workspace too small");
  if (reinterpret_cast<uintptr_t>(ws) & 255) return fail(SALT_BAD_ARG, "workspace not 256-byte aligned");
  float_conv_carve(d, p, B, E, ws, s);
  cudaStream_t st = (cudaStream_t)stream;

  ConvLaunch L;
  memset(&L, 0, sizeof(L));
  L.ic = d->ic; L.h_in = d->h_in; L.w_in = d->w_in; L.hw_in = d->h_in * d->w_in;
  L.oc = d->oc; L.k = d->k; L.s = d->s; L.p = d->p;
  L.h_out = p.h_out; L.w_out = p.w_out; L.n_sp = p.n_sp; L.n_neurons = p.n_neurons;
  L.ncand = p.ncand; L.nslots = p.nslots;
  L.L = d->max_queue_len; L.M = d->max_out_spikes; L.max_extra = d->max_extra_steps;
  L.lpu = p.lpu; L.G = p.G; L.ocp = p.ocp;
  L.tile_h = p.h_out; L.tile_w = p.w_out; L.tiles_x = 1; L.T = 1;
  L.fd_hw = FastDiv((uint32_t)(d->h_in * d->w_in));
  L.fd_w = FastDiv((uint32_t)d->w_in);
  L.fd_s = FastDiv((uint32_t)d->s);
  L.fd_G = FastDiv((uint32_t)p.G);
  L.fd_tw = FastDiv((uint32_t)p.w_out);
  L.in.times = in->times; L.in.src = in->src; L.in.capacity = E; L.in.virtual_pads = in->virtual_pads;
  L.in_nreal = in->n_real; L.batch = B;
  L.sw = s.sw; L.sw_stride = (int64_t)E * p.nslots * p.G;
  L.chunk_spikes = s.chunk; L.chunk_off = s.chunk; L.n_spk_chunks = p.n_spk_chunks;
  L.s_total = s.s_total; L.oc_total = s.oc_total; L.needed = s.needed;
  L.tail_total = s.tail_total; L.tail_mode = 1; L.tail_cnt = s.tail_cnt;

  FConvArgs X;
  memset(&X, 0, sizeof(X));
  X.wT = s.wT; X.gain = in_gain; X.base = decay_base; X.v_th = d->v_th;
  X.C = d->chunk_size; X.max_steps = p.max_steps; X.base_steps = p.base;
  X.v_final = v_final; X.needed_extra = s.needed_extra;
  float *v_max = nullptr, *v_min = nullptr;
  if (trace) {
    X.v_steps = trace->v_steps; X.event_ms = trace->event_ms; X.spike_mask = trace->spike_mask;
    if (trace->v_max) {
      X.vkey_max = s.vkey_max; X.vkey_min = s.vkey_min;
      v_max = trace->v_max; v_min = trace->v_min;
    }
  }
  SALT_CUDA(cudaMemsetAsync(s.stats, 0, s.stats_bytes, st));
  if (v_max) {  // keys below / above every finite float: 0x80808080 and 0x7f7f7f7f
    SALT_CUDA(cudaMemsetAsync(s.vkey_max, 0x80, sizeof(int32_t) * (size_t)B * d->oc, st));
    SALT_CUDA(cudaMemsetAsync(s.vkey_min, 0x7f, sizeof(int32_t) * (size_t)B * d->oc, st));
  }
  SALT_CUDA(float_conv_launch(L, X, w, s.wT, out->n_real, stats, v_max, v_min, st));
  g_launches += 3;
  spike_chunk_scan<<<(B * 32 + 255) / 256, 256, 0, st>>>(s.chunk, p.n_spk_chunks, B, nullptr);
  SALT_LAUNCHED("spike_chunk_scan");
  {
    salt_stream_out so = *out;
    void* cargs[] = {&L, &so};
    SALT_CUDA(cudaLaunchKernel(conv_compact_kernel(p.ncand, p.G, L.addr_table != nullptr),
                               dim3(conv_compact_blocks(p.n_spk_chunks, B), B),
                               dim3(kCompactThreads), cargs, 0, st));
  }
  SALT_LAUNCHED("conv_compact");
  conv_tail_append<<<B, kCompactThreads, 0, st>>>(L, *out);
  SALT_LAUNCHED("conv_tail_append");
  conv_truncated<<<B, kTruncThreads, 0, st>>>(L, *out, s.hist);
  SALT_LAUNCHED("conv_truncated");
  return SALT_OK;
}

salt_status salt_float_fc_layer_trace(const salt_float_fc_desc* d, const float* w,
                                      const float* decay_base, int32_t B,
                                      const salt_stream_in* in, const float* in_gain,
                                      float* v_final, const salt_float_trace* trace,
                                      void* stream) {
  salt_status rc = check_float(d);
  if (rc) return rc;
  if ((rc = check_stream_in(in, B))) return rc;
  if (!w || !decay_base) return fail(SALT_BAD_ARG, "float fc trace: NULL weights or decay base");
  if (trace && ((trace->v_max == nullptr) != (trace->v_min == nullptr)))
    return fail(SALT_BAD_ARG, "float fc trace: v_max and v_min go together");
  const int64_t steps = (int64_t)(in->capacity + d->chunk_size - 1) / d->chunk_size +
                        d->max_extra_steps;
  if (steps > (1 << 30)) return fail(SALT_BAD_ARG, "too many scan steps");
  FTraceArgs T;
  memset(&T, 0, sizeof(T));
  T.n_in = d->n_in; T.n_out = d->n_out; T.C = d->chunk_size; T.max_steps = (int32_t)steps;
  T.batch = B; T.v_th = d->v_th;
  T.in.times = in->times; T.in.src = in->src; T.in.capacity = in->capacity;
  T.in.virtual_pads = in->virtual_pads; T.in_nreal = in->n_real;
  T.w = w; T.decay_base = decay_base; T.gain = in_gain; T.v_final = v_final;
  if (trace) {
    T.v_max = trace->v_max; T.v_min = trace->v_min; T.v_steps = trace->v_steps;
    T.event_ms = trace->event_ms; T.spike_mask = trace->spike_mask;
  }
  SALT_CUDA(float_fc_trace_launch(T, (cudaStream_t)stream));
  ++g_launches;
  return SALT_OK;
}

salt_status salt_float_fc_set_profiling(int32_t enable) {
  g_fprof.on = enable != 0;
  return SALT_OK;
}

salt_status salt_float_fc_profile_read(float* segment_ms, float* layer_ms, int32_t* layers,
                                       int32_t reset) {
  auto drain = [](std::vector<cudaEvent_t>& v, double& acc) -> cudaError_t {
    for (size_t i = 0; i + 1 < v.size(); i += 2) {
      cudaError_t e = cudaEventSynchronize(v[i + 1]);
      if (e != cudaSuccess) return e;
      float ms = 0;
      e = cudaEventElapsedTime(&ms, v[i], v[i + 1]);
      if (e != cudaSuccess) return e;
      acc += ms;
    }
    for (cudaEvent_t e : v) cudaEventDestroy(e);
    v.clear();
    return cudaSuccess;
  };
  const int32_t added = (int32_t)(g_fprof.layer.size() / 2);
  SALT_CUDA(drain(g_fprof.seg, g_fprof.seg_ms));
  SALT_CUDA(drain(g_fprof.layer, g_fprof.layer_ms));
  g_fprof.n += added;
  if (segment_ms) *segment_ms = (float)g_fprof.seg_ms;
  if (layer_ms) *layer_ms = (float)g_fprof.layer_ms;
  if (layers) *layers = g_fprof.n;
  if (reset) {
    g_fprof.seg_ms = g_fprof.layer_ms = 0;
    g_fprof.n = 0;
  }
  return SALT_OK;
}

salt_status salt_fc_layer_workspace_size(const salt_fc_desc* layer, const salt_quant_desc* quant,
                                         int32_t batch, int32_t in_capacity, size_t* bytes) {
  salt_status rc = check_quant(quant);
  if (rc) return rc;
  if ((rc = check_fc(layer))) return rc;
  if (!bytes || batch < 1 || in_capacity < 1) return fail(SALT_BAD_ARG, "bad batch/capacity");
  FCScratch s;
  *bytes = fc_carve(layer, quant, batch, in_capacity, true, nullptr, s);
  return SALT_OK;
}

salt_status salt_fc_layer_forward(const salt_fc_desc* layer, const salt_quant_desc* quant,
                                  const int32_t* q, const int32_t* lut, const int32_t* vth,
                                  int32_t batch, const salt_stream_in* in, salt_stream_out* out,
                                  int32_t* v_final, const salt_layer_stats* stats, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  return fc_forward_impl(layer, quant, q, false, lut, vth, batch, in, out, v_final, stats,
                         workspace, workspace_bytes, (cudaStream_t)stream);
}

static salt_status dense_scan_impl(const salt_quant_desc* quant, int32_t n, int32_t L,
                                   const int32_t* a_int, const uint8_t* is_identity,
                                   const int32_t* q_int, const int32_t* vth, uint8_t* spike_mask,
                                   uint8_t* overflowed, int32_t* v_final, int32_t* vmin,
                                   int32_t* vmax, int32_t* v_steps, cudaStream_t stream) {
  salt_status rc = check_quant(quant);
  if (rc) return rc;
  if (n < 1 || L < 1 || !a_int || !is_identity || !q_int || !v_final || !vmin || !vmax ||
      (quant->has_vth && !vth))
    return fail(SALT_BAD_ARG, "dense scan: bad sizes or NULL pointers");
  dense_scan<<<(unsigned)((n + 127) / 128), 128, 0, stream>>>(
      make_qc(quant), n, L, a_int, is_identity, q_int, quant->has_vth ? vth : nullptr, spike_mask,
      overflowed, v_final, vmin, vmax, v_steps);
  SALT_LAUNCHED("dense_scan");
  return SALT_OK;
}

salt_status salt_quant_scan_dense(const salt_quant_desc* quant, int32_t n, int32_t L,
                                  const int32_t* a_int, const uint8_t* is_identity,
                                  const int32_t* q_int, const int32_t* vth, uint8_t* spike_mask,
                                  uint8_t* overflowed, int32_t* v_final, int32_t* vmin,
                                  int32_t* vmax, void* stream) {
  return dense_scan_impl(quant, n, L, a_int, is_identity, q_int, vth, spike_mask, overflowed,
                         v_final, vmin, vmax, nullptr, (cudaStream_t)stream);
}

salt_status salt_quant_scan_dense_trace(const salt_quant_desc* quant, int32_t n, int32_t L,
                                        const int32_t* a_int, const uint8_t* is_identity,
                                        const int32_t* q_int, const int32_t* vth,
                                        uint8_t* spike_mask, uint8_t* overflowed,
                                        int32_t* v_final, int32_t* vmin, int32_t* vmax,
                                        int32_t* v_steps, void* stream) {
  if (!v_steps) return fail(SALT_BAD_ARG, "dense scan trace: v_steps is NULL");
  return dense_scan_impl(quant, n, L, a_int, is_identity, q_int, vth, spike_mask, overflowed,
                         v_final, vmin, vmax, v_steps, (cudaStream_t)stream);
}

// ---------------------------------------------------------------- network plan

static int q_bits_of(const int32_t* q, int64_t n) {
  int bits = 8;
  for (int64_t i = 0; i < n; ++i) {
    if (q[i] < -32768 || q[i] > 32767) return 32;
    if (q[i] < -128 || q[i] > 127) bits = 16;
  }
  return bits;
}

salt_status salt_network_create(const salt_layer_spec* layers, int32_t n_layers,
                                salt_network** out) {
  if (!layers || n_layers < 1 || !out) return fail(SALT_BAD_ARG, "network: no layers");
  auto* net = new salt_network();
  for (int l = 0; l < n_layers; ++l) {
    LayerRec r;
    r.spec = layers[l];
    salt_quant_desc& qd = r.spec.quant;
    salt_status rc = check_quant(&qd);
    int64_t nq = 0, nvth = 0;
    if (!rc && r.spec.kind == 0) {
      ConvPlan p;
      rc = plan_conv(&r.spec.conv, &qd, 1, 1, p);
      nq = (int64_t)r.spec.conv.oc * r.spec.conv.ic * r.spec.conv.k * r.spec.conv.k;
      nvth = p.n_neurons;
      r.n_neurons = p.n_neurons;
      r.M = r.spec.conv.max_out_spikes;
    } else if (!rc && r.spec.kind == 1) {
      rc = check_fc(&r.spec.fc);
      nq = (int64_t)r.spec.fc.n_in * r.spec.fc.n_out;
      nvth = r.spec.fc.n_out;
      r.n_neurons = r.spec.fc.n_out;
      r.M = r.spec.fc.max_out_spikes;
    } else if (!rc) {
      rc = fail(SALT_BAD_ARG, "layer kind must be 0 (conv) or 1 (fc)");
    }
    if (!rc && (!r.spec.q_host || (qd.lut_len > 0 && !r.spec.lut_host) ||
                (qd.has_vth && !r.spec.vth_host)))
      rc = fail(SALT_BAD_ARG, "network: NULL host parameter pointer");
    if (rc) {
      salt_network_destroy(net);
      return rc;
    }
    qd.q_bits = q_bits_of(r.spec.q_host, nq);
    bool tail = false;
    if (qd.has_vth)
      for (int64_t i = 0; i < nvth; ++i) tail |= r.spec.vth_host[i] <= 0;
    for (int i = 0; i < qd.lut_len; ++i)
      tail |= r.spec.lut_host[i] < 0 || r.spec.lut_host[i] >= (1 << qd.f_a);
    qd.needs_tail = qd.needs_tail || tail;
    std::vector<int32_t> qbuf(r.spec.q_host, r.spec.q_host + nq);
    if (r.spec.kind == 1) {  // store FC weights transposed: (n_in, n_out)
      const int n_in = r.spec.fc.n_in, n_out = r.spec.fc.n_out;
      for (int o = 0; o < n_out; ++o)
        for (int i = 0; i < n_in; ++i) qbuf[(int64_t)i * n_out + o] = r.spec.q_host[(int64_t)o * n_in + i];
    }
    cudaError_t e = cudaMalloc(&r.d_q, sizeof(int32_t) * std::max<int64_t>(nq, 1));
    if (e == cudaSuccess)
      e = cudaMemcpy(r.d_q, qbuf.data(), sizeof(int32_t) * nq, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && qd.lut_len > 0) {
      e = cudaMalloc(&r.d_lut, sizeof(int32_t) * qd.lut_len);
      if (e == cudaSuccess)
        e = cudaMemcpy(r.d_lut, r.spec.lut_host, sizeof(int32_t) * qd.lut_len,
                       cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess && qd.has_vth) {
      e = cudaMalloc(&r.d_vth, sizeof(int32_t) * nvth);
      if (e == cudaSuccess)
        e = cudaMemcpy(r.d_vth, r.spec.vth_host, sizeof(int32_t) * nvth, cudaMemcpyHostToDevice);
    }
    r.spec.q_host = r.spec.lut_host = r.spec.vth_host = nullptr;
    net->layers.push_back(r);
    if (e != cudaSuccess) {
      salt_network_destroy(net);
      return fail(SALT_CUDA_ERROR, std::string("network parameter upload: ") + cudaGetErrorString(e));
    }
  }
  *out = net;
  return SALT_OK;
}

salt_status salt_network_destroy(salt_network* net) {
  if (!net) return SALT_OK;
  for (auto& t : net->timed) net->pool.push_back(t.ev);
  for (auto& e : net->pool) {
    cudaEventDestroy(e.start);
    cudaEventDestroy(e.stop);
  }
  for (auto& r : net->layers) {
    cudaFree(r.d_q);
    cudaFree(r.d_lut);
    cudaFree(r.d_vth);
  }
  delete net;
  return SALT_OK;
}

struct NetLayout {
  float* st_t[2];
  int32_t* st_s[2];
  int32_t* st_n[2];
  int32_t* vtmp;
  int32_t* stats;  // 6 * n_layers * B
  void* scratch;
  size_t scratch_bytes, total;
};

static salt_status net_layout(const salt_network* net, int32_t B, int32_t E0, void* ws,
                              NetLayout& o) {
  const int nl = (int)net->layers.size();
  // every layer writes its output stream into the ping-pong buffers, the last one too (a firing
  // last layer compacts up to its max_out_spikes per sample); v_final of all but the last layer
  // goes to vtmp (the last one's is the logits)
  int32_t maxM = 1;
  int64_t maxN = 1;
  for (int l = 0; l < nl; ++l) maxM = std::max(maxM, net->layers[l].M);
  for (int l = 0; l + 1 < nl; ++l) maxN = std::max(maxN, net->layers[l].n_neurons);
  size_t scratch = 0;
  int32_t E = E0;
  for (int l = 0; l < nl; ++l) {
    const LayerRec& r = net->layers[l];
    size_t b = 0;
    if (r.spec.kind == 0) {
      salt_status rc = conv_scratch_bytes(&r.spec.conv, &r.spec.quant, B, E, b);
      if (rc) return rc;
    } else {
      FCScratch s;
      b = fc_carve(&r.spec.fc, &r.spec.quant, B, E, false, nullptr, s);
    }
    scratch = std::max(scratch, b);
    E = r.M;
  }
  Carver c(ws);
  for (int i = 0; i < 2; ++i) {
    o.st_t[i] = c.take<float>((size_t)B * maxM);
    o.st_s[i] = c.take<int32_t>((size_t)B * maxM);
    o.st_n[i] = c.take<int32_t>((size_t)B);
  }
  o.vtmp = c.take<int32_t>((size_t)B * maxN);
  o.stats = c.take<int32_t>((size_t)6 * nl * B);
  o.scratch = c.take<char>(scratch);
  o.scratch_bytes = scratch;
  o.total = c.size();
  return SALT_OK;
}

salt_status salt_network_workspace_size(const salt_network* net, int32_t batch,
                                        int32_t in_capacity, size_t* bytes) {
  if (!net || !bytes || batch < 1 || in_capacity < 1)
    return fail(SALT_BAD_ARG, "network workspace: bad arguments");
  NetLayout o;
  salt_status rc = net_layout(net, batch, in_capacity, nullptr, o);
  if (rc) return rc;
  *bytes = o.total;
  return SALT_OK;
}

// Layers [l0, l1) of a batch-`batch` forward on rows [row0, row0 + rows).  Layer l0 reads `in`
// (those rows only) when l0 == 0, else the workspace stream layer l0 - 1 left for these rows;
// outputs and per-layer stats land at the rows' places in the full-batch arrays.  When l1 is the
// last layer, fits (AND over all layers) is written for the rows.
static salt_status network_run(salt_network* net, int32_t batch, int32_t in_capacity,
                               int32_t row0, int32_t rows, int32_t l0, int32_t l1,
                               const salt_stream_in* in, int32_t* logits,
                               int32_t* spike_count, int32_t* overflowed, int32_t* vmin,
                               int32_t* vmax, int32_t* needed_queue, int32_t* fits,
                               void* workspace, size_t workspace_bytes, cudaStream_t st) {
  const int nl = (int)net->layers.size();
  if (!logits && l1 == nl) return fail(SALT_BAD_ARG, "network forward: NULL logits");
  if (batch < 1 || row0 < 0 || rows < 1 || row0 + rows > batch || l0 < 0 || l1 > nl || l0 >= l1)
    return fail(SALT_BAD_ARG, "network forward: bad row or layer range");
  if (l0 == 0) {
    salt_status rc = check_stream_in(in, rows);
    if (rc) return rc;
    if (in->capacity != in_capacity)
      return fail(SALT_BAD_ARG, "network forward: input capacity differs from the planned one");
  }
  if (in_capacity < 1) return fail(SALT_BAD_ARG, "network forward: in_capacity must be >= 1");
  // the workspace layout depends only on the full batch and the first layer's input capacity
  NetLayout o;
  salt_status rc = net_layout(net, batch, in_capacity, nullptr, o);
  if (rc) return rc;
  if (!workspace || workspace_bytes < o.total)
    return fail(SALT_WORKSPACE_TOO_SMALL, "network workspace too small");
  net_layout(net, batch, in_capacity, workspace, o);
  const int64_t launches0 = g_launches;
  const int B = batch;
  salt_stream_in cur{};
  if (l0 == 0) {
    cur = *in;
  } else {
    const LayerRec& prev = net->layers[l0 - 1];
    cur.times = o.st_t[(l0 - 1) & 1] + (size_t)row0 * prev.M;
    cur.src = o.st_s[(l0 - 1) & 1] + (size_t)row0 * prev.M;
    cur.n_real = o.st_n[(l0 - 1) & 1] + row0;
    cur.capacity = prev.M;
    cur.virtual_pads = 1;
  }
  for (int l = l0; l < l1; ++l) {
    LayerRec& r = net->layers[l];
    const bool last = l == nl - 1;
    salt_stream_out so{o.st_t[l & 1] + (size_t)row0 * r.M, o.st_s[l & 1] + (size_t)row0 * r.M,
                       o.st_n[l & 1] + row0};
    int32_t* vf = last ? logits + (size_t)row0 * r.n_neurons : o.vtmp + (size_t)row0 * r.n_neurons;
    int32_t* sb = o.stats + (size_t)6 * l * B + row0;
    auto at = [&](int32_t* a) { return a ? a + (size_t)l * B + row0 : nullptr; };
    salt_layer_stats ls{spike_count ? at(spike_count) : sb, needed_queue ? at(needed_queue) : sb + B,
                        overflowed ? at(overflowed) : sb + 2 * B, vmin ? at(vmin) : sb + 3 * B,
                        vmax ? at(vmax) : sb + 4 * B, sb + 5 * B};
    KernelTimer timer, whole;
    auto take = [&](KernelTimer& t) -> salt_status {
      if (net->pool.empty()) {
        SALT_CUDA(cudaEventCreate(&t.start));
        SALT_CUDA(cudaEventCreate(&t.stop));
      } else {
        t = net->pool.back();
        net->pool.pop_back();
      }
      return SALT_OK;
    };
    if (net->profiling) {
      if ((rc = take(whole))) return rc;
      net->timed.push_back({l, 1, whole});
      SALT_CUDA(cudaEventRecord(whole.start, st));
      if (r.spec.kind == 0) {
        if ((rc = take(timer))) return rc;
        net->timed.push_back({l, 0, timer});
      }
    }
    if (r.spec.kind == 0)
      rc = conv_forward_impl(&r.spec.conv, &r.spec.quant, r.d_q, r.d_lut, r.d_vth, rows, &cur,
                             &so, vf, &ls, o.scratch, o.scratch_bytes, st,
                             timer.start ? &timer : nullptr);
    else
      rc = fc_forward_impl(&r.spec.fc, &r.spec.quant, r.d_q, true, r.d_lut, r.d_vth, rows, &cur,
                           &so, vf, &ls, o.scratch, o.scratch_bytes, st);
    if (rc) return rc;
    if (whole.stop) SALT_CUDA(cudaEventRecord(whole.stop, st));
    cur.times = so.times;
    cur.src = so.src;
    cur.n_real = so.n_real;
    cur.capacity = r.M;
    cur.virtual_pads = 1;
  }
  if (fits && l1 == nl) {  // per-layer fits sit at offset 5*B of each layer's (6, B) stats block
    fits_and<<<(rows + 255) / 256, 256, 0, st>>>(o.stats + 5 * B + row0, nl, (int64_t)6 * B, rows,
                                                 fits + row0);
    SALT_LAUNCHED("fits_and");
  }
  net->last_launches = (int32_t)(g_launches - launches0);
  return SALT_OK;
}

salt_status salt_network_forward(salt_network* net, int32_t batch, const salt_stream_in* in,
                                 int32_t* logits, int32_t* spike_count, int32_t* overflowed,
                                 int32_t* vmin, int32_t* vmax, int32_t* needed_queue,
                                 int32_t* fits, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  if (!net || !logits) return fail(SALT_BAD_ARG, "network forward: NULL network or logits");
  if (!in) return fail(SALT_BAD_ARG, "input stream pointers must be non-NULL");
  return network_run(net, batch, in->capacity, 0, batch, 0, (int32_t)net->layers.size(), in,
                     logits,
                     spike_count, overflowed, vmin, vmax, needed_queue, fits, workspace,
                     workspace_bytes, (cudaStream_t)stream);
}

salt_status salt_network_forward_part(salt_network* net, int32_t batch, int32_t in_capacity,
                                      int32_t row0, int32_t rows, int32_t layer_begin,
                                      int32_t layer_end, const salt_stream_in* in,
                                      int32_t* logits, int32_t* spike_count, int32_t* overflowed,
                                      int32_t* vmin, int32_t* vmax, int32_t* needed_queue,
                                      int32_t* fits, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  if (!net) return fail(SALT_BAD_ARG, "network forward: NULL network");
  return network_run(net, batch, in_capacity, row0, rows, layer_begin, layer_end, in, logits,
                     spike_count,
                     overflowed, vmin, vmax, needed_queue, fits, workspace, workspace_bytes,
                     (cudaStream_t)stream);
}

int32_t salt_network_last_launch_count(const salt_network* net) {
  return net ? net->last_launches : 0;
}

salt_status salt_network_set_profiling(salt_network* net, int32_t enable) {
  if (!net) return fail(SALT_BAD_ARG, "NULL network");
  net->profiling = enable != 0;
  return SALT_OK;
}

salt_status salt_network_profile_read(salt_network* net, float* fused_ms, float* layer_ms,
                                      int32_t* launches, int32_t reset) {
  if (!net || !fused_ms || !layer_ms || !launches)
    return fail(SALT_BAD_ARG, "profile_read: NULL argument");
  const size_t nl = net->layers.size();
  for (size_t l = 0; l < nl; ++l) {
    fused_ms[l] = 0.0f;
    layer_ms[l] = 0.0f;
    launches[l] = 0;
  }
  for (auto& t : net->timed) {
    SALT_CUDA(cudaEventSynchronize(t.ev.stop));
    float ms = 0.0f;
    SALT_CUDA(cudaEventElapsedTime(&ms, t.ev.start, t.ev.stop));
    if (t.whole_layer) {
      layer_ms[t.layer] += ms;
      launches[t.layer] += 1;
    } else {
      fused_ms[t.layer] += ms;
    }
  }
  if (reset) {
    for (auto& t : net->timed) net->pool.push_back(t.ev);
    net->timed.clear();
  }
  return SALT_OK;
}


}  // extern "C"
