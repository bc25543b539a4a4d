// Integer conv layer pipeline for B200 (sm_100a).
//
// Replaces, for a batch of samples, ConvLayer.forward with QuantBackend
// (salt_core/layers/conv.py:124-149): queue construction (connectivity/conv.py:128-172), the
// integer LIF scan over every queue column (quant/scan.py:97-132), spike compaction into the
// next EventStream (stream.py:24-64, :84-100) and the layer diagnostics (layers/base.py:73-79).
//
// Kernels (one launch each, all on the caller's stream):
//   conv_tile_count / conv_tile_scan_offsets / conv_tile_scatter
//        only when the output plane is split into several tiles: a stable partition of each
//        sample's events by the tiles their receptive-field candidates fall in.
//   conv_fused   one block per (tile, sample).  Streams the tile's events in arrival order in
//        chunks.  Per chunk it buckets the candidates by output position into per-position
//        bitmasks (one word per warp of events, built with match_any, so every position's
//        queue comes out in global event order: the stable (position, j) order of conv.py:71);
//        then lane groups (one lane per output channel) run their position's integer
//        recurrence over the chunk.  Spikes are recorded as per-(event, candidate slot) channel
//        bitmasks ("spike words"), staged in shared memory and written out once per chunk.
//   conv_compact       per (event chunk, sample): emits spikes in (event, neuron) order — the
//        stable sort of stream.py:40 — into the output stream.
//   conv_tail_append / conv_truncated   rare paths: spikes on catch-up/identity columns
//        (only possible when some v_th_int <= 0 or a decay code is out of range) and samples
//        whose spike count exceeds max_out_spikes (the first max_out spikes in neuron-major
//        order are kept, stream.py:60, then sorted by event).
#include "salt_layers.cuh"

namespace salt {

// ------------------------------------------------------------------ schedule

// Samples by decreasing event count: a stable-enough counting sort over 1024 bins of
// min(n_real, capacity) (ties in any order; only the block schedule depends on it).
__global__ void __launch_bounds__(kOrderThreads)
sample_order_desc(const int32_t* __restrict__ n_real, int32_t capacity, int32_t batch,
                  int32_t* __restrict__ order) {
  __shared__ int32_t bins[kOrderThreads];
  __shared__ int32_t s_scan[kScanSmem];
  const int tid = threadIdx.x;
  bins[tid] = 0;
  __syncthreads();
  auto bin_of = [&](int b) {
    const int32_t n = min(max(n_real[b], 0), capacity);
    const int bin = (int)(((int64_t)n * (kOrderThreads - 1)) / max(capacity, 1));
    return kOrderThreads - 1 - bin;  // heaviest first
  };
  for (int b = tid; b < batch; b += blockDim.x) atomicAdd(&bins[bin_of(b)], 1);
  __syncthreads();
  int32_t total;
  const int32_t off = block_exclusive_scan(bins[tid], s_scan, total);
  bins[tid] = off;
  __syncthreads();
  for (int b = tid; b < batch; b += blockDim.x) order[atomicAdd(&bins[bin_of(b)], 1)] = b;
}

// ------------------------------------------------------------------ tile partition

// Partition chunks of a sample that hold real events; chunks past them are neither counted
// nor scanned.  Blocks of a sample loop over its chunks (grid x = blocks per sample).
__device__ __forceinline__ int32_t part_chunks(const ConvLaunch& P, int b) {
  return (P.n_eff(b) + kPartChunk - 1) / kPartChunk;
}

// The kPartPer events of a thread in partition chunk ch, decoded (empty ranges past n_eff).  The
// source loads are issued together so that their latencies overlap.
__device__ __forceinline__ void part_events(const ConvLaunch& P, int b, int ch, int32_t n_eff,
                                            EvCand (&k)[kPartPer]) {
  int32_t src[kPartPer];
#pragma unroll
  for (int i = 0; i < kPartPer; ++i) {
    const int32_t jj = ch * kPartChunk + i * kPartThreads + (int)threadIdx.x;
    src[i] = jj < n_eff ? P.in.src[(int64_t)b * P.in.capacity + jj] : 0;
  }
#pragma unroll
  for (int i = 0; i < kPartPer; ++i) {
    const int32_t jj = ch * kPartChunk + i * kPartThreads + (int)threadIdx.x;
    int32_t c, y, x;
    k[i] = event_cand(P, src[i], c, y, x);
    if (jj >= n_eff) k[i] = EvCand{0, 1, 0, 0, 1, 0};
  }
}

// Tile rows and columns an event's valid candidates reach (an empty range for empty events).
struct TileRange {
  int32_t ty0, ty1, tx0, tx1;
};
__device__ __forceinline__ TileRange tile_range(const ConvLaunch& P, const EvCand& k) {
  if (k.empty()) return TileRange{1, 0, 1, 0};
  return TileRange{(int32_t)P.fd_th.div(k.oy_lo), (int32_t)P.fd_th.div(k.oy_hi),
                   (int32_t)P.fd_tw.div(k.ox_lo), (int32_t)P.fd_tw.div(k.ox_hi)};
}

__global__ void __launch_bounds__(kPartThreads)
conv_tile_count(ConvLaunch P, int32_t* __restrict__ counts) {
  extern __shared__ int32_t s_cnt[];
  const int b = blockIdx.y;
  const int32_t n_eff = P.n_eff(b), nch = part_chunks(P, b);
  for (int ch = blockIdx.x; ch < nch; ch += gridDim.x) {
    for (int t = threadIdx.x; t < P.T; t += blockDim.x) s_cnt[t] = 0;
    __syncthreads();
    EvCand k[kPartPer];
    part_events(P, b, ch, n_eff, k);
#pragma unroll
    for (int i = 0; i < kPartPer; ++i) {
      if (k[i].empty()) continue;
      for (int ty = (int)P.fd_th.div(k[i].oy_lo), ty1 = (int)P.fd_th.div(k[i].oy_hi); ty <= ty1; ++ty)
        for (int tx = (int)P.fd_tw.div(k[i].ox_lo), tx1 = (int)P.fd_tw.div(k[i].ox_hi); tx <= tx1; ++tx)
          atomicAdd(&s_cnt[ty * P.tiles_x + tx], 1);
    }
    __syncthreads();
    for (int t = threadIdx.x; t < P.T; t += blockDim.x)
      counts[((int64_t)b * P.n_part_chunks + ch) * P.T + t] = s_cnt[t];
    __syncthreads();
  }
}

// One warp per sample: turns the per-(chunk, tile) counts into absolute offsets inside the
// sample's list region (tile-major, chunks in arrival order) and records each tile's length.
__global__ void conv_tile_scan_offsets(ConvLaunch P, int32_t* __restrict__ counts,
                                       int32_t* __restrict__ tile_len,
                                       int32_t* __restrict__ tile_off) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= P.batch) return;
  const int b = warp;
  const int32_t nch = part_chunks(P, b);
  int32_t tile_base = 0;
  for (int t = 0; t < P.T; ++t) {
    int32_t carry = 0;
    for (int base = 0; base < nch; base += 32) {
      const int c = base + lane;
      const int64_t idx = ((int64_t)b * P.n_part_chunks + c) * P.T + t;
      const int32_t v = c < nch ? counts[idx] : 0;
      int32_t incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (c < nch) counts[idx] = tile_base + carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      tile_len[(int64_t)b * P.T + t] = carry;
      tile_off[(int64_t)b * P.T + t] = tile_base;
    }
    tile_base += carry;
  }
}

__global__ void __launch_bounds__(kPartThreads)
conv_tile_scatter(ConvLaunch P, const int32_t* __restrict__ counts, int32_t* __restrict__ lists) {
  // [T][kPartChunk/32] masks, then the word prefix [T][kPartChunk/32], then the chunk's [T] bases
  extern __shared__ uint32_t s_mask[];
  constexpr int W = kPartChunk / 32;
  static_assert(W == 32, "one warp scans one tile's words");
  uint32_t* s_pre = s_mask + P.T * W;
  int32_t* s_base = reinterpret_cast<int32_t*>(s_pre + P.T * W);
  const int b = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int32_t n_eff = P.n_eff(b), nch = part_chunks(P, b);
  int32_t* list_b = lists + (int64_t)b * P.list_stride;
  for (int ch = blockIdx.x; ch < nch; ch += gridDim.x) {
    for (int i = threadIdx.x; i < P.T * W; i += blockDim.x) s_mask[i] = 0;
    __syncthreads();
    TileRange r[kPartPer];  // kept in registers for the write pass
    {
      EvCand k[kPartPer];
      part_events(P, b, ch, n_eff, k);
#pragma unroll
      for (int i = 0; i < kPartPer; ++i) r[i] = tile_range(P, k[i]);
    }
#pragma unroll
    for (int i = 0; i < kPartPer; ++i) {
      const int e = i * kPartThreads + (int)threadIdx.x;
      for (int ty = r[i].ty0; ty <= r[i].ty1; ++ty)
        for (int tx = r[i].tx0; tx <= r[i].tx1; ++tx)
          atomicOr(&s_mask[(ty * P.tiles_x + tx) * W + (e >> 5)], 1u << (e & 31));
    }
    __syncthreads();
    for (int t = warp; t < P.T; t += nwarps) {  // word prefix per tile: one warp scan per tile
      const int32_t v = __popc(s_mask[t * W + lane]);
      int32_t incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      s_pre[t * W + lane] = (uint32_t)(incl - v);
    }
    for (int t = threadIdx.x; t < P.T; t += blockDim.x)
      s_base[t] = counts[((int64_t)b * P.n_part_chunks + ch) * P.T + t];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPartPer; ++i) {
      const int e = i * kPartThreads + (int)threadIdx.x;
      const int32_t jj = ch * kPartChunk + e;
      for (int ty = r[i].ty0; ty <= r[i].ty1; ++ty)
        for (int tx = r[i].tx0; tx <= r[i].tx1; ++tx) {
          const int t = ty * P.tiles_x + tx;
          const uint32_t m = s_mask[t * W + (e >> 5)] & ((1u << (e & 31)) - 1u);
          const int32_t rank = (int32_t)(s_pre[t * W + (e >> 5)] + __popc(m));
          list_b[s_base[t] + rank] = jj;
        }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ fused bucket + scan

// Shared-memory record of one chunk event (16 bytes: one vector load).
struct __align__(16) EvRec {
  float t;
  int32_t ckk;     // clamped channel * k * k (weight tap base)
  uint32_t yx;     // (y + p) << 16 | (x + p)
  uint32_t omin;   // (o_min_y + 32768) << 16 | (o_min_x + 32768)
};

// Shared-memory layout of conv_fused; the host sizes it with the same function.
struct FusedSmem {
  size_t w, lut, v, tprev, cnt, mask, ev, ej, sw, list, posoff, poscnt, act, park, vote, misc,
      total;
  __host__ __device__ FusedSmem(const ConvLaunch& P, int wt_bytes) {
    const size_t npm = (size_t)P.tile_h * P.tile_w;
    size_t o = 0;
    // weights [ic*k*k][ocp], then one zero row (the padding steps of the no-fit walk)
    w = o;     o += align16((size_t)(P.ic * P.k * P.k + 1) * P.ocp * wt_bytes);
    lut = o;   o += align16((size_t)(P.lut_in_smem ? P.qc.lut_len : 0) * 4);
    v = o;     o += align16(npm * P.ocp * 4);
    tprev = o; o += align16(npm * P.G * 4);   // one copy per (position, channel group)
    cnt = o;   o += align16(npm * P.G * 4);
    mask = o;  o += align16(npm * (kFusedChunk / 32) * 4);
    ev = o;    o += align16((size_t)kFusedChunk * sizeof(EvRec));
    ej = o;    o += align16((size_t)(P.T > 1 ? kFusedChunk : 0) * 4);
    sw = o;    o += align16((size_t)kFusedChunk * P.nslots * P.G * 4);
    list = o;  o += align16((size_t)kFusedChunk * P.nslots * 2);
    posoff = o; o += align16(npm * 4);
    poscnt = o; o += align16(npm * 4);
    act = o;   o += align16(npm * 4);
    // 32-lane groups park each batch's (decay code, weight row) pairs and step ballots per warp
    park = o;  o += align16((size_t)(P.lpu == 32 ? kFusedThreads : 0) * sizeof(int2));
    vote = o;  o += align16((size_t)(P.lpu == 32 ? kFusedThreads : 0) * 4);
    misc = o;  o += 64;
    total = o;
  }
};

size_t conv_fused_smem_bytes(const ConvLaunch& P, int wt_bytes) {
  return FusedSmem(P, wt_bytes).total;
}

// The 32-lane no-fit walk is held to 5 blocks per SM (48 registers; as many blocks as its shared
// memory allows at the benchmark sizes), which it would otherwise trade for registers; the other
// variants keep the compiler's choice (a minimum of 0 blocks sets no bound).
template <int LPU, int FORM>
constexpr int fused_min_blocks() { return (LPU == 32 && FORM == kStepWideNoFit) ? 5 : 0; }

template <typename WT, int LPU, bool SAT, int FORM>
__global__ void __launch_bounds__(kFusedThreads, fused_min_blocks<LPU, FORM>())
conv_fused(ConvLaunch P) {
  constexpr int UPW = 32 / LPU;  // units (position x channel group) per warp
  constexpr int CHW = kFusedChunk / 32;
  extern __shared__ __align__(16) uint8_t smem[];
  const FusedSmem L(P, sizeof(WT));
  WT* w_s = reinterpret_cast<WT*>(smem + L.w);
  int32_t* lut_s = reinterpret_cast<int32_t*>(smem + L.lut);
  int32_t* v_s = reinterpret_cast<int32_t*>(smem + L.v);
  float* tprev_s = reinterpret_cast<float*>(smem + L.tprev);
  int32_t* cnt_s = reinterpret_cast<int32_t*>(smem + L.cnt);
  uint32_t* mask_s = reinterpret_cast<uint32_t*>(smem + L.mask);
  EvRec* ev_s = reinterpret_cast<EvRec*>(smem + L.ev);
  int32_t* ej_s = reinterpret_cast<int32_t*>(smem + L.ej);
  uint32_t* sw_s = reinterpret_cast<uint32_t*>(smem + L.sw);
  uint16_t* list_s = reinterpret_cast<uint16_t*>(smem + L.list);
  int32_t* posoff_s = reinterpret_cast<int32_t*>(smem + L.posoff);
  int32_t* poscnt_s = reinterpret_cast<int32_t*>(smem + L.poscnt);
  int32_t* act_s = reinterpret_cast<int32_t*>(smem + L.act);
  __shared__ int32_t s_scan[kScanSmem];
  int32_t* misc_s = reinterpret_cast<int32_t*>(smem + L.misc);
  // 32-lane groups: per-warp parking of the batch's (a, T) pairs and of the step ballots (one
  // broadcast load per step instead of two shuffles, one store instead of a select); the
  // 16-lane walk keeps them in registers, where it needs fewer
  constexpr bool PARK = LPU == 32;
  int2* park_w = reinterpret_cast<int2*>(smem + L.park) + (threadIdx.x & ~31);
  uint32_t* vote_w = reinterpret_cast<uint32_t*>(smem + L.vote) + (threadIdx.x & ~31);

  // blocks run in launch order, so the heaviest samples start first (a longest-first schedule)
  const int b = P.order ? P.order[blockIdx.y] : blockIdx.y, tile = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gi = lane / LPU, glane = lane % LPU;
  const uint32_t gmask_bits = LPU == 32 ? 0xffffffffu : ((1u << LPU) - 1u);
  const int OCP = P.ocp, NPM = P.tile_h * P.tile_w, KK = P.k * P.k;
  const int SWW = P.nslots * P.G;  // spike words per event

  const int ty = tile / P.tiles_x, tx = tile - ty * P.tiles_x;
  const int oy0 = ty * P.tile_h, ox0 = tx * P.tile_w;
  const int th = min(P.tile_h, P.h_out - oy0), tw = min(P.tile_w, P.w_out - ox0);

  const int zero_row = P.ic * KK * OCP;
  // the weight table's loads are issued kConvStageLoads at a time before they are stored
  for (int i0 = tid; i0 < zero_row + OCP; i0 += blockDim.x * kConvStageLoads) {
    int32_t v[kConvStageLoads];
#pragma unroll
    for (int u = 0; u < kConvStageLoads; ++u) {
      const int i = i0 + u * (int)blockDim.x;
      const int tap = i / OCP, oc = i - tap * OCP;
      v[u] = (oc < P.oc && i < zero_row) ? __ldg(&P.q[(int64_t)oc * P.ic * KK + tap]) : 0;
    }
#pragma unroll
    for (int u = 0; u < kConvStageLoads; ++u) {
      const int i = i0 + u * (int)blockDim.x;
      if (i < zero_row + OCP) w_s[i] = (WT)v[u];
    }
  }
  if (P.lut_in_smem)
    for (int i = tid; i < P.qc.lut_len; i += blockDim.x) lut_s[i] = P.lut[i];
  for (int i = tid; i < NPM * OCP; i += blockDim.x) v_s[i] = 0;
  for (int i = tid; i < NPM * P.G; i += blockDim.x) {
    tprev_s[i] = 0.0f;
    cnt_s[i] = 0;
  }
  if (tid < 8) misc_s[tid] = 0;
  const int32_t* lut = P.lut_in_smem ? lut_s : P.lut;

  const int32_t n_eff = P.n_eff(b);
  const int32_t nev = P.T == 1 ? n_eff : P.tile_len[(int64_t)b * P.T + tile];
  const int32_t* list = P.T == 1 ? nullptr
                                 : P.tile_lists + (int64_t)b * P.list_stride +
                                       P.tile_off[(int64_t)b * P.T + tile];
  const int64_t row = b;
  uint32_t* sw_b = P.sw + (int64_t)b * P.sw_stride;
  int32_t* chunk_spk_b = P.chunk_spikes + (int64_t)b * P.n_spk_chunks;

  int32_t acc_min = 0, acc_max = 0, acc_ovf = 0, acc_spk = 0;
  const StepConsts sc(P.qc);
  const int ntasks_all = (NPM * P.G + UPW - 1) / UPW;
  __syncthreads();

  for (int32_t base = 0; base < nev; base += kFusedChunk) {
    const int32_t nchunk = min(kFusedChunk, nev - base);
    // -------- phase 1: decode the chunk and bucket its candidates by position
    auto load_ev = [&](int e, int32_t& j, float& t, int32_t& sv) {
      j = e < nchunk ? (list ? list[base + e] : base + e) : -1;
      if (j >= 0) {
        t = P.in.times[row * P.in.capacity + j];
        sv = P.in.src[row * P.in.capacity + j];
      }
    };
    for (int i = tid; i < NPM * CHW; i += blockDim.x) mask_s[i] = 0;
    for (int i = tid; i < kFusedChunk * SWW; i += blockDim.x) sw_s[i] = 0;
    if (tid == 0) misc_s[0] = 0;
    __syncthreads();
    auto decode = [&](int e0, int32_t j, float t, int32_t srcv) {  // warp-uniform e0
      const int e = e0 + lane;
      const bool in = j >= 0;
      EvCand k{0, 1, 0, 0, 1, 0};
      if (in) {
        int32_t c, y, x;
        k = event_cand(P, srcv, c, y, x);
        EvRec r;
        r.t = t;
        r.ckk = c * KK;
        r.yx = ((uint32_t)(y + P.p) << 16) | (uint32_t)(x + P.p);
        r.omin = ((uint32_t)(k.oy_min + 32768) << 16) | (uint32_t)(k.ox_min + 32768);
        ev_s[e] = r;
        if (list) ej_s[e] = j;
        // clip to this tile
        k.oy_lo = max(k.oy_lo, oy0);
        k.oy_hi = min(k.oy_hi, oy0 + th - 1);
        k.ox_lo = max(k.ox_lo, ox0);
        k.ox_hi = min(k.ox_hi, ox0 + tw - 1);
      }
      // one candidate slot per round; lanes hitting the same position share one mask word,
      // written by the group's first lane (no other warp writes this word).  Different lanes
      // may lead the same position in different rounds, and the match gives no memory order
      // between them, so the update is an atomic OR.
      const int wrd = e0 >> 5;
      if (P.ncand == 2) {
        // 2x2 windows: one match per event.  Lanes whose windows start at the same position with
        // the same valid slots share all their candidate positions, so the group's first lane
        // sets the group's bits in every one of them (a tile holds at most 256 positions, so
        // the tile-local origin, offset by 2, fits in 9 bits per axis).
        uint32_t vb = 0;
        if (in) {
          const bool y0 = k.oy_min >= k.oy_lo && k.oy_min <= k.oy_hi;
          const bool y1 = k.oy_min + 1 >= k.oy_lo && k.oy_min + 1 <= k.oy_hi;
          const bool x0 = k.ox_min >= k.ox_lo && k.ox_min <= k.ox_hi;
          const bool x1 = k.ox_min + 1 >= k.ox_lo && k.ox_min + 1 <= k.ox_hi;
          vb = (uint32_t)(y0 && x0) | ((uint32_t)(y0 && x1) << 1) | ((uint32_t)(y1 && x0) << 2) |
               ((uint32_t)(y1 && x1) << 3);
        }
        const int ly = k.oy_min - oy0, lx = k.ox_min - ox0;
        const int32_t key = vb ? (((ly + 2) << 13) | ((lx + 2) << 4) | (int32_t)vb) : -1;
        const uint32_t same = __match_any_sync(0xffffffffu, key);
        if (vb && (__ffs(same) - 1) == lane) {
          const int i0 = (ly * P.tile_w + lx) * CHW + wrd;  // slot (0, 0); used only if valid
          if (vb & 1u) atomicOr(&mask_s[i0], same);
          if (vb & 2u) atomicOr(&mask_s[i0 + CHW], same);
          if (vb & 4u) atomicOr(&mask_s[i0 + P.tile_w * CHW], same);
          if (vb & 8u) atomicOr(&mask_s[i0 + (P.tile_w + 1) * CHW], same);
        }
      } else {
        for (int a = 0; a < P.ncand; ++a)
          for (int bb = 0; bb < P.ncand; ++bb) {
            const int oy = k.oy_min + a, ox = k.ox_min + bb;
            const bool ok = in && oy >= k.oy_lo && oy <= k.oy_hi && ox >= k.ox_lo && ox <= k.ox_hi;
            const int pl = ok ? (oy - oy0) * P.tile_w + (ox - ox0) : -1;
            const uint32_t same = __match_any_sync(0xffffffffu, pl);
            if (ok && (__ffs(same) - 1) == lane) atomicOr(&mask_s[pl * CHW + wrd], same);
          }
      }
    };
#pragma unroll 1
    for (int e0 = warp * 32; e0 < kFusedChunk; e0 += kFusedThreads) {  // warp-uniform trip count
      int32_t j, sv = 0;
      float t = 0.0f;
      load_ev(e0 + lane, j, t, sv);
      decode(e0, j, t, sv);
    }
    __syncthreads();

    // -------- phase 1.5: per-position event lists (arrival order) and the active positions.
    // The NPM x CHW mask words are dealt to all threads in position-major order (per = a power of
    // two, so each position's words belong to tpp consecutive lanes); one block scan of
    // (active-position flag << 20) + popcount gives every word its place in the position-major
    // list and every active position its place in the active list, then all threads expand.
    int32_t n_active = 0;
    {
      int per = 1;
      while (per * (int)blockDim.x < NPM * CHW) per <<= 1;  // <= CHW since NPM <= blockDim
      const int tpp = CHW / per;                              // threads per position
      const int p = tid / tpp, wbase = (tid % tpp) * per;
      int32_t c = 0;
      if (p < NPM)
        for (int i = 0; i < per; ++i) c += __popc(mask_s[p * CHW + wbase + i]);
      int32_t cpos = c;
      for (int o = 1; o < tpp; o <<= 1) cpos += __shfl_xor_sync(0xffffffffu, cpos, o);
      const bool head = p < NPM && wbase == 0;
      int32_t tot;
      const int32_t pre =
          block_exclusive_scan(((head && cpos > 0) ? (1 << 20) : 0) + c, s_scan, tot);
      int32_t off = pre & 0xfffff;  // list entries per chunk stay below 2^20
      n_active = tot >> 20;
      if (head) {
        posoff_s[p] = off;
        poscnt_s[p] = cpos;
        if (cpos > 0) act_s[pre >> 20] = p;
      }
      if (p < NPM)
        for (int i = 0; i < per; ++i) {
          const int w = wbase + i;
          uint32_t m = mask_s[p * CHW + w];
          while (m) {
            list_s[off++] = (uint16_t)(w * 32 + __ffs(m) - 1);
            m &= m - 1u;
          }
        }
    }
    __syncthreads();

    // -------- phase 2: lane groups run the active positions' queues over this chunk.  A batch
    // of up to LPU events is prepared lane-parallel (one event per lane: Δt, decay code, weight
    // tap, spike-word slot); only the register update itself walks the batch sequentially.
    const int ntasks = (n_active * P.G + UPW - 1) / UPW;
    for (;;) {
      int task = 0;
      if (lane == 0) task = atomicAdd(&misc_s[0], 1);
      task = __shfl_sync(0xffffffffu, task, 0);
      if (task >= ntasks) break;
      const int unit = task * UPW + gi;
      const bool unit_ok = unit < n_active * P.G;
      const int ai = P.G == 1 ? unit : (int)P.fd_G.div((uint32_t)unit);
      const int g = unit - ai * P.G;
      const int pl = unit_ok ? act_s[ai] : 0;
      const int ly = (int)P.fd_tw.div((uint32_t)pl), lx = pl - ly * P.tile_w;
      const int oc = g * LPU + glane;
      const bool lane_ok = unit_ok && oc < P.oc;
      const int oy = oy0 + ly, ox = ox0 + lx;
      const int oys = oy * P.s, oxs = ox * P.s;
      const int32_t n = unit_ok ? poscnt_s[pl] : 0;
      const int32_t lbase = unit_ok ? posoff_s[pl] : 0;
      int32_t V = 0, cn = 0, vth = 0;
      float tp = 0.0f;
      if (unit_ok) {
        V = v_s[pl * OCP + oc];
        tp = tprev_s[pl * P.G + g];
        cn = cnt_s[pl * P.G + g];
      }
      // a layer without a threshold, and lanes past the channel count, never fire: their register
      // stays inside total_bits < 31 bits, below INT32_MAX
      vth = INT32_MAX;
      if (lane_ok && P.has_vth) vth = __ldg(&P.vth[(int64_t)oc * P.n_sp + oy * P.w_out + ox]);
      const int32_t nmax = __reduce_max_sync(0xffffffffu, n);
      for (int32_t b0 = 0; b0 < nmax; b0 += LPU) {
        const int32_t idx = b0 + glane;
        const bool has = idx < n;
        const int e = has ? list_s[lbase + idx] : 0;
        const EvRec r = ev_s[e];
        float tpv = __shfl_up_sync(0xffffffffu, r.t, 1, LPU);
        if (glane == 0) tpv = tp;
        const bool kept = has && (cn + glane) < P.L;  // cn already counts earlier batches
        const int32_t dt = dt_from_times(r.t, tpv);
        const int32_t ky = (int32_t)(r.yx >> 16) - oys;
        const int32_t kx = (int32_t)(r.yx & 0xffffu) - oxs;
        // weight row offset of the event's tap; lanes without a kept event (their placeholder
        // record may give a negative tap) get -1, or in the no-fit form an identity step on the
        // zero row: there it changes nothing (V stays, already inside the tracked range, and
        // below every threshold, all positive without needs_tail), so the walk needs no guard
        constexpr bool kPadIdentity = FORM == kStepWideNoFit;
        const int32_t a = (dt == 0 || (kPadIdentity && !kept))
                              ? sc.ident_a : decay_code(dt, lut, P.qc.lut_len);
        const int32_t T = kept ? (r.ckk + ky * P.k + kx) * OCP : (kPadIdentity ? zero_row : -1);
        const int sy = oy - ((int32_t)(r.omin >> 16) - 32768);
        const int sx = ox - ((int32_t)(r.omin & 0xffffu) - 32768);
        const int widx = e * SWW + (sy * P.ncand + sx) * P.G + g;
        const int32_t nb = min(n - b0, LPU);  // this group's events in the batch (may be <= 0)
        const float last_t = __shfl_sync(0xffffffffu, r.t, nb > 0 ? nb - 1 : 0, LPU);
        if (nb > 0) tp = last_t;
        const int32_t nbw = min(nmax - b0, LPU);  // warp-uniform batch length
        uint32_t myvote = 0;  // the warp's spike ballot of this lane's step
        if (PARK) {
          __syncwarp();
          park_w[lane] = make_int2(a, T);
          __syncwarp();
        }
        // 16-lane groups: the walk is unrolled so that the broadcasts and weight loads of later
        // steps are issued ahead of the dependent register updates
        auto walk = [&](int st) {
          int32_t as, Ts;
          if (PARK) {
            const int2 at = park_w[st];
            as = at.x;
            Ts = at.y;
          } else {
            as = __shfl_sync(0xffffffffu, a, st, LPU);
            Ts = __shfl_sync(0xffffffffu, T, st, LPU);
          }
          bool spike = false;
          if (kPadIdentity || (Ts >= 0 && lane_ok)) {
            const int32_t qv = (int32_t)w_s[Ts + oc];
            int32_t u;
            const int32_t w = sc.step<SAT, FORM != kStepSplit, FORM != kStepWideNoFit>(V, as, qv, u);
            spike = w >= vth;
            V = spike ? 0 : w;
            // overflow is read off the unfitted range at the end of the layer (layer_finish)
            acc_min = min(acc_min, u);
            acc_max = max(acc_max, u);
          }
          const uint32_t vote = __ballot_sync(0xffffffffu, spike);
          if (PARK) {
            if (lane == 0) vote_w[st] = vote;
          } else if (glane == st) {
            myvote = vote;
          }
        };
        if (LPU <= 16) {
          if (nbw == LPU) {
#pragma unroll
            for (int st = 0; st < LPU; ++st) walk(st);
          } else {
#pragma unroll
            for (int st = 0; st < LPU; ++st)
              if (st < nbw) walk(st);
          }
        } else {  // 32-lane groups: unrolling (by 8: +4 %, fully: +33 %) and a one-step
                  // software pipeline (+12 %) all measured slower than the plain loop
          for (int st = 0; st < nbw; ++st) walk(st);
        }
        if (PARK) {
          __syncwarp();
          myvote = vote_w[lane];
          __syncwarp();
        }
        if (has) sw_s[widx] = (myvote >> (gi * LPU)) & gmask_bits;
        cn += max(nb, 0);
      }
      if (unit_ok) {
        v_s[pl * OCP + oc] = V;
        if (glane == 0) {
          tprev_s[pl * P.G + g] = tp;
          cnt_s[pl * P.G + g] = cn;
        }
      }
    }
    __syncthreads();

    // -------- flush the chunk's spike words and its spike counts per 256-event group
    if (!list) {
      uint32_t* dst = sw_b + (int64_t)base * SWW;
      for (int i = tid; i < nchunk * SWW; i += blockDim.x) dst[i] = sw_s[i];
      for (int e0 = warp * 32; e0 < kFusedChunk; e0 += blockDim.x) {
        const int e = e0 + lane;
        int32_t cnt = 0;
        if (e < nchunk)
          for (int i = 0; i < SWW; ++i) cnt += __popc(sw_s[e * SWW + i]);
        cnt = warp_sum(cnt);
        if (lane == 0 && cnt) atomicAdd(&chunk_spk_b[(base + e0) >> kConvGroupShift], cnt);
      }
    } else {
      // several tiles share an event: write only the slots whose position is in this tile
      for (int e = tid; e < nchunk; e += blockDim.x) {
        const int32_t j = ej_s[e];
        const EvRec r = ev_s[e];
        const int oym = (int32_t)(r.omin >> 16) - 32768, oxm = (int32_t)(r.omin & 0xffffu) - 32768;
        int32_t cnt = 0;
        for (int sy = 0; sy < P.ncand; ++sy)
          for (int sx = 0; sx < P.ncand; ++sx) {
            const int oy = oym + sy, ox = oxm + sx;
            if (oy < oy0 || oy >= oy0 + th || ox < ox0 || ox >= ox0 + tw) continue;
            for (int g = 0; g < P.G; ++g) {
              const int slot = (sy * P.ncand + sx) * P.G + g;
              const uint32_t wd = sw_s[e * SWW + slot];
              sw_b[(int64_t)j * SWW + slot] = wd;
              cnt += __popc(wd);
            }
          }
        if (cnt) atomicAdd(&chunk_spk_b[j >> kConvGroupShift], cnt);
      }
    }
    __syncthreads();
  }

  // -------- finalize: catch-up column, identity tail, outputs (conv.py:102-125 regimes)
  const int32_t E = P.in.capacity;
  const int32_t n_in = P.in_nreal[b];
  const int32_t gl_idx = (int32_t)jax_index((int64_t)n_in - 1, E);
  const float global_last = P.in.time(row, gl_idx, n_eff);
  if (tid == 0) misc_s[0] = 0;
  __syncthreads();
  for (;;) {
    int task = 0;
    if (lane == 0) task = atomicAdd(&misc_s[0], 1);
    task = __shfl_sync(0xffffffffu, task, 0);
    if (task >= ntasks_all) break;
    const int unit = task * UPW + gi;
    const int pl = P.G == 1 ? unit : (int)P.fd_G.div((uint32_t)unit);
    const int g = unit - pl * P.G;
    const int ly = (int)P.fd_tw.div((uint32_t)pl), lx = pl - ly * P.tile_w;
    const bool unit_ok = pl < NPM && ly < th && lx < tw;
    const int oc = g * LPU + glane;
    if (unit_ok && oc < P.oc) {
      const int oy = oy0 + ly, ox = ox0 + lx, pos = oy * P.w_out + ox;
      int32_t V = v_s[pl * OCP + oc];
      const int32_t cn = cnt_s[pl * P.G + g];
      const float tp = tprev_s[pl * P.G + g];
      const int32_t vth = P.has_vth ? P.vth[(int64_t)oc * P.n_sp + pos] : 0;
      int32_t tail = 0;
      if (cn < P.L) {
        // catch-up column: Δt = global last input time - this position's last real event
        // time (zero when the position received nothing), weight code 0.
        const int32_t dt = cn > 0 ? dt_from_times(global_last, tp) : 0;
        const int32_t a = decay_code(dt, lut, P.qc.lut_len);
        int32_t u;
        bool ovf;
        const int32_t w = quant_step(V, a, dt == 0, 0, P.qc, u, ovf);
        acc_min = min(acc_min, u);
        acc_max = max(acc_max, u);
        acc_ovf |= (int32_t)ovf;
        const bool spike = P.has_vth && w >= vth;
        V = spike ? 0 : w;
        tail += spike;
        const int32_t n_ident = P.L - cn - 1;  // identity columns: U = V, no decay, q = 0
        if (n_ident > 0) {
          acc_min = min(acc_min, V);
          acc_max = max(acc_max, V);
          if (P.has_vth && V >= vth) {
            tail += 1 + (0 >= vth ? n_ident - 1 : 0);
            V = 0;
          }
        }
      }
      const int64_t neuron = (int64_t)oc * P.n_sp + pos;
      P.v_final[(int64_t)b * P.n_neurons + neuron] = V;
      if (P.tail_mode) P.tail_cnt[(int64_t)b * P.n_neurons + neuron] = tail;
      if (tail) {
        atomicAdd(&P.tail_total[b], tail);
        acc_spk += tail;
      }
      if (glane == 0 && g == 0) atomicMax(&P.needed[b], cn + 1);
    }
  }

  // -------- block reductions -> per-sample scratch
  acc_min = warp_min(acc_min);
  acc_max = warp_max(acc_max);
  acc_ovf = warp_or(acc_ovf);
  acc_spk = warp_sum(acc_spk);
  if (lane == 0) {
    atomicMin(&misc_s[1], acc_min);
    atomicMax(&misc_s[2], acc_max);
    atomicOr(&misc_s[3], acc_ovf);
    atomicAdd(&misc_s[4], acc_spk);
  }
  __syncthreads();
  if (tid == 0) {
    atomicMin(&P.vmin[b], misc_s[1]);
    atomicMax(&P.vmax[b], misc_s[2]);
    if (misc_s[3]) atomicOr(&P.ovf[b], 1);
    if (misc_s[4]) atomicAdd(&P.s_total[b], misc_s[4]);  // tail spikes; spike_chunk_scan
  }                                                      // adds the spike words' count
}

// ------------------------------------------------------------------ compaction

// r-th spike (0-based) of an event whose candidate slots s < 4 hold spike words w[s] (bit = channel,
// valid slots only), in neuron order: channel ascending, then slot.  The per-channel counts are
// summed bit-sliced (lo + 2 mid + 4 hi, a carry-save add of the four words), the channel is found
// by binary lifting over prefix counts, then the slot among that channel's set bits.
__device__ __forceinline__ void rank_in_words(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                                              int32_t r, int& channel, int& slot) {
  const uint32_t s1 = w0 ^ w1, c1 = w0 & w1, s2 = w2 ^ w3, c2 = w2 & w3;
  const uint32_t lo = s1 ^ s2, cl = s1 & s2;
  const uint32_t mid = c1 ^ c2 ^ cl, hi = (c1 & c2) | (cl & (c1 ^ c2));
  int c = 0, below = 0;  // channels [0, c) hold `below` spikes, below <= r
#pragma unroll
  for (int step = 16; step > 0; step >>= 1) {
    const int t = c + step;
    const uint32_t m = t >= 32 ? 0xffffffffu : ((1u << t) - 1u);
    const int cum = __popc(lo & m) + 2 * __popc(mid & m) + 4 * __popc(hi & m);
    if (cum <= r) {
      c = t;
      below = cum;
    }
  }
  int rem = r - below, sl = 0;
  const uint32_t bit = 1u << c;
  const bool b0 = w0 & bit, b1 = w1 & bit, b2 = w2 & bit;
  if (b0 && rem-- == 0) sl = 0;
  else if (b1 && rem-- == 0) sl = 1;
  else if (b2 && rem-- == 0) sl = 2;
  else sl = 3;
  channel = c;
  slot = sl;
}

// Emits sample b's spikes in (event, neuron) order.  One warp per group of 32 input events (the
// groups' output offsets come from the scanned per-group spike counts); the warps of block x take
// groups x * warps + warp, stepping by the grid.  Within an event the order is channel group,
// channel, then position (oy, ox) ascending, i.e. neuron index order.  Each lane counts its
// event's spikes over the valid candidate slots; a warp scan gives every event its offset; then
// the expansion is load-balanced: lane q of each 32-output round finds its event by a binary
// search over the lanes' inclusive offsets, decodes which of the event's spikes it is and writes
// it, so the warp writes consecutive entries and its work follows the spikes.  Warps never wait
// on one another (no shared memory, no block barrier).  FOUR: at most 2 candidates per axis and
// one channel group (the benchmark geometries): the event's four slot words stay in registers
// and the decode is bit arithmetic on them (rank_in_words); otherwise the words are re-read.
// Spikes per channel of a truncated sample (its spike words over the valid candidate slots),
// added into the sample's zeroed oc_total row by all of the sample's compaction blocks; the
// catch-up/identity spikes are added by conv_truncated, which then places the channel cut.
__device__ __forceinline__ void count_channels(const ConvLaunch& P, int b) {
  const int32_t n_eff = P.n_eff(b);
  const int SWW = P.nslots * P.G;
  int32_t* oct = P.oc_total + (int64_t)b * P.oc;
  for (int32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < n_eff; j += gridDim.x * blockDim.x) {
    int32_t cc, y, x;
    const EvCand k = event_cand(P, P.in.src[(int64_t)b * P.in.capacity + j], cc, y, x);
    const uint32_t* sw_j = P.sw + (int64_t)b * P.sw_stride + (int64_t)j * SWW;
    for (int oy = k.oy_lo; oy <= k.oy_hi; ++oy)
      for (int ox = k.ox_lo; ox <= k.ox_hi; ++ox)
        for (int g = 0; g < P.G; ++g) {
          uint32_t wd = sw_j[((oy - k.oy_min) * P.ncand + (ox - k.ox_min)) * P.G + g];
          while (wd) {
            atomicAdd(&oct[g * P.lpu + __ffs(wd) - 1], 1);
            wd &= wd - 1u;
          }
        }
  }
}

// TAB (2x2 windows with an address table): the window comes from the table and the event's four
// slot words from one 16-byte load, masked by the slots valid in the plane.
template <bool FOUR, bool TAB>
__global__ void __launch_bounds__(kCompactThreads, 6)
conv_compact(ConvLaunch P, salt_stream_out out) {
  constexpr uint32_t kAll = 0xffffffffu;
  const int b = P.order ? P.order[blockIdx.y] : blockIdx.y;  // heaviest samples first
  const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const int32_t S = P.s_total[b];
  if (S > P.M) {  // truncated samples are emitted by conv_truncated; count their channels for it
    count_channels(P, b);
    return;
  }
  const int32_t n_eff = P.n_eff(b);
  const int SWW = P.nslots * P.G;
  const uint32_t* sw_b = P.sw + (int64_t)b * P.sw_stride;
  float* ot = out.times + (int64_t)b * P.M;
  int32_t* os = out.src + (int64_t)b * P.M;
  const int32_t n_groups = (n_eff + kConvGroup - 1) >> kConvGroupShift;
  for (int32_t grp = blockIdx.x * wpb + (threadIdx.x >> 5); grp < n_groups;
       grp += gridDim.x * wpb) {
    const int32_t j = (grp << kConvGroupShift) + lane;
    int32_t cnt = 0;
    uint32_t om = 0, rg = 0, w0 = 0, w1 = 0, w2 = 0, w3 = 0;
    float t = 0.0f;
    if (TAB && j < n_eff) {
      const uint4 wv = *reinterpret_cast<const uint4*>(sw_b + (int64_t)j * 4);
      const int32_t sv = P.in.src[(int64_t)b * P.in.capacity + j];
      uint32_t vb;
      int32_t oym, oxm;
      if ((uint32_t)sv < (uint32_t)P.n_addr) {
        const uint32_t en = __ldg(&P.addr_table[sv]);
        vb = en & 15u;
        oym = (int32_t)((en >> 4) & 255u) - 1;
        oxm = (int32_t)((en >> 12) & 255u) - 1;
      } else {  // a source index outside the input plane: decoded as the reference does
        int32_t cc, y, x;
        const EvCand k = event_cand(P, sv, cc, y, x);
        const bool y0 = k.oy_min >= k.oy_lo && k.oy_min <= k.oy_hi;
        const bool y1 = k.oy_min + 1 >= k.oy_lo && k.oy_min + 1 <= k.oy_hi;
        const bool x0 = k.ox_min >= k.ox_lo && k.ox_min <= k.ox_hi;
        const bool x1 = k.ox_min + 1 >= k.ox_lo && k.ox_min + 1 <= k.ox_hi;
        vb = (uint32_t)(y0 && x0) | ((uint32_t)(y0 && x1) << 1) | ((uint32_t)(y1 && x0) << 2) |
             ((uint32_t)(y1 && x1) << 3);
        oym = k.oy_min;
        oxm = k.ox_min;
      }
      w0 = (vb & 1u) ? wv.x : 0u;
      w1 = (vb & 2u) ? wv.y : 0u;
      w2 = (vb & 4u) ? wv.z : 0u;
      w3 = (vb & 8u) ? wv.w : 0u;
      cnt = __popc(w0) + __popc(w1) + __popc(w2) + __popc(w3);
      if (cnt) {
        om = ((uint32_t)(oym + 32768) << 16) | (uint32_t)(oxm + 32768);
        t = P.in.time(b, j, n_eff);
      }
    } else if (!TAB && j < n_eff) {
      int32_t cc, y, x;
      const EvCand k = event_cand(P, P.in.src[(int64_t)b * P.in.capacity + j], cc, y, x);
      const uint32_t* sw_j = sw_b + (int64_t)j * SWW;
      if (FOUR) {  // slot s = (sy, sx) = (s / ncand, s % ncand), ncand <= 2, G == 1
        const bool two = P.ncand == 2;
        const bool y0 = k.oy_min >= k.oy_lo && k.oy_min <= k.oy_hi;
        const bool y1 = two && k.oy_min + 1 >= k.oy_lo && k.oy_min + 1 <= k.oy_hi;
        const bool x0 = k.ox_min >= k.ox_lo && k.ox_min <= k.ox_hi;
        const bool x1 = two && k.ox_min + 1 >= k.ox_lo && k.ox_min + 1 <= k.ox_hi;
        if (y0 && x0) w0 = sw_j[0];
        if (two) {
          if (y0 && x1) w1 = sw_j[1];
          if (y1 && x0) w2 = sw_j[2];
          if (y1 && x1) w3 = sw_j[3];
        }
        cnt = __popc(w0) + __popc(w1) + __popc(w2) + __popc(w3);
      } else {
        for (int oy = k.oy_lo; oy <= k.oy_hi; ++oy)
          for (int ox = k.ox_lo; ox <= k.ox_hi; ++ox) {
            const int slot = (oy - k.oy_min) * P.ncand + (ox - k.ox_min);
            for (int g = 0; g < P.G; ++g) cnt += __popc(sw_j[slot * P.G + g]);
          }
      }
      if (cnt) {
        om = ((uint32_t)(k.oy_min + 32768) << 16) | (uint32_t)(k.ox_min + 32768);
        rg = (uint32_t)(k.oy_lo - k.oy_min) | ((uint32_t)(k.oy_hi - k.oy_min) << 4) |
             ((uint32_t)(k.ox_lo - k.ox_min) << 8) | ((uint32_t)(k.ox_hi - k.ox_min) << 12);
        t = P.in.time(b, j, n_eff);
      }
    }
    int32_t incl = cnt;  // inclusive scan over the warp's events
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t n = __shfl_up_sync(kAll, incl, o);
      if (lane >= o) incl += n;
    }
    const int32_t total = __shfl_sync(kAll, incl, 31);
    if (total == 0) continue;
    const int32_t base = P.chunk_off[(int64_t)b * P.n_spk_chunks + grp];
    for (int32_t q0 = 0; q0 < total; q0 += 32) {
      const int32_t q = q0 + lane;
      int e = 0;  // lanes whose inclusive offset is <= q: the event holding output q
#pragma unroll
      for (int step = 16; step > 0; step >>= 1)
        if (__shfl_sync(kAll, incl, e + step - 1) <= q) e += step;
      const int32_t before = __shfl_sync(kAll, incl, e > 0 ? e - 1 : 0);
      const uint32_t eom = __shfl_sync(kAll, om, e);
      const float et = __shfl_sync(kAll, t, e);
      const int oy_min = (int)(eom >> 16) - 32768, ox_min = (int)(eom & 0xffffu) - 32768;
      int32_t r = q - (e > 0 ? before : 0);  // rank among the event's spikes
      int32_t neuron = -1;
      if (FOUR) {
        const uint32_t e0 = __shfl_sync(kAll, w0, e), e1 = __shfl_sync(kAll, w1, e);
        const uint32_t e2 = __shfl_sync(kAll, w2, e), e3 = __shfl_sync(kAll, w3, e);
        int ch, sl;
        rank_in_words(e0, e1, e2, e3, r, ch, sl);
        const int sy = P.ncand == 2 ? sl >> 1 : 0, sx = P.ncand == 2 ? sl & 1 : 0;
        neuron = ch * P.n_sp + (oy_min + sy) * P.w_out + (ox_min + sx);
      }
      if (!FOUR) {
        const uint32_t erg = __shfl_sync(kAll, rg, e);
        if (q < total) {
          const int ylo = erg & 15, yhi = (erg >> 4) & 15, xlo = (erg >> 8) & 15;
          const int xhi = (erg >> 12) & 15;
          const uint32_t* sw_j = sw_b + (int64_t)((grp << kConvGroupShift) + e) * SWW;
          for (int g = 0; g < P.G && neuron < 0; ++g) {
            uint32_t uni = 0;
            for (int sy = ylo; sy <= yhi; ++sy)
              for (int sx = xlo; sx <= xhi; ++sx) uni |= sw_j[(sy * P.ncand + sx) * P.G + g];
            while (uni && neuron < 0) {
              const int bit = __ffs(uni) - 1;
              uni &= uni - 1u;
              for (int sy = ylo; sy <= yhi && neuron < 0; ++sy)
                for (int sx = xlo; sx <= xhi; ++sx)
                  if ((sw_j[(sy * P.ncand + sx) * P.G + g] >> bit) & 1u) {
                    if (r == 0) {
                      neuron = (g * P.lpu + bit) * P.n_sp + (oy_min + sy) * P.w_out + (ox_min + sx);
                      break;
                    }
                    --r;
                  }
            }
          }
        }
      }
      if (q < total) {
        ot[base + q] = et;
        os[base + q] = neuron;
      }
    }
  }
}

void* conv_compact_kernel(int ncand, int G, bool table) {
  if (table && ncand == 2 && G == 1) return (void*)conv_compact<true, true>;
  return (ncand <= 2 && G == 1) ? (void*)conv_compact<true, false>
                                : (void*)conv_compact<false, false>;
}

// Spikes on catch-up / identity columns (tail mode only): they map to the empty queue entry
// (global index = stream length, stream.py:36-38), so they sort after every real spike, in
// neuron order; their time is the input stream's last entry.
__global__ void conv_tail_append(ConvLaunch P, salt_stream_out out) {
  __shared__ int32_t s_scan[kScanSmem];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int32_t S = P.s_total[b], Tb = P.tail_total[b];
  if (S > P.M || Tb == 0) return;
  const int32_t E = P.in.capacity;
  const float t = P.in.time(b, E - 1, P.n_eff(b));
  int32_t written = S - Tb;
  for (int64_t n0 = 0; n0 < P.n_neurons; n0 += blockDim.x) {
    const int64_t n = n0 + tid;
    const int32_t c = n < P.n_neurons ? P.tail_cnt[(int64_t)b * P.n_neurons + n] : 0;
    int32_t total;
    const int32_t off = block_exclusive_scan(c, s_scan, total);
    for (int32_t k = 0; k < c; ++k) {
      out.times[(int64_t)b * P.M + written + off + k] = t;
      out.src[(int64_t)b * P.M + written + off + k] = (int32_t)n;
    }
    written += total;
  }
}

// Samples with more spikes than max_out_spikes: keep the first M in neuron-major order
// (jnp.nonzero(size=M) over the (neuron, column) grid, stream.py:60), then emit them in
// (event, neuron) order.  One block per sample; only truncated samples do any work.
__global__ void __launch_bounds__(kTruncThreads)
conv_truncated(ConvLaunch P, salt_stream_out out, int32_t* __restrict__ scratch_hist) {
  __shared__ int32_t s_scan[kScanSmem];
  __shared__ int32_t s_cut[8];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int32_t S = P.s_total[b], M = P.M;
  if (S <= M || M <= 0) return;
  const int32_t n_eff = P.n_eff(b);
  const int SWW = P.nslots * P.G;
  int32_t* hist = scratch_hist + (int64_t)b * P.n_sp * 2;  // [n_sp] real, [n_sp] tail
  // 1. spikes per channel: conv_compact counted the spike words into the oc_total row; the
  // catch-up/identity spikes are added here.  Then the channel cut: the channel holding the
  // M-th spike in neuron-major order
  int32_t* oct = P.oc_total + (int64_t)b * P.oc;
  if (P.tail_mode)
    for (int64_t n = tid; n < P.n_neurons; n += blockDim.x) {
      const int32_t c = P.tail_cnt[(int64_t)b * P.n_neurons + n];
      if (c) atomicAdd(&oct[n / P.n_sp], c);
    }
  __syncthreads();
  if (tid == 0) {
    int32_t cum = 0, occ = P.oc - 1;
    for (int oc = 0; oc < P.oc; ++oc) {
      const int32_t t = oct[oc];
      if (cum + t >= M) {
        occ = oc;
        break;
      }
      cum += t;
    }
    s_cut[0] = occ;
    s_cut[1] = M - cum;  // spikes to keep inside channel occ (>= 1)
  }
  for (int i = tid; i < 2 * P.n_sp; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int occ = s_cut[0];
  const int gq = occ / P.lpu, bq = occ % P.lpu;
  // 2. per-position spike counts of channel occ
  for (int32_t j = tid; j < n_eff; j += blockDim.x) {
    int32_t cc, y, x;
    const EvCand k = event_cand(P, P.in.src[(int64_t)b * P.in.capacity + j], cc, y, x);
    const uint32_t* sw_j = P.sw + (int64_t)b * P.sw_stride + (int64_t)j * SWW;
    for (int oy = k.oy_lo; oy <= k.oy_hi; ++oy)
      for (int ox = k.ox_lo; ox <= k.ox_hi; ++ox)
        if (sw_j[((oy - k.oy_min) * P.ncand + (ox - k.ox_min)) * P.G + gq] & (1u << bq))
          atomicAdd(&hist[oy * P.w_out + ox], 1);
  }
  if (P.tail_mode)
    for (int pos = tid; pos < P.n_sp; pos += blockDim.x)
      hist[P.n_sp + pos] = P.tail_cnt[(int64_t)b * P.n_neurons + (int64_t)occ * P.n_sp + pos];
  __syncthreads();
  if (tid == 0) {
    const int32_t need = s_cut[1];
    int32_t cum = 0, pstar = P.n_sp - 1;
    for (int pos = 0; pos < P.n_sp; ++pos) {
      const int32_t t = hist[pos] + hist[P.n_sp + pos];
      if (cum + t >= need) {
        pstar = pos;
        break;
      }
      cum += t;
    }
    const int32_t r2 = need - cum;  // spikes kept of neuron (occ, pstar), in column order
    s_cut[1] = pstar;
    if (r2 <= hist[pstar]) {
      s_cut[2] = r2;  // the r2-th real spike is the last kept one: located below
      s_cut[3] = 0;
    } else {
      s_cut[2] = hist[pstar];
      s_cut[3] = r2 - hist[pstar];
    }
    s_cut[4] = 0x7fffffff;  // j_cut
  }
  __syncthreads();
  const int pstar = s_cut[1];
  // 3. the event index of the s_cut[2]-th real spike of neuron (occ, pstar)
  if (s_cut[2] > 0) {
    int32_t seen = 0;
    const int py = pstar / P.w_out, px = pstar % P.w_out;
    for (int32_t j0 = 0; j0 < n_eff; j0 += blockDim.x) {
      const int32_t j = j0 + tid;
      int32_t hit = 0;
      if (j < n_eff) {
        int32_t cc, y, x;
        const EvCand k = event_cand(P, P.in.src[(int64_t)b * P.in.capacity + j], cc, y, x);
        if (py >= k.oy_lo && py <= k.oy_hi && px >= k.ox_lo && px <= k.ox_hi) {
          const uint32_t* sw_j = P.sw + (int64_t)b * P.sw_stride + (int64_t)j * SWW;
          hit = (sw_j[((py - k.oy_min) * P.ncand + (px - k.ox_min)) * P.G + gq] >> bq) & 1u;
        }
      }
      int32_t total;
      const int32_t off = block_exclusive_scan(hit, s_scan, total);
      if (hit && seen + off + 1 == s_cut[2]) s_cut[4] = j;
      seen += total;
      __syncthreads();
      if (s_cut[4] != 0x7fffffff) break;
    }
  }
  __syncthreads();
  const int32_t j_cut = s_cut[4];
  const int64_t nstar = (int64_t)occ * P.n_sp + pstar;
  // 4. emit kept real spikes in (event, neuron) order
  int32_t written = 0;
  float* ot = out.times + (int64_t)b * M;
  int32_t* os = out.src + (int64_t)b * M;
  for (int32_t j0 = 0; j0 < n_eff; j0 += blockDim.x) {
    const int32_t j = j0 + tid;
    int32_t cnt = 0;
    EvCand k{0, 1, 0, 0, 1, 0};
    const uint32_t* sw_j = P.sw + (int64_t)b * P.sw_stride + (int64_t)j * SWW;
    if (j < n_eff) {
      int32_t cc, y, x;
      k = event_cand(P, P.in.src[(int64_t)b * P.in.capacity + j], cc, y, x);
      for (int g = 0; g < P.G; ++g)
        for (int oy = k.oy_lo; oy <= k.oy_hi; ++oy)
          for (int ox = k.ox_lo; ox <= k.ox_hi; ++ox) {
            uint32_t wd = sw_j[((oy - k.oy_min) * P.ncand + (ox - k.ox_min)) * P.G + g];
            while (wd) {
              const int bit = __ffs(wd) - 1;
              wd &= wd - 1u;
              const int64_t n = (int64_t)(g * P.lpu + bit) * P.n_sp + oy * P.w_out + ox;
              cnt += (n < nstar) || (n == nstar && j <= j_cut);
            }
          }
    }
    int32_t total;
    const int32_t off = block_exclusive_scan(cnt, s_scan, total);
    if (cnt) {
      const float t = P.in.time(b, j, n_eff);
      int32_t kk = written + off;
      for (int g = 0; g < P.G; ++g) {
        uint32_t uni = 0;
        for (int oy = k.oy_lo; oy <= k.oy_hi; ++oy)
          for (int ox = k.ox_lo; ox <= k.ox_hi; ++ox)
            uni |= sw_j[((oy - k.oy_min) * P.ncand + (ox - k.ox_min)) * P.G + g];
        while (uni) {
          const int bit = __ffs(uni) - 1;
          uni &= uni - 1u;
          const int oc = g * P.lpu + bit;
          for (int oy = k.oy_lo; oy <= k.oy_hi; ++oy)
            for (int ox = k.ox_lo; ox <= k.ox_hi; ++ox) {
              const uint32_t wd = sw_j[((oy - k.oy_min) * P.ncand + (ox - k.ox_min)) * P.G + g];
              const int64_t n = (int64_t)oc * P.n_sp + oy * P.w_out + ox;
              if ((wd & (1u << bit)) && ((n < nstar) || (n == nstar && j <= j_cut))) {
                ot[kk] = t;
                os[kk] = (int32_t)n;
                ++kk;
              }
            }
        }
      }
    }
    written += total;
    if (written >= M) break;  // all M kept spikes are real ones and have been written
  }
  // 5. kept tail spikes (neurons before nstar, plus s_cut[3] of nstar), in neuron order
  if (P.tail_mode) {
    const float t = P.in.time(b, P.in.capacity - 1, n_eff);
    const int32_t tail_keep = s_cut[3];
    for (int64_t n0 = 0; n0 <= nstar; n0 += blockDim.x) {
      const int64_t n = n0 + tid;
      int32_t c = 0;
      if (n < nstar) c = P.tail_cnt[(int64_t)b * P.n_neurons + n];
      else if (n == nstar) c = tail_keep;
      int32_t total;
      const int32_t off = block_exclusive_scan(c, s_scan, total);
      for (int32_t kq = 0; kq < c; ++kq) {
        ot[written + off + kq] = t;
        os[written + off + kq] = (int32_t)n;
      }
      written += total;
    }
  }
}

// Host-side dispatch over the (weight width, lanes per channel group, overflow mode, step form)
// instantiations; the no-fit form ignores the overflow mode.
template <typename WT, bool SAT, int FORM>
static void* fused_for_lpu(int lpu) {
  switch (lpu) {
    case 1: return (void*)conv_fused<WT, 1, SAT, FORM>;
    case 2: return (void*)conv_fused<WT, 2, SAT, FORM>;
    case 4: return (void*)conv_fused<WT, 4, SAT, FORM>;
    case 8: return (void*)conv_fused<WT, 8, SAT, FORM>;
    case 16: return (void*)conv_fused<WT, 16, SAT, FORM>;
    default: return (void*)conv_fused<WT, 32, SAT, FORM>;
  }
}

template <bool SAT, int FORM>
static void* fused_for_wt(int wt_bytes, int lpu) {
  if (wt_bytes == 1) return fused_for_lpu<int8_t, SAT, FORM>(lpu);
  if (wt_bytes == 2) return fused_for_lpu<int16_t, SAT, FORM>(lpu);
  return fused_for_lpu<int32_t, SAT, FORM>(lpu);
}

void* conv_fused_kernel(int wt_bytes, int lpu, bool saturate, int form) {
  if (form == kStepWideNoFit) return fused_for_wt<false, kStepWideNoFit>(wt_bytes, lpu);
  if (saturate)
    return form == kStepWide ? fused_for_wt<true, kStepWide>(wt_bytes, lpu)
                             : fused_for_wt<true, kStepSplit>(wt_bytes, lpu);
  return form == kStepWide ? fused_for_wt<false, kStepWide>(wt_bytes, lpu)
                           : fused_for_wt<false, kStepSplit>(wt_bytes, lpu);
}

}  // namespace salt
