// Integer conv layer, queue form, for B200 (sm_100a).
//
// Replaces, like conv_fused, the queue construction (salt_core/connectivity/conv.py:128-172) and
// the integer LIF scan over every queue column (salt_core/quant/scan.py:97-132) of one (tile,
// sample) block, for layers whose catch-up and identity columns cannot fire (no needs_tail).
// conv_fused interleaves bucketing and recurrence 512 events at a time, so each position's
// recurrence state is reloaded, and a batch of its events prepared, once per chunk; here the
// block first builds every position's complete queue for the sample, then walks each queue once:
//
//   1. count    each event's receptive-field candidates inside the tile are counted per
//               position.  The kept lengths min(n, max_queue_len) give each position's queue
//               offset, and the positions are ordered by decreasing kept length (quarter-octave
//               buckets), so that lane groups sharing a warp walk queues of similar length and
//               the longest queues start first.
//   2. queue    256-event chunks in arrival order are bucketed by position into one bitmask word
//               per warp (match_any); a column scan per position turns the words into ranks, and
//               every candidate writes its queue entry at (position offset + entries already
//               queued + rank) — the (position, arrival) order of conv.py:71 — holding its event
//               time, the weight row of its tap and its spike-word index; past max_queue_len it
//               writes a zero spike word instead (a dropped column never fires).
//   3. walk     lane groups (one lane per output channel) take the positions in that order and
//               run each whole queue with the membrane register in a register: per batch of
//               entries the lanes form each Δt to the previous entry and its decay code, then the
//               recurrence walks the batch; then the catch-up column (conv.py:102-125 regimes).
//               Spike words go straight to the event's slot; spikes per 32-event group are
//               counted in shared memory.
//
// The queues live in global memory (8 bytes per kept candidate); a block reads back only what it
// wrote moments before, so they are served from L2.
#pragma once
#include "salt_layers.cuh"

namespace salt {

namespace {

constexpr int kQBuckets = 64;   // quarter-octave buckets of the kept queue length

// Shared-memory layout of conv_queue; the host sizes it with the same function.
struct QueueSmem {
  size_t w, lut, cnt, off, run, lastt, order, mask, pre, evt, grp, bucket, park, vote, misc, total;
  __host__ __device__ QueueSmem(const ConvLaunch& P, int wt_bytes, int threads) {
    const size_t npm = (size_t)P.tile_h * P.tile_w;
    const size_t chw = (size_t)threads / 32;
    size_t o = 0;
    // weights [ic*k*k][ocp], then one zero row (the padding steps of the no-fit walk)
    w = o;      o += align16((size_t)(P.ic * P.k * P.k + 1) * P.ocp * wt_bytes);
    lut = o;    o += align16((size_t)(P.lut_in_smem ? P.qc.lut_len : 0) * 4);
    cnt = o;    o += align16(npm * 4);           // events per position (all, kept or not)
    off = o;    o += align16(npm * 4);           // queue offset per position
    run = o;    o += align16(npm * 4);           // entries queued so far per position
    lastt = o;  o += align16(npm * 4);           // time of the position's latest event so far
    order = o;  o += align16(npm * 4);           // positions by decreasing kept length
    mask = o;   o += align16(2 * chw * npm * 4); // [chunk parity][warp word][position] bitmasks
    pre = o;    o += align16(chw * npm * 4);     // [warp word][position] entries before the word
    evt = o;    o += align16(2 * (size_t)threads * 4);  // [chunk parity] event times
    grp = o;    o += align16((size_t)(P.grp_in_smem ? P.n_spk_chunks : 0) * 4);
    bucket = o; o += align16((size_t)kQBuckets * 4);
    // 32-lane groups park each batch's (decay code, weight row) pairs and step ballots per warp
    park = o;   o += align16((size_t)(P.lpu == 32 ? threads : 0) * sizeof(int2));
    vote = o;   o += align16((size_t)(P.lpu == 32 ? threads : 0) * 4);
    misc = o;   o += 64;
    total = o;
  }
};

// Quarter-octave bucket of a kept queue length, longest first (bucket 0); empty queues last.
__device__ __forceinline__ int length_bucket(int32_t n) {
  if (n <= 0) return kQBuckets - 1;
  const int e = 31 - __clz(n);
  const int frac = e >= 2 ? (n >> (e - 2)) & 3 : (n << (2 - e)) & 3;
  return kQBuckets - 2 - min(kQBuckets - 2, e * 4 + frac);
}

// Candidate slots of a 2x2 window (ncand == 2) inside the clipped ranges: bit (sy * 2 + sx).
__device__ __forceinline__ uint32_t window_bits(const EvCand& k) {
  const bool y0 = k.oy_min >= k.oy_lo && k.oy_min <= k.oy_hi;
  const bool y1 = k.oy_min + 1 >= k.oy_lo && k.oy_min + 1 <= k.oy_hi;
  const bool x0 = k.ox_min >= k.ox_lo && k.ox_min <= k.ox_hi;
  const bool x1 = k.ox_min + 1 >= k.ox_lo && k.ox_min + 1 <= k.ox_hi;
  return (uint32_t)(y0 && x0) | ((uint32_t)(y0 && x1) << 1) | ((uint32_t)(y1 && x0) << 2) |
         ((uint32_t)(y1 && x1) << 3);
}

// The 2x2 window (ncand == 2) of one event inside a tile: tile-local origin, the slots valid in
// the tile (bit sy * 2 + sx) and the tap of slot (0, 0).
struct Win {
  int32_t ly, lx;
  uint32_t vb;
  int32_t tap0;
};

}  // namespace

// Six blocks (48 warps) per SM: the walk's queue loads come from L2, and the count and queue
// phases wait at block barriers, so the kernel needs the warps to hide them (40 registers).
// WIN: 2x2 windows read from the layer's address table (conv_addr_table) instead of decoding
// every source index twice.
// THREADS: 256 (six blocks per SM) or 512 (three), the events a chunk buckets.  512-thread
// blocks halve the block barriers per event and the tiles a small batch needs (configuration 3,
// G events/s, 256 -> 512: 4096 samples 7.16 -> 7.68, 1024 samples 5.61 -> 6.50, 512 samples
// 4.19 -> 4.93).
template <typename WT, int LPU, bool SAT, int FORM, bool WIN, int THREADS>
__global__ void __launch_bounds__(THREADS, THREADS == 256 ? 6 : 3)
conv_queue(ConvLaunch P) {
  static_assert(FORM != kStepSplit, "the queue form serves layers without needs_tail only");
  constexpr int UPW = 32 / LPU;  // units (position x channel group) per warp
  constexpr int CHW = THREADS / 32;
  constexpr uint32_t kAll = 0xffffffffu;
  extern __shared__ __align__(16) uint8_t smem[];
  const QueueSmem L(P, sizeof(WT), THREADS);
  WT* w_s = reinterpret_cast<WT*>(smem + L.w);
  int32_t* lut_s = reinterpret_cast<int32_t*>(smem + L.lut);
  int32_t* cnt_s = reinterpret_cast<int32_t*>(smem + L.cnt);
  int32_t* off_s = reinterpret_cast<int32_t*>(smem + L.off);
  int32_t* run_s = reinterpret_cast<int32_t*>(smem + L.run);
  float* lastt_s = reinterpret_cast<float*>(smem + L.lastt);
  int32_t* order_s = reinterpret_cast<int32_t*>(smem + L.order);
  uint32_t* mask_s = reinterpret_cast<uint32_t*>(smem + L.mask);
  uint32_t* pre_s = reinterpret_cast<uint32_t*>(smem + L.pre);
  float* evt_s = reinterpret_cast<float*>(smem + L.evt);
  int32_t* grp_s = reinterpret_cast<int32_t*>(smem + L.grp);
  int32_t* bucket_s = reinterpret_cast<int32_t*>(smem + L.bucket);
  int32_t* misc_s = reinterpret_cast<int32_t*>(smem + L.misc);
  __shared__ int32_t s_scan[kScanSmem];
  constexpr bool PARK = LPU == 32;
  int2* park_w = reinterpret_cast<int2*>(smem + L.park) + (threadIdx.x & ~31);
  uint32_t* vote_w = reinterpret_cast<uint32_t*>(smem + L.vote) + (threadIdx.x & ~31);

  // blocks run in launch order, so the heaviest samples start first (a longest-first schedule)
  const int b = P.order ? P.order[blockIdx.y] : blockIdx.y, tile = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gi = lane / LPU, glane = lane % LPU;
  const uint32_t gmask_bits = LPU == 32 ? kAll : ((1u << LPU) - 1u);
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
  for (int i = tid; i < NPM; i += blockDim.x) {
    cnt_s[i] = 0;
    run_s[i] = 0;
    lastt_s[i] = 0.0f;  // a queue's first Δt is measured from time 0
  }
  for (int i = tid; i < 2 * CHW * NPM; i += blockDim.x) mask_s[i] = 0u;
  const int32_t n_eff = P.n_eff(b);
  const int32_t n_groups = (n_eff + kConvGroup - 1) >> kConvGroupShift;
  if (P.grp_in_smem)
    for (int i = tid; i < n_groups; i += blockDim.x) grp_s[i] = 0;
  if (tid < kQBuckets) bucket_s[tid] = 0;
  if (tid < 8) misc_s[tid] = 0;
  const int32_t* lut = P.lut_in_smem ? lut_s : P.lut;

  // tiles come with event lists from the partition kernels, or (few tiles) read the whole stream
  // and keep their own candidates
  const bool part = P.T > 1 && P.tile_lists != nullptr;
  const int32_t nev = !part ? n_eff : P.tile_len[(int64_t)b * P.T + tile];
  const int32_t* list = !part ? nullptr
                                 : P.tile_lists + (int64_t)b * P.list_stride +
                                       P.tile_off[(int64_t)b * P.T + tile];
  const int64_t row = b;
  uint32_t* sw_b = P.sw + (int64_t)b * P.sw_stride;
  int32_t* chunk_spk_b = P.chunk_spikes + (int64_t)b * P.n_spk_chunks;
  // this tile's queues: at most nslots entries per tile event
  int2* q_b = P.queues + (int64_t)b * P.queue_stride +
              (part ? (int64_t)P.nslots * P.tile_off[(int64_t)b * P.T + tile]
                    : (int64_t)tile * P.nslots * P.in.capacity);
  const StepConsts sc(P.qc);

  // Tile-clipped candidates of tile event e (an empty range past the tile's events).
  auto candidates = [&](int32_t e, int32_t& j, int32_t& c, int32_t& y, int32_t& x) {
    EvCand k{0, 1, 0, 0, 1, 0};
    if (e < nev) {
      j = list ? list[e] : e;
      k = event_cand(P, P.in.src[row * P.in.capacity + j], c, y, x);
      k.oy_lo = max(k.oy_lo, oy0);
      k.oy_hi = min(k.oy_hi, oy0 + th - 1);
      k.ox_lo = max(k.ox_lo, ox0);
      k.ox_hi = min(k.ox_hi, ox0 + tw - 1);
    }
    return k;
  };
  // WIN: the window of tile event e from the address table (an empty window past the tile's
  // events).  A source index outside the input plane is decoded as the reference does.
  auto window = [&](int32_t e, int32_t& j) {
    Win w{0, 0, 0u, 0};
    if (e < nev) {
      j = list ? list[e] : e;
      const int32_t sv = P.in.src[row * P.in.capacity + j];
      int32_t oym, oxm;
      uint32_t vb;
      if ((uint32_t)sv < (uint32_t)P.n_addr) {
        const uint32_t en = __ldg(&P.addr_table[sv]);
        vb = en & 15u;
        oym = (int32_t)((en >> 4) & 255u) - 1;
        oxm = (int32_t)((en >> 12) & 255u) - 1;
        w.tap0 = (int32_t)(en >> 20);
      } else {
        int32_t c, y, x;
        const EvCand k = event_cand(P, sv, c, y, x);
        vb = window_bits(k);
        oym = k.oy_min;
        oxm = k.ox_min;
        w.tap0 = c * KK + (y + P.p - oym * P.s) * P.k + (x + P.p - oxm * P.s);
      }
      w.ly = oym - oy0;
      w.lx = oxm - ox0;
      const bool r0 = (uint32_t)w.ly < (uint32_t)th, r1 = (uint32_t)(w.ly + 1) < (uint32_t)th;
      const bool c0 = (uint32_t)w.lx < (uint32_t)tw, c1 = (uint32_t)(w.lx + 1) < (uint32_t)tw;
      w.vb = vb & ((uint32_t)(r0 && c0) | ((uint32_t)(r0 && c1) << 1) |
                   ((uint32_t)(r1 && c0) << 2) | ((uint32_t)(r1 && c1) << 3));
    }
    return w;
  };
  __syncthreads();

  // -------- 1. count each position's events.  Lanes whose 2x2 windows start at the same
  // position with the same valid slots add together (one atomic per group and slot).
#pragma unroll 1
  for (int32_t base = 0; base < nev; base += THREADS) {  // block-uniform trip count
    int32_t j = 0, c = 0, y = 0, x = 0;
    if constexpr (WIN) {
      const Win w = window(base + tid, j);
      const int32_t key = w.vb ? (((w.ly + 2) << 13) | ((w.lx + 2) << 4) | (int32_t)w.vb) : -1;
      const uint32_t same = __match_any_sync(kAll, key);
      if (w.vb && (__ffs(same) - 1) == lane) {
        const int32_t n = __popc(same);
        const int i0 = w.ly * P.tile_w + w.lx;  // slot (0, 0); used only if valid
        if (w.vb & 1u) atomicAdd(&cnt_s[i0], n);
        if (w.vb & 2u) atomicAdd(&cnt_s[i0 + 1], n);
        if (w.vb & 4u) atomicAdd(&cnt_s[i0 + P.tile_w], n);
        if (w.vb & 8u) atomicAdd(&cnt_s[i0 + P.tile_w + 1], n);
      }
      continue;
    }
    const EvCand k = candidates(base + tid, j, c, y, x);
    if (P.ncand == 2) {
      const uint32_t vb = window_bits(k);
      const int ly = k.oy_min - oy0, lx = k.ox_min - ox0;
      const int32_t key = vb ? (((ly + 2) << 13) | ((lx + 2) << 4) | (int32_t)vb) : -1;
      const uint32_t same = __match_any_sync(kAll, key);
      if (vb && (__ffs(same) - 1) == lane) {
        const int32_t n = __popc(same);
        const int i0 = ly * P.tile_w + lx;  // slot (0, 0); used only if valid
        if (vb & 1u) atomicAdd(&cnt_s[i0], n);
        if (vb & 2u) atomicAdd(&cnt_s[i0 + 1], n);
        if (vb & 4u) atomicAdd(&cnt_s[i0 + P.tile_w], n);
        if (vb & 8u) atomicAdd(&cnt_s[i0 + P.tile_w + 1], n);
      }
    } else {
      for (int a = 0; a < P.ncand; ++a)
        for (int bb = 0; bb < P.ncand; ++bb) {
          const int oy = k.oy_min + a, ox = k.ox_min + bb;
          const bool ok = oy >= k.oy_lo && oy <= k.oy_hi && ox >= k.ox_lo && ox <= k.ox_hi;
          const int pl = ok ? (oy - oy0) * P.tile_w + (ox - ox0) : -1;
          const uint32_t same = __match_any_sync(kAll, pl);
          if (ok && (__ffs(same) - 1) == lane) atomicAdd(&cnt_s[pl], __popc(same));
        }
    }
  }
  __syncthreads();

  // queue offsets (kept lengths, position order) and the walk order (one thread per position;
  // the host keeps NPM <= blockDim)
  {
    const bool real = tid < NPM && tid / P.tile_w < th && tid % P.tile_w < tw;
    const int32_t nk = real ? min(cnt_s[tid], P.L) : 0;
    int32_t tot;
    const int32_t qoff = block_exclusive_scan(nk, s_scan, tot);
    int bk = 0, rk = 0;
    if (tid < NPM) off_s[tid] = qoff;
    if (real) {
      bk = length_bucket(nk);
      rk = atomicAdd(&bucket_s[bk], 1);
    }
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the 64 bucket sizes, two per lane
      const int32_t v0 = bucket_s[2 * lane], v1 = bucket_s[2 * lane + 1];
      int32_t incl = v0 + v1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t n = __shfl_up_sync(kAll, incl, o);
        if (lane >= o) incl += n;
      }
      const int32_t ex = incl - v0 - v1;
      bucket_s[2 * lane] = ex;
      bucket_s[2 * lane + 1] = ex + v0;
    }
    __syncthreads();
    if (real) order_s[bucket_s[bk] + rk] = tid;
  }

  // -------- 2. queue entries, 256 events (one per thread) at a time in arrival order.  The
  // chunk bitmasks and event times are double-buffered, so a chunk needs two block barriers:
  // after bucketing and after the column scan; the scan also retires the previous chunk
  // (queued counts, latest event time, clearing its masks).
  const uint32_t lt_mask = (1u << lane) - 1u;
  int32_t prev_col = 0, prev_last = -1;
  int par = 0;
#pragma unroll 1
  for (int32_t base = 0; base < nev; base += THREADS, par ^= 1) {  // block-uniform
    uint32_t* mask_c = mask_s + par * CHW * NPM;
    float* evt_c = evt_s + par * THREADS;
    int32_t j = 0, c = 0, y = 0, x = 0;
    const int32_t e = base + tid;
    EvCand k{0, 1, 0, 0, 1, 0};
    Win w{0, 0, 0u, 0};
    if constexpr (WIN) w = window(e, j);
    else k = candidates(e, j, c, y, x);
    const float t = e < nev ? P.in.times[row * P.in.capacity + j] : 0.0f;
    evt_c[tid] = t;
    // bucket: one word per warp and position; the group's first lane ORs the group's lanes in
    if (WIN) {
      const int32_t key = w.vb ? (((w.ly + 2) << 13) | ((w.lx + 2) << 4) | (int32_t)w.vb) : -1;
      const uint32_t same = __match_any_sync(kAll, key);
      if (w.vb && (__ffs(same) - 1) == lane) {
        uint32_t* m0 = mask_c + warp * NPM + w.ly * P.tile_w + w.lx;  // slot (0, 0)
        if (w.vb & 1u) atomicOr(m0, same);
        if (w.vb & 2u) atomicOr(m0 + 1, same);
        if (w.vb & 4u) atomicOr(m0 + P.tile_w, same);
        if (w.vb & 8u) atomicOr(m0 + P.tile_w + 1, same);
      }
    } else if (P.ncand == 2) {
      const uint32_t vb = window_bits(k);
      const int ly = k.oy_min - oy0, lx = k.ox_min - ox0;
      const int32_t key = vb ? (((ly + 2) << 13) | ((lx + 2) << 4) | (int32_t)vb) : -1;
      const uint32_t same = __match_any_sync(kAll, key);
      if (vb && (__ffs(same) - 1) == lane) {
        uint32_t* m0 = mask_c + warp * NPM + ly * P.tile_w + lx;  // slot (0, 0)
        if (vb & 1u) atomicOr(m0, same);
        if (vb & 2u) atomicOr(m0 + 1, same);
        if (vb & 4u) atomicOr(m0 + P.tile_w, same);
        if (vb & 8u) atomicOr(m0 + P.tile_w + 1, same);
      }
    } else {
      for (int a = 0; a < P.ncand; ++a)
        for (int bb = 0; bb < P.ncand; ++bb) {
          const int oy = k.oy_min + a, ox = k.ox_min + bb;
          const bool ok = oy >= k.oy_lo && oy <= k.oy_hi && ox >= k.ox_lo && ox <= k.ox_hi;
          const int pl = ok ? (oy - oy0) * P.tile_w + (ox - ox0) : -1;
          const uint32_t same = __match_any_sync(kAll, pl);
          if (ok && (__ffs(same) - 1) == lane) atomicOr(&mask_c[warp * NPM + pl], same);
        }
    }
    __syncthreads();
    if (tid < NPM) {
      // retire the previous chunk of this position
      if (base > 0) {
        uint32_t* mask_p = mask_s + (par ^ 1) * CHW * NPM;
        run_s[tid] += prev_col;
        if (prev_last >= 0) lastt_s[tid] = evt_s[(par ^ 1) * THREADS + prev_last];
#pragma unroll
        for (int w = 0; w < CHW; ++w) mask_p[w * NPM + tid] = 0u;
      }
      // column scan: entries of this position before each warp's word
      int32_t col = 0, last = -1;
#pragma unroll
      for (int w = 0; w < CHW; ++w) {
        const uint32_t m = mask_c[w * NPM + tid];
        pre_s[w * NPM + tid] = (uint32_t)col;
        col += __popc(m);
        if (m) last = w * 32 + 31 - __clz(m);
      }
      prev_col = col;
      prev_last = last;
    }
    __syncthreads();
    if (WIN && e < nev && w.vb) {
      const int32_t tb = __float_as_int(t), sk = P.s * P.k;
#pragma unroll
      for (int sl = 0; sl < 4; ++sl) {
        if (!((w.vb >> sl) & 1u)) continue;
        const int sy = sl >> 1, sx = sl & 1;
        const int pl = (w.ly + sy) * P.tile_w + w.lx + sx;
        const uint32_t before = mask_c[warp * NPM + pl] & lt_mask;
        const int32_t qi = run_s[pl] + (int32_t)pre_s[warp * NPM + pl] + __popc(before);
        const uint32_t widx = (uint32_t)(j * SWW + sl * P.G);
        if (qi < P.L) {
          const uint32_t T = (uint32_t)((w.tap0 - sy * sk - sx * P.s) * OCP);
          q_b[off_s[pl] + qi] = make_int2(tb, (int32_t)((T << P.q_shift) | widx));
        } else {
          for (int g = 0; g < P.G; ++g) sw_b[widx + g] = 0u;
        }
      }
    } else if (!WIN && e < nev) {
      const int32_t ckk = c * KK, yp = y + P.p, xp = x + P.p;
      const int32_t tb = __float_as_int(t);
      for (int oy = k.oy_lo; oy <= k.oy_hi; ++oy)
        for (int ox = k.ox_lo; ox <= k.ox_hi; ++ox) {
          const int pl = (oy - oy0) * P.tile_w + (ox - ox0);
          const uint32_t before = mask_c[warp * NPM + pl] & lt_mask;
          const int32_t qi = run_s[pl] + (int32_t)pre_s[warp * NPM + pl] + __popc(before);
          const int slot = (oy - k.oy_min) * P.ncand + (ox - k.ox_min);
          const uint32_t widx = (uint32_t)(j * SWW + slot * P.G);
          if (qi < P.L) {
            const uint32_t T = (uint32_t)((ckk + (yp - oy * P.s) * P.k + (xp - ox * P.s)) * OCP);
            q_b[off_s[pl] + qi] = make_int2(tb, (int32_t)((T << P.q_shift) | widx));
          } else {
            for (int g = 0; g < P.G; ++g) sw_b[widx + g] = 0u;
          }
        }
    }
  }
  if (tid < NPM && prev_last >= 0)  // the last chunk's latest event per position
    lastt_s[tid] = evt_s[(par ^ 1) * THREADS + prev_last];
  __syncthreads();

  // -------- 3. walk: lane groups run whole queues, longest first, then the catch-up column
  const int32_t E = P.in.capacity;
  const int32_t n_in = P.in_nreal[b];
  const int32_t gl_idx = (int32_t)jax_index((int64_t)n_in - 1, E);
  const float global_last = P.in.time(row, gl_idx, n_eff);
  const int n_units = th * tw * P.G;
  const int ntasks = (n_units + UPW - 1) / UPW;
  int32_t acc_min = 0, acc_max = 0, acc_ovf = 0, acc_spk = 0;
  constexpr bool kPadIdentity = FORM == kStepWideNoFit;
  for (;;) {
    int task = 0;
    if (lane == 0) task = atomicAdd(&misc_s[0], 1);
    task = __shfl_sync(kAll, task, 0);
    if (task >= ntasks) break;
    const int unit = task * UPW + gi;
    const bool unit_ok = unit < n_units;
    const int ri = P.G == 1 ? unit : (int)P.fd_G.div((uint32_t)unit);
    const int g = unit - ri * P.G;
    const int pl = unit_ok ? order_s[ri] : 0;
    const int ly = (int)P.fd_tw.div((uint32_t)pl), lx = pl - ly * P.tile_w;
    const int oc = g * LPU + glane;
    const bool lane_ok = unit_ok && oc < P.oc;
    const int oy = oy0 + ly, ox = ox0 + lx;
    const int32_t n = unit_ok ? cnt_s[pl] : 0;
    const int32_t nk = min(n, P.L);
    const int2* qp = q_b + (unit_ok ? off_s[pl] : 0);
    // a layer without a threshold, and lanes past the channel count, never fire: their register
    // stays inside total_bits < 31 bits, below INT32_MAX
    int32_t vth = INT32_MAX;
    if (lane_ok && P.has_vth) vth = __ldg(&P.vth[(int64_t)oc * P.n_sp + oy * P.w_out + ox]);
    int32_t V = 0;
    float tp = 0.0f;  // time of the unit's previous queue entry (a queue starts at time 0)
    const int32_t nmax = __reduce_max_sync(kAll, nk);
    const uint32_t widx_mask = (1u << P.q_shift) - 1u;
    // each batch's entries are loaded one batch ahead (they come from L2)
    int2 ahead = glane < nk ? qp[glane] : make_int2(0, 0);
    for (int32_t b0 = 0; b0 < nmax; b0 += LPU) {
      const int32_t idx = b0 + glane;
      const bool has = idx < nk;
      const int2 en = ahead;
      if (idx + LPU < nk) ahead = qp[idx + LPU];
      // Δt to the previous entry of the same queue (the batch's first lane: the carry)
      const float te = __int_as_float(en.x);
      float tprev = __shfl_up_sync(kAll, te, 1, LPU);
      if (glane == 0) tprev = tp;
      const int32_t nb = min(nk - b0, LPU);
      const float tlast = __shfl_sync(kAll, te, nb > 0 ? nb - 1 : 0, LPU);
      if (nb > 0) tp = tlast;
      // lanes without an entry take an identity step on the zero row in the no-fit form (it
      // changes nothing: V stays inside the tracked range and below every threshold), else -1
      int32_t a = sc.ident_a, T = kPadIdentity ? zero_row : -1;
      uint32_t widx = 0;
      if (has) {
        const int32_t dt = dt_from_times(te, tprev);
        if (dt != 0) a = decay_code(dt, lut, P.qc.lut_len);
        T = (int32_t)((uint32_t)en.y >> P.q_shift);
        widx = (uint32_t)en.y & widx_mask;
      }
      const int32_t nbw = min(nmax - b0, LPU);  // warp-uniform batch length
      uint32_t myvote = 0;  // the warp's spike ballot of this lane's step
      if (PARK) {
        __syncwarp();
        park_w[lane] = make_int2(a, T);
        __syncwarp();
      }
      auto walk = [&](int st) {
        int32_t as, Ts;
        if (PARK) {
          const int2 at = park_w[st];
          as = at.x;
          Ts = at.y;
        } else {
          as = __shfl_sync(kAll, a, st, LPU);
          Ts = __shfl_sync(kAll, T, st, LPU);
        }
        bool spike = false;
        if (kPadIdentity || (Ts >= 0 && lane_ok)) {
          const int32_t qv = (int32_t)w_s[Ts + oc];
          int32_t u;
          const int32_t w = sc.step<SAT, true, FORM != kStepWideNoFit>(V, as, qv, u);
          spike = w >= vth;
          V = spike ? 0 : w;
          // overflow is read off the unfitted range at the end of the layer (layer_finish)
          acc_min = min(acc_min, u);
          acc_max = max(acc_max, u);
        }
        const uint32_t vote = __ballot_sync(kAll, spike);
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
      } else {
        for (int st = 0; st < nbw; ++st) walk(st);
      }
      if (PARK) {
        __syncwarp();
        myvote = vote_w[lane];
        __syncwarp();
      }
      if (has) {
        const uint32_t word = (myvote >> (gi * LPU)) & gmask_bits;
        sw_b[widx + g] = word;
        if (word) {
          const int32_t grp = (int32_t)(P.fd_sww.div(widx) >> kConvGroupShift);
          if (P.grp_in_smem) atomicAdd(&grp_s[grp], __popc(word));
          else atomicAdd(&chunk_spk_b[grp], __popc(word));
        }
      }
    }
    if (lane_ok) {
      // catch-up column: Δt = global last input time - this position's last event time (zero
      // when the position received nothing), weight code 0; then identity columns (U = V)
      const int pos = oy * P.w_out + ox;
      const float tp = lastt_s[pl];
      int32_t tail = 0;
      if (n < P.L) {
        const int32_t dt = n > 0 ? dt_from_times(global_last, tp) : 0;
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
        const int32_t n_ident = P.L - n - 1;
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
      if (tail) {
        atomicAdd(&P.tail_total[b], tail);
        acc_spk += tail;
      }
      if (glane == 0 && g == 0) atomicMax(&P.needed[b], n + 1);
    }
  }
  __syncthreads();
  if (P.grp_in_smem)
    for (int i = tid; i < n_groups; i += blockDim.x)
      if (grp_s[i]) atomicAdd(&chunk_spk_b[i], grp_s[i]);

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
    if (misc_s[4]) atomicAdd(&P.s_total[b], misc_s[4]);
  }
}

}  // namespace salt
