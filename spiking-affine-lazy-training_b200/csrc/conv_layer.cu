// Integer conv layer pipeline for B200 (sm_100a).
//
// Replaces, for a batch of samples, ConvLayer.forward with QuantBackend
// (salt_core/layers/conv.py:209-234): queue construction (connectivity/conv.py:128-172), the
// integer LIF scan over every queue column (quant/scan.py:97-132), spike compaction into the
// next EventStream (stream.py:24-64, :84-100) and the layer diagnostics (layers/base.py:73-79).
//
// Kernels (one launch each, all on the caller's stream):
//   conv_tile_count / conv_tile_scan_offsets / conv_tile_scatter
//        only when the output plane is split into several tiles: a stable partition of each
//        sample's events by the tiles their receptive-field candidates fall in.
//   conv_fused   one block per (tile, sample).  Streams the tile's events in arrival order in
//        chunks; per chunk it buckets the candidates by output position with order-independent
//        shared-memory atomicOr bitmasks (so the per-position queues come out in global
//        event order, exactly the stable (position, j) order of conv.py:71), then lane groups
//        (one lane per output channel) run the integer recurrence of their position over the
//        chunk.  Spikes leave as per-(event, candidate-slot) channel bitmasks ("spike words").
//   spike_chunk_scan   per-sample exclusive scan of spike counts per event chunk.
//   conv_compact       per (event chunk, sample): emits spikes in (event, neuron) order — the
//        stable sort of stream.py:40 — into the output stream.
//   conv_tail_append / conv_truncated   rare paths: spikes on catch-up/identity columns
//        (only possible when some v_th_int <= 0) and samples whose spike count exceeds
//        max_out_spikes (the first max_out spikes in neuron-major order are kept,
//        stream.py:60, then sorted by event).
//   layer_finish       per-sample diagnostics and Capacity.fits.
#include "salt_layers.cuh"

namespace salt {

// ------------------------------------------------------------------ geometry helpers

struct Cand {  // receptive-field candidates of one event along one axis (conv.py:15-29)
  int32_t o_min;  // first candidate output coordinate (may be invalid)
  int32_t lo, hi; // valid output coordinates are [lo, hi] (empty when lo > hi)
};

__host__ __device__ __forceinline__ Cand axis_cand(int32_t i, int32_t K, int32_t S, int32_t P,
                                                   int32_t N, int32_t O) {
  Cand c;
  c.o_min = floordiv(i + P - K + S, S);   // ceil((i+P-K+1)/S)
  int32_t upper = floordiv(i + P, S);
  c.lo = max(c.o_min, 0);
  c.hi = min(min(upper, c.o_min + N - 1), O - 1);
  return c;
}

// ------------------------------------------------------------------ tile partition

__global__ void conv_tile_count(ConvLaunch P, int32_t* __restrict__ counts) {
  extern __shared__ int32_t s_cnt[];
  const int b = blockIdx.y, ch = blockIdx.x;
  for (int t = threadIdx.x; t < P.T; t += blockDim.x) s_cnt[t] = 0;
  __syncthreads();
  const int32_t n_eff = P.n_eff(b);
  for (int32_t e = threadIdx.x; e < kPartChunk; e += blockDim.x) {
    int32_t jj = ch * kPartChunk + e;
    if (jj >= n_eff) break;
    int32_t s = P.in.src[(int64_t)b * P.in.capacity + jj];
    int32_t rem = floormod(s, P.hw_in);
    int32_t y = rem / P.w_in, x = rem % P.w_in;
    Cand cy = axis_cand(y, P.k, P.s, P.p, P.ncand, P.h_out);
    Cand cx = axis_cand(x, P.k, P.s, P.p, P.ncand, P.w_out);
    if (cy.lo > cy.hi || cx.lo > cx.hi) continue;
    for (int ty = cy.lo / P.tile_h; ty <= cy.hi / P.tile_h; ++ty)
      for (int tx = cx.lo / P.tile_w; tx <= cx.hi / P.tile_w; ++tx)
        atomicAdd(&s_cnt[ty * P.tiles_x + tx], 1);
  }
  __syncthreads();
  for (int t = threadIdx.x; t < P.T; t += blockDim.x)
    counts[((int64_t)b * P.n_part_chunks + ch) * P.T + t] = s_cnt[t];
}

// One warp per sample: turns the per-(chunk, tile) counts into absolute offsets inside the
// sample's list region (tile-major, chunks in arrival order) and records each tile's length.
__global__ void conv_tile_scan_offsets(ConvLaunch P, int32_t* __restrict__ counts,
                                       int32_t* __restrict__ tile_len,
                                       int32_t* __restrict__ tile_off) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= P.batch) return;
  const int b = warp;
  int32_t tile_base = 0;
  for (int t = 0; t < P.T; ++t) {
    int32_t carry = 0;
    for (int base = 0; base < P.n_part_chunks; base += 32) {
      const int c = base + lane;
      const int64_t idx = ((int64_t)b * P.n_part_chunks + c) * P.T + t;
      const int32_t v = c < P.n_part_chunks ? counts[idx] : 0;
      int32_t incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (c < P.n_part_chunks) counts[idx] = tile_base + carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      tile_len[(int64_t)b * P.T + t] = carry;
      tile_off[(int64_t)b * P.T + t] = tile_base;
    }
    tile_base += carry;
  }
}

__global__ void conv_tile_scatter(ConvLaunch P, const int32_t* __restrict__ counts,
                                  int32_t* __restrict__ lists) {
  extern __shared__ uint32_t s_mask[];  // [T][kPartChunk/32] then word prefix [T][kPartChunk/32]
  constexpr int W = kPartChunk / 32;
  uint32_t* s_pre = s_mask + P.T * W;
  const int b = blockIdx.y, ch = blockIdx.x;
  for (int i = threadIdx.x; i < P.T * W; i += blockDim.x) s_mask[i] = 0;
  __syncthreads();
  const int32_t n_eff = P.n_eff(b);
  for (int32_t e = threadIdx.x; e < kPartChunk; e += blockDim.x) {
    int32_t jj = ch * kPartChunk + e;
    if (jj >= n_eff) break;
    int32_t s = P.in.src[(int64_t)b * P.in.capacity + jj];
    int32_t rem = floormod(s, P.hw_in);
    int32_t y = rem / P.w_in, x = rem % P.w_in;
    Cand cy = axis_cand(y, P.k, P.s, P.p, P.ncand, P.h_out);
    Cand cx = axis_cand(x, P.k, P.s, P.p, P.ncand, P.w_out);
    if (cy.lo > cy.hi || cx.lo > cx.hi) continue;
    for (int ty = cy.lo / P.tile_h; ty <= cy.hi / P.tile_h; ++ty)
      for (int tx = cx.lo / P.tile_w; tx <= cx.hi / P.tile_w; ++tx)
        atomicOr(&s_mask[(ty * P.tiles_x + tx) * W + (e >> 5)], 1u << (e & 31));
  }
  __syncthreads();
  for (int t = threadIdx.x; t < P.T; t += blockDim.x) {  // word prefix per tile
    uint32_t acc = 0;
    for (int w = 0; w < W; ++w) {
      s_pre[t * W + w] = acc;
      acc += __popc(s_mask[t * W + w]);
    }
  }
  __syncthreads();
  int32_t* list_b = lists + (int64_t)b * P.list_stride;
  for (int32_t e = threadIdx.x; e < kPartChunk; e += blockDim.x) {
    int32_t jj = ch * kPartChunk + e;
    if (jj >= n_eff) break;
    int32_t s = P.in.src[(int64_t)b * P.in.capacity + jj];
    int32_t rem = floormod(s, P.hw_in);
    int32_t y = rem / P.w_in, x = rem % P.w_in;
    Cand cy = axis_cand(y, P.k, P.s, P.p, P.ncand, P.h_out);
    Cand cx = axis_cand(x, P.k, P.s, P.p, P.ncand, P.w_out);
    if (cy.lo > cy.hi || cx.lo > cx.hi) continue;
    for (int ty = cy.lo / P.tile_h; ty <= cy.hi / P.tile_h; ++ty)
      for (int tx = cx.lo / P.tile_w; tx <= cx.hi / P.tile_w; ++tx) {
        int t = ty * P.tiles_x + tx;
        uint32_t m = s_mask[t * W + (e >> 5)] & ((1u << (e & 31)) - 1u);
        int32_t rank = (int32_t)(s_pre[t * W + (e >> 5)] + __popc(m));
        int32_t base = counts[((int64_t)b * P.n_part_chunks + ch) * P.T + t];
        list_b[base + rank] = jj;
      }
  }
}

// ------------------------------------------------------------------ fused bucket + scan

// Shared-memory event record of one chunk entry.
struct EvRec {
  float t;
  int32_t j;
  int32_t ckk;      // clamped channel * k * k (weight tap base)
  uint32_t yx;      // (y + p) << 16 | (x + p)
  uint32_t omin;    // (o_min_y + 32768) << 16 | (o_min_x + 32768)
};

template <typename WT, int LPU>
__global__ void __launch_bounds__(kFusedThreads)
conv_fused(ConvLaunch P) {
  constexpr int UPW = 32 / LPU;  // units (positions x channel groups) per warp
  constexpr int CHW = kFusedChunk / 32;
  extern __shared__ __align__(16) uint8_t smem[];
  const int b = blockIdx.y, tile = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const int gi = lane / LPU, glane = lane % LPU;
  const uint32_t gmask_bits = LPU == 32 ? 0xffffffffu : ((1u << LPU) - 1u);

  // ---- shared memory carve-up (sizes computed identically on the host)
  const int OCP = P.ocp, NPM = P.tile_h * P.tile_w, KK = P.k * P.k;
  uint8_t* sp = smem;
  WT* w_s = reinterpret_cast<WT*>(sp);
  sp += align16((size_t)P.ic * KK * OCP * sizeof(WT));
  int32_t* lut_s = reinterpret_cast<int32_t*>(sp);
  sp += align16((size_t)(P.lut_in_smem ? P.qc.lut_len : 0) * 4);
  int32_t* v_s = reinterpret_cast<int32_t*>(sp);
  sp += align16((size_t)NPM * OCP * 4);
  float* tprev_s = reinterpret_cast<float*>(sp);
  sp += align16((size_t)NPM * 4);
  int32_t* cnt_s = reinterpret_cast<int32_t*>(sp);
  sp += align16((size_t)NPM * 4);
  uint32_t* mask_s = reinterpret_cast<uint32_t*>(sp);
  sp += align16((size_t)NPM * CHW * 4);
  EvRec* ev_s = reinterpret_cast<EvRec*>(sp);
  sp += align16((size_t)kFusedChunk * sizeof(EvRec));
  int32_t* ocspk_s = reinterpret_cast<int32_t*>(sp);
  sp += align16((size_t)OCP * 4);
  int32_t* misc_s = reinterpret_cast<int32_t*>(sp);  // [0] task counter, [1..] reductions

  // ---- tile geometry
  const int ty = tile / P.tiles_x, tx = tile % P.tiles_x;
  const int oy0 = ty * P.tile_h, ox0 = tx * P.tile_w;
  const int th = min(P.tile_h, P.h_out - oy0), tw = min(P.tile_w, P.w_out - ox0);

  // ---- init
  for (int i = tid; i < P.ic * KK * OCP; i += blockDim.x) {
    int tap = i / OCP, oc = i % OCP;
    w_s[i] = oc < P.oc ? (WT)P.q[(int64_t)oc * P.ic * KK + tap] : (WT)0;
  }
  if (P.lut_in_smem)
    for (int i = tid; i < P.qc.lut_len; i += blockDim.x) lut_s[i] = P.lut[i];
  for (int i = tid; i < NPM * OCP; i += blockDim.x) v_s[i] = 0;
  for (int i = tid; i < NPM; i += blockDim.x) {
    tprev_s[i] = 0.0f;
    cnt_s[i] = 0;
  }
  for (int i = tid; i < OCP; i += blockDim.x) ocspk_s[i] = 0;
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

  // lane-level accumulators for the block reductions
  int32_t acc_min = 0, acc_max = 0, acc_ovf = 0, acc_spk = 0;
  const int ntasks = (NPM * P.G + UPW - 1) / UPW;
  __syncthreads();

  for (int32_t base = 0; base < nev; base += kFusedChunk) {
    // -------- phase 1: load chunk, bucket by position (bitmask per position)
    for (int i = tid; i < NPM * CHW; i += blockDim.x) mask_s[i] = 0;
    if (tid == 0) misc_s[0] = 0;
    __syncthreads();
    const int32_t nchunk = min(kFusedChunk, nev - base);
    for (int e = tid; e < nchunk; e += blockDim.x) {
      int32_t j = list ? list[base + e] : base + e;
      float t = P.in.times[row * P.in.capacity + j];
      int32_t s = P.in.src[row * P.in.capacity + j];
      int32_t c = floordiv(s, P.hw_in);
      int32_t rem = floormod(s, P.hw_in);
      int32_t y = rem / P.w_in, x = rem % P.w_in;
      Cand cy = axis_cand(y, P.k, P.s, P.p, P.ncand, P.h_out);
      Cand cx = axis_cand(x, P.k, P.s, P.p, P.ncand, P.w_out);
      EvRec r;
      r.t = t;
      r.j = j;
      r.ckk = (int32_t)jax_index(c, P.ic) * KK;
      r.yx = ((uint32_t)(y + P.p) << 16) | (uint32_t)(x + P.p);
      r.omin = ((uint32_t)(cy.o_min + 32768) << 16) | (uint32_t)(cx.o_min + 32768);
      ev_s[e] = r;
      int lo_y = max(cy.lo, oy0), hi_y = min(cy.hi, oy0 + th - 1);
      int lo_x = max(cx.lo, ox0), hi_x = min(cx.hi, ox0 + tw - 1);
      for (int oy = lo_y; oy <= hi_y; ++oy)
        for (int ox = lo_x; ox <= hi_x; ++ox)
          atomicOr(&mask_s[((oy - oy0) * P.tile_w + (ox - ox0)) * CHW + (e >> 5)],
                   1u << (e & 31));
    }
    __syncthreads();

    // -------- phase 2: lane groups run their position's queue over this chunk
    for (;;) {
      int task = 0;
      if (lane == 0) task = atomicAdd(&misc_s[0], 1);
      task = __shfl_sync(0xffffffffu, task, 0);
      if (task >= ntasks) break;
      const int unit = task * UPW + gi;
      const int pl = unit / P.G, g = unit % P.G;
      const int ly = pl / P.tile_w, lx = pl % P.tile_w;
      const bool unit_ok = pl < NPM && ly < th && lx < tw;
      const int oc = g * LPU + glane;
      const bool lane_ok = unit_ok && oc < P.oc;
      const int oy = oy0 + ly, ox = ox0 + lx, pos = oy * P.w_out + ox;
      int32_t V = 0, cn = 0, vth = 0;
      float tp = 0.0f;
      if (unit_ok) {
        V = v_s[pl * OCP + oc];
        tp = tprev_s[pl];
        cn = cnt_s[pl];
      }
      if (lane_ok && P.has_vth) vth = P.vth[(int64_t)oc * P.n_sp + pos];
      // Groups without a unit in this tile start exhausted: they must not walk any mask row.
      const uint32_t* mrow = mask_s + (unit_ok ? pl : 0) * CHW;
      int wi = unit_ok ? 0 : CHW;
      uint32_t cur = unit_ok ? mrow[0] : 0u;
      int32_t spk_visit = 0;
      for (;;) {
        while (cur == 0u && wi < CHW - 1) cur = mrow[++wi];
        const bool has = cur != 0u;
        if (!__any_sync(0xffffffffu, has)) break;
        bool spike = false;
        int e = 0;
        if (has) {
          e = wi * 32 + __ffs(cur) - 1;
          cur &= cur - 1u;
          const EvRec r = ev_s[e];
          if (cn < P.L) {
            int32_t dt = dt_from_times(r.t, tp);
            tp = r.t;
            int32_t a = decay_code(dt, lut, P.qc.lut_len);
            int32_t ky = (int32_t)(r.yx >> 16) - oy * P.s;
            int32_t kx = (int32_t)(r.yx & 0xffffu) - ox * P.s;
            int32_t qv = (int32_t)w_s[(r.ckk + ky * P.k + kx) * OCP + oc];
            int32_t u;
            bool ovf;
            int32_t w = quant_step(V, a, dt == 0, qv, P.qc, u, ovf);
            spike = lane_ok && P.has_vth && w >= vth;
            V = spike ? 0 : w;
            if (lane_ok) {
              acc_min = min(acc_min, u);
              acc_max = max(acc_max, u);
              acc_ovf |= (int32_t)ovf;
            }
          }
          ++cn;
        }
        const uint32_t bal = __ballot_sync(0xffffffffu, spike);
        if (has && glane == 0) {
          const EvRec r = ev_s[e];
          const int sy = oy - ((int32_t)(r.omin >> 16) - 32768);
          const int sx = ox - ((int32_t)(r.omin & 0xffffu) - 32768);
          const uint32_t bits = (bal >> (gi * LPU)) & gmask_bits;
          sw_b[((int64_t)r.j * P.nslots + sy * P.ncand + sx) * P.G + g] = bits;
          if (bits) atomicAdd(&chunk_spk_b[r.j >> kSpkChunkShift], __popc(bits));
        }
        spk_visit += spike;
      }
      if (unit_ok) {
        v_s[pl * OCP + oc] = V;
        if (glane == 0 && g == 0) {
          tprev_s[pl] = tp;
          cnt_s[pl] = cn;
        }
        if (spk_visit && oc < P.oc) atomicAdd(&ocspk_s[oc], spk_visit);
      }
      acc_spk += spk_visit;
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
    if (task >= ntasks) break;
    const int unit = task * UPW + gi;
    const int pl = unit / P.G, g = unit % P.G;
    const int ly = pl / P.tile_w, lx = pl % P.tile_w;
    const bool unit_ok = pl < NPM && ly < th && lx < tw;
    const int oc = g * LPU + glane;
    if (unit_ok && oc < P.oc) {
      const int oy = oy0 + ly, ox = ox0 + lx, pos = oy * P.w_out + ox;
      int32_t V = v_s[pl * OCP + oc];
      const int32_t cn = cnt_s[pl];
      const float tp = tprev_s[pl];
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
        atomicAdd(&ocspk_s[oc], tail);
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
    if (misc_s[4]) atomicAdd(&P.s_total[b], misc_s[4]);
  }
  for (int oc = tid; oc < P.oc; oc += blockDim.x)
    if (ocspk_s[oc]) atomicAdd(&P.oc_total[(int64_t)b * P.oc + oc], ocspk_s[oc]);
}

// ------------------------------------------------------------------ compaction

// Emits the spikes of events [c*CHC, (c+1)*CHC) of sample b, in (event, neuron) order.
__global__ void __launch_bounds__(kCompactThreads)
conv_compact(ConvLaunch P, salt_stream_out out) {
  __shared__ int32_t s_scan[kScanSmem];
  const int b = blockIdx.y, c = blockIdx.x, tid = threadIdx.x;
  const int32_t S = P.s_total[b];
  if (S > P.M) return;  // truncated samples go through conv_truncated
  const int32_t n_eff = P.n_eff(b);
  const int32_t j = c * kSpkChunk + tid;
  const bool ok = j < n_eff;
  const uint32_t* sw_j = P.sw + (int64_t)b * P.sw_stride + (int64_t)j * P.nslots * P.G;
  int32_t cnt = 0;
  Cand cy{}, cx{};
  if (ok) {
    int32_t s = P.in.src[(int64_t)b * P.in.capacity + j];
    int32_t rem = floormod(s, P.hw_in);
    int32_t y = rem / P.w_in, x = rem % P.w_in;
    cy = axis_cand(y, P.k, P.s, P.p, P.ncand, P.h_out);
    cx = axis_cand(x, P.k, P.s, P.p, P.ncand, P.w_out);
    for (int oy = cy.lo; oy <= cy.hi; ++oy)
      for (int ox = cx.lo; ox <= cx.hi; ++ox) {
        const int slot = (oy - cy.o_min) * P.ncand + (ox - cx.o_min);
        for (int g = 0; g < P.G; ++g) cnt += __popc(sw_j[slot * P.G + g]);
      }
  }
  int32_t total;
  int32_t off = block_exclusive_scan(cnt, s_scan, total);
  if (cnt == 0) return;
  const int32_t base = P.chunk_off[(int64_t)b * P.n_spk_chunks + c] + off;
  const float t = P.in.time(b, j, n_eff);
  float* ot = out.times + (int64_t)b * P.M;
  int32_t* os = out.src + (int64_t)b * P.M;
  int32_t k = 0;
  const int lpu = P.lpu;
  for (int g = 0; g < P.G; ++g) {
    uint32_t uni = 0;
    for (int oy = cy.lo; oy <= cy.hi; ++oy)
      for (int ox = cx.lo; ox <= cx.hi; ++ox)
        uni |= sw_j[((oy - cy.o_min) * P.ncand + (ox - cx.o_min)) * P.G + g];
    while (uni) {
      const int bit = __ffs(uni) - 1;
      uni &= uni - 1u;
      const int oc = g * lpu + bit;
      for (int oy = cy.lo; oy <= cy.hi; ++oy)
        for (int ox = cx.lo; ox <= cx.hi; ++ox) {
          const uint32_t wd = sw_j[((oy - cy.o_min) * P.ncand + (ox - cx.o_min)) * P.G + g];
          if (wd & (1u << bit)) {
            ot[base + k] = t;
            os[base + k] = oc * P.n_sp + oy * P.w_out + ox;
            ++k;
          }
        }
    }
  }
}

// Spikes on catch-up / identity columns (tail mode only): they map to the empty queue entry
// (global index = stream length, stream.py:36-38), so they sort after every real spike, in
// neuron order; their time is the input stream's last entry.
__global__ void conv_tail_append(ConvLaunch P, salt_stream_out out) {
  __shared__ int32_t s_scan[kScanSmem];
  __shared__ int32_t s_carry;
  const int b = blockIdx.x, tid = threadIdx.x;
  const int32_t S = P.s_total[b], Tb = P.tail_total[b];
  if (S > P.M || Tb == 0) return;
  const int32_t E = P.in.capacity;
  const float t = P.in.time(b, E - 1, P.n_eff(b));
  int32_t base = S - Tb;
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int64_t n0 = 0; n0 < P.n_neurons; n0 += blockDim.x) {
    const int64_t n = n0 + tid;
    const int32_t c = n < P.n_neurons ? P.tail_cnt[(int64_t)b * P.n_neurons + n] : 0;
    int32_t total;
    const int32_t off = block_exclusive_scan(c, s_scan, total);
    for (int32_t k = 0; k < c; ++k) {
      out.times[(int64_t)b * P.M + base + s_carry + off + k] = t;
      out.src[(int64_t)b * P.M + base + s_carry + off + k] = (int32_t)n;
    }
    __syncthreads();
    if (tid == 0) s_carry += total;
    __syncthreads();
  }
}

// Samples with more spikes than max_out_spikes: keep the first M in neuron-major order
// (jnp.nonzero(size=M) over the (neuron, column) grid, stream.py:60), then emit them in
// (event, neuron) order.  One block per sample; only truncated samples do any work.
__global__ void __launch_bounds__(kCompactThreads)
conv_truncated(ConvLaunch P, salt_stream_out out, int32_t* __restrict__ scratch_hist) {
  __shared__ int32_t s_scan[kScanSmem];
  __shared__ int32_t s_cut[8];  // oc*, pos*, j_cut, tail_keep, running base
  const int b = blockIdx.x, tid = threadIdx.x;
  const int32_t S = P.s_total[b], M = P.M;
  if (S <= M || M <= 0) return;
  const int32_t n_eff = P.n_eff(b);
  int32_t* hist = scratch_hist + (int64_t)b * P.n_sp * 2;  // [n_sp] real, [n_sp] tail
  // 1. channel cut
  if (tid == 0) {
    int32_t cum = 0, occ = P.oc - 1;
    for (int oc = 0; oc < P.oc; ++oc) {
      int32_t t = P.oc_total[(int64_t)b * P.oc + oc];
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
    int32_t s = P.in.src[(int64_t)b * P.in.capacity + j];
    int32_t rem = floormod(s, P.hw_in);
    Cand cy = axis_cand(rem / P.w_in, P.k, P.s, P.p, P.ncand, P.h_out);
    Cand cx = axis_cand(rem % P.w_in, P.k, P.s, P.p, P.ncand, P.w_out);
    const uint32_t* sw_j = P.sw + (int64_t)b * P.sw_stride + (int64_t)j * P.nslots * P.G;
    for (int oy = cy.lo; oy <= cy.hi; ++oy)
      for (int ox = cx.lo; ox <= cx.hi; ++ox)
        if (sw_j[((oy - cy.o_min) * P.ncand + (ox - cx.o_min)) * P.G + gq] & (1u << bq))
          atomicAdd(&hist[oy * P.w_out + ox], 1);
  }
  if (P.tail_mode)
    for (int pos = tid; pos < P.n_sp; pos += blockDim.x)
      hist[P.n_sp + pos] = P.tail_cnt[(int64_t)b * P.n_neurons + (int64_t)occ * P.n_sp + pos];
  __syncthreads();
  if (tid == 0) {
    int32_t need = s_cut[1], cum = 0, pstar = P.n_sp - 1;
    for (int pos = 0; pos < P.n_sp; ++pos) {
      int32_t t = hist[pos] + hist[P.n_sp + pos];
      if (cum + t >= need) {
        pstar = pos;
        break;
      }
      cum += t;
    }
    int32_t r2 = need - cum;  // spikes to keep of neuron (occ, pstar), counted in column order
    s_cut[1] = pstar;
    if (r2 <= hist[pstar]) {
      s_cut[2] = r2;  // the r2-th real spike is the last kept one: located below
      s_cut[3] = 0;
    } else {
      s_cut[2] = hist[pstar] > 0 ? hist[pstar] : 0;
      s_cut[3] = r2 - hist[pstar];
    }
    s_cut[4] = 0x7fffffff;  // j_cut
  }
  __syncthreads();
  const int pstar = s_cut[1];
  // 3. locate the j of the s_cut[2]-th real spike of neuron (occ, pstar)
  if (s_cut[2] > 0) {
    int32_t seen = 0;  // block-uniform running count
    for (int32_t j0 = 0; j0 < n_eff; j0 += blockDim.x) {
      const int32_t j = j0 + tid;
      int32_t hit = 0;
      if (j < n_eff) {
        int32_t s = P.in.src[(int64_t)b * P.in.capacity + j];
        int32_t rem = floormod(s, P.hw_in);
        Cand cy = axis_cand(rem / P.w_in, P.k, P.s, P.p, P.ncand, P.h_out);
        Cand cx = axis_cand(rem % P.w_in, P.k, P.s, P.p, P.ncand, P.w_out);
        const int py = pstar / P.w_out, px = pstar % P.w_out;
        if (py >= cy.lo && py <= cy.hi && px >= cx.lo && px <= cx.hi) {
          const uint32_t* sw_j = P.sw + (int64_t)b * P.sw_stride + (int64_t)j * P.nslots * P.G;
          hit = (sw_j[((py - cy.o_min) * P.ncand + (px - cx.o_min)) * P.G + gq] >> bq) & 1u;
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
    Cand cy{}, cx{};
    const uint32_t* sw_j = P.sw + (int64_t)b * P.sw_stride + (int64_t)j * P.nslots * P.G;
    if (j < n_eff) {
      int32_t s = P.in.src[(int64_t)b * P.in.capacity + j];
      int32_t rem = floormod(s, P.hw_in);
      cy = axis_cand(rem / P.w_in, P.k, P.s, P.p, P.ncand, P.h_out);
      cx = axis_cand(rem % P.w_in, P.k, P.s, P.p, P.ncand, P.w_out);
      for (int g = 0; g < P.G; ++g)
        for (int oy = cy.lo; oy <= cy.hi; ++oy)
          for (int ox = cx.lo; ox <= cx.hi; ++ox) {
            uint32_t wd = sw_j[((oy - cy.o_min) * P.ncand + (ox - cx.o_min)) * P.G + g];
            while (wd) {
              const int bit = __ffs(wd) - 1;
              wd &= wd - 1u;
              const int64_t n = (int64_t)(g * P.lpu + bit) * P.n_sp + oy * P.w_out + ox;
              cnt += (n < nstar) || (n == nstar && j <= j_cut);
            }
          }
    } else {
      cy.lo = 1;
      cy.hi = 0;
    }
    int32_t total;
    const int32_t off = block_exclusive_scan(cnt, s_scan, total);
    if (cnt) {
      const float t = P.in.time(b, j, n_eff);
      int32_t k = written + off;
      for (int g = 0; g < P.G; ++g) {
        uint32_t uni = 0;
        for (int oy = cy.lo; oy <= cy.hi; ++oy)
          for (int ox = cx.lo; ox <= cx.hi; ++ox)
            uni |= sw_j[((oy - cy.o_min) * P.ncand + (ox - cx.o_min)) * P.G + g];
        while (uni) {
          const int bit = __ffs(uni) - 1;
          uni &= uni - 1u;
          const int oc = g * P.lpu + bit;
          for (int oy = cy.lo; oy <= cy.hi; ++oy)
            for (int ox = cx.lo; ox <= cx.hi; ++ox) {
              const uint32_t wd = sw_j[((oy - cy.o_min) * P.ncand + (ox - cx.o_min)) * P.G + g];
              const int64_t n = (int64_t)oc * P.n_sp + oy * P.w_out + ox;
              if ((wd & (1u << bit)) && ((n < nstar) || (n == nstar && j <= j_cut))) {
                ot[k] = t;
                os[k] = (int32_t)n;
                ++k;
              }
            }
        }
      }
    }
    written += total;
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
      for (int32_t k = 0; k < c; ++k) {
        ot[written + off + k] = t;
        os[written + off + k] = (int32_t)n;
      }
      written += total;
    }
  }
}

// Host-side dispatch over the (weight width, lanes per channel group) instantiations.
template <typename WT>
static void* fused_for_lpu(int lpu) {
  switch (lpu) {
    case 1: return (void*)conv_fused<WT, 1>;
    case 2: return (void*)conv_fused<WT, 2>;
    case 4: return (void*)conv_fused<WT, 4>;
    case 8: return (void*)conv_fused<WT, 8>;
    case 16: return (void*)conv_fused<WT, 16>;
    default: return (void*)conv_fused<WT, 32>;
  }
}

void* conv_fused_kernel(int wt_bytes, int lpu) {
  if (wt_bytes == 1) return fused_for_lpu<int8_t>(lpu);
  if (wt_bytes == 2) return fused_for_lpu<int16_t>(lpu);
  return fused_for_lpu<int32_t>(lpu);
}

}  // namespace salt
