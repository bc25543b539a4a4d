// Float FC layer for B200 (sm_100a): the float chunked affine scan.
//
// Replaces FCLayer.forward with FloatBackend (salt_core/layers/fc.py:84-106):
// fc_float_values (connectivity/fc.py:36-51: a = (1 - 1/tau)^Δt, b = w[:, src] * gain, pads
// (1, 0)), float.scan.run_layer (float/scan.py:34-50, 97-131) over process_chunk
// (float/affine.py:99-126), extract_output_events_fc (stream.py:67-81) and
// extra_steps_upper_bound (float/affine.py:57-88).
//
// The reference composes each chunk's maps with an associative scan and fires at the first
// event whose composed value reaches v_th; after a fire the next chunk starts at the following
// event from v = 0.  That is the sequential recurrence v = a * v + b with fire-and-reset at
// every event, cut short only when max_steps chunks have been used up.  Each step consumes
// either a whole chunk or the events up to a fire, so with S spikes the queue needs at most
// ceil(L / chunk) + S steps: a neuron with S <= max_extra_steps is never cut.
//
// Parallel form (neurons are independent; time is split into segments):
//  1. ffc_segment: every (segment, 32-neuron group) warp runs its segment from v = 0 (a guess
//     for the true incoming state), writing one spike word per event and a record per neuron:
//     first spike (event, pre-reset value u1, decay product A1 up to it), the largest value
//     before it (M), the product of all decays (Aseg), the end state and the spike count.
//  2. ffc_fixup: one warp per group walks the segments in order with the true incoming state
//     v_in.  Before the guessed run's first spike the true value is guess + A_k * v_in with
//     0 <= A_k <= 1, so the records decide most segments outright: with v_in > 0 and
//     M + v_in < v_th, or v_in < 0 and u1 + A1 * v_in >= v_th, both runs fire first at the same
//     event and agree from there on; without any spike the end state is Aseg * v_in + guess.
//     Otherwise the lanes concerned re-run the segment from v_in, rewriting their spike bits,
//     until they fire at an event where the guess also fired.
//  3. ffc_exact: groups holding a neuron that the step limit may cut are re-run sequentially
//     with the reference's step accounting (chunk phase, step count, cut-off).
// Spike words then go through the FC compaction (fc_layer.cu) in (event, neuron) order.
#include "salt_layers.cuh"

namespace salt {

constexpr uint32_t kFull = 0xffffffffu;

// ------------------------------------------------------------------ parameter preparation

__global__ void ffc_transpose(const float* __restrict__ w, float* __restrict__ wT, int n_out,
                              int n_in) {  // wT[i][o] = w[o][i]
  __shared__ float tile[32][33];
  const int i0 = blockIdx.x * 32, o0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int o = o0 + r, i = i0 + threadIdx.x;
    if (o < n_out && i < n_in) tile[r][threadIdx.x] = w[(int64_t)o * n_in + i];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int i = i0 + r, o = o0 + threadIdx.x;
    if (o < n_out && i < n_in) wT[(int64_t)i * n_out + o] = tile[threadIdx.x][r];
  }
}

// lut[d][o] = base_o ^ d for whole d in [0, kFloatLut): the same powf the scan would call.
__global__ void ffc_lut(const float* __restrict__ decay_base, float* __restrict__ lut, int n_out) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= (int64_t)kFloatLut * n_out) return;
  const int d = (int)(k / n_out), o = (int)(k % n_out);
  lut[k] = powf(decay_base[o], (float)d);
}

// Real events per source (the no-gain form of spike_step_upper_bound's sums).
__global__ void ffc_hist(FloatLaunch P) {
  const int b = blockIdx.y;
  const int32_t n_eff = P.n_eff(b);
  for (int32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < n_eff; j += gridDim.x * blockDim.x) {
    const int32_t s = (int32_t)jax_index(P.in.src[(int64_t)b * P.in.capacity + j], P.n_in);
    atomicAdd(&P.hist[(int64_t)b * P.n_in + s], 1);
  }
}

// float/affine.py:57-88 for one neuron from its count and sum of positive b, in the
// reference's float32 arithmetic; returns extra_steps_upper_bound.
__device__ __forceinline__ int32_t extra_steps_bound(int32_t m_pos, double sum_pos,
                                                     const FloatLaunch& P) {
  const float energy = floorf((float)sum_pos / P.vth);
  const float m_star = fminf((float)m_pos, energy);
  const float steps = m_star + ceilf(((float)P.in.capacity - m_star) / (float)P.C);
  return __float2int_rz(steps) - P.base_steps;
}

// With unit gains b = w[o][src], so the sums over events are sums over sources weighted by the
// number of events each source sent.
__global__ void ffc_bound(FloatLaunch P) {
  const int b = blockIdx.y;
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  const int32_t* h = P.hist + (int64_t)b * P.n_in;
  int32_t m = 0;
  double sum = 0.0;
  if (o < P.n_out)
    for (int s = 0; s < P.n_in; ++s) {
      const int32_t c = __ldg(&h[s]);
      if (c == 0) continue;  // uniform across the block
      const float w = __ldg(&P.wT[(int64_t)s * P.n_out + o]);
      if (w > 0.0f) {
        m += c;
        sum += (double)c * (double)w;
      }
    }
  int32_t extra = o < P.n_out ? extra_steps_bound(m, sum, P) : 0;
  extra = max(extra, __shfl_xor_sync(kFull, extra, 16));
  extra = max(extra, __shfl_xor_sync(kFull, extra, 8));
  extra = max(extra, __shfl_xor_sync(kFull, extra, 4));
  extra = max(extra, __shfl_xor_sync(kFull, extra, 2));
  extra = max(extra, __shfl_xor_sync(kFull, extra, 1));
  if ((threadIdx.x & 31) == 0) atomicMax(&P.needed[b], extra);
}

// ------------------------------------------------------------------ shared event handling

// Decay row of Δt: 0 for Δt = 0 (a = 1), d for whole 0 < d < kFloatLut, -1 for powf.
__device__ __forceinline__ int32_t decay_row(float dt) {
  if (dt == 0.0f) return 0;
  const int di = __float2int_rz(dt);
  return ((float)di == dt && di > 0 && di < kFloatLut) ? di : -1;
}

// One 32-event batch starting at `base` (< jend), prepared lane-parallel: lane e holds event
// base + e.  dt against the previous event (the first event of the stream against t = 0,
// connectivity/fc.py:26-29); tprev carries across batches.
struct Batch {
  float dt;
  int32_t row, src;
  float gain;
  int cnt;
};

template <bool GAIN>
__device__ __forceinline__ Batch load_batch(const FloatLaunch& P, int b, int32_t base,
                                            int32_t jend, float& tprev, int lane) {
  Batch x;
  const int32_t j = base + lane;
  const int64_t row = (int64_t)b * P.in.capacity;
  float t = 0.0f;
  x.src = 0;
  x.gain = 1.0f;
  if (j < jend) {
    t = P.in.times[row + j];
    x.src = (int32_t)jax_index(P.in.src[row + j], P.n_in);
    if (GAIN) x.gain = P.gain[row + j];
  }
  float tp = __shfl_up_sync(kFull, t, 1);
  if (lane == 0) tp = tprev;
  x.cnt = min(32, jend - base);
  tprev = __shfl_sync(kFull, t, x.cnt - 1);
  x.dt = t - tp;
  x.row = decay_row(x.dt);
  return x;
}

// b of the 32 events for this lane's neuron: w[o][src] * gain (0 for lanes that sit out).
template <bool GAIN>
__device__ __forceinline__ void load_b(const FloatLaunch& P, const Batch& x, int o, bool use,
                                       float (&bv)[32]) {
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const int32_t s = __shfl_sync(kFull, x.src, e);
    float w = (e < x.cnt && use) ? __ldg(&P.wT[(int64_t)s * P.n_out + o]) : 0.0f;
    if (GAIN) w *= __shfl_sync(kFull, x.gain, e);
    bv[e] = w;
  }
}

__device__ __forceinline__ float decay_of(const Batch& x, int e, float base, const float* lut_s,
                                          int lane) {
  const int32_t row = __shfl_sync(kFull, x.row, e);
  const float dt = __shfl_sync(kFull, x.dt, e);
  return row >= 0 ? lut_s[row * 32 + lane] : powf(base, dt);
}

// The group's decay table rows into shared memory: lut_s[d * 32 + lane].
__device__ __forceinline__ void load_lut(const FloatLaunch& P, int g, float* lut_s, int tid,
                                         int nthreads) {
  for (int k = tid; k < kFloatLut * 32; k += nthreads) {
    const int o = g * 32 + (k & 31);
    lut_s[k] = o < P.n_out ? P.lut[(int64_t)(k >> 5) * P.n_out + o] : 1.0f;
  }
}

__device__ __forceinline__ void segment_bounds(const FloatLaunch& P, int32_t n_eff, int s,
                                               int32_t& j0, int32_t& j1) {
  const int32_t len = P.seg_len(n_eff);
  j0 = min((int32_t)((int64_t)s * len), n_eff);
  j1 = (int32_t)min((int64_t)j0 + len, (int64_t)n_eff);
}

// ------------------------------------------------------------------ 1. speculative segments

template <bool GAIN>
__global__ void __launch_bounds__(32 * kFloatSegWarps, 4) ffc_segment(FloatLaunch P) {
  __shared__ float lut_s[kFloatLut * 32];
  const int g = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31;
  load_lut(P, g, lut_s, threadIdx.x, blockDim.x);
  __syncthreads();
  const int s = blockIdx.x * kFloatSegWarps + (threadIdx.x >> 5);
  if (s >= P.S) return;
  const int o = g * 32 + lane;
  const bool active = o < P.n_out;
  const float base = active ? P.decay_base[o] : 1.0f;
  const float vth = P.vth;
  const int32_t n_eff = P.n_eff(b);
  int32_t j0, j1;
  segment_bounds(P, n_eff, s, j0, j1);
  float tprev = j0 > 0 ? P.in.times[(int64_t)b * P.in.capacity + j0 - 1] : 0.0f;
  uint32_t* swb = P.sw + (int64_t)b * P.sw_stride;
  int32_t* chunk = P.chunk_spikes + (int64_t)b * P.n_spk_chunks;

  float v = 0.0f, Ap = 1.0f, M = -INFINITY, u1 = 0.0f, A1 = 1.0f, psum = 0.0f;
  int32_t k1 = -1, nspk = 0, pcnt = 0;
  bool mono = true;
  for (int32_t bs = j0; bs < j1; bs += 32) {
    const Batch x = load_batch<GAIN>(P, b, bs, j1, tprev, lane);
    mono &= __all_sync(kFull, lane >= x.cnt || x.dt >= 0.0f);
    float bv[32];
    load_b<GAIN>(P, x, o, active, bv);
    if (GAIN) {
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        pcnt += bv[e] > 0.0f;
        psum += fmaxf(bv[e], 0.0f);
      }
    }
    uint32_t mybits = 0;
    // Until every lane has fired once, also track the first fire and the values before it.
    if (__any_sync(kFull, active && k1 < 0)) {
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        if (e < x.cnt) {
          const float a = decay_of(x, e, base, lut_s, lane);
          v = fmaf(a, v, bv[e]);
          Ap *= a;
          const bool spike = v >= vth;
          const bool before = k1 < 0;
          M = (before && !spike) ? fmaxf(M, v) : M;
          const bool first = before && spike;
          A1 = first ? Ap : A1;
          u1 = first ? v : u1;
          k1 = first ? bs + e : k1;
          v = spike ? 0.0f : v;
          nspk += spike;
          const uint32_t bal = __ballot_sync(kFull, spike);
          mybits = lane == e ? bal : mybits;
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        if (e < x.cnt) {
          const float a = decay_of(x, e, base, lut_s, lane);
          v = fmaf(a, v, bv[e]);
          const bool spike = v >= vth;
          v = spike ? 0.0f : v;
          nspk += spike;
          const uint32_t bal = __ballot_sync(kFull, spike);
          mybits = lane == e ? bal : mybits;
        }
      }
    }
    if (lane < x.cnt) swb[(int64_t)(bs + lane) * P.G + g] = mybits;
    const int32_t tot = warp_sum(lane < x.cnt ? __popc(mybits) : 0);
    if (lane == 0 && tot) atomicAdd(&chunk[bs >> kSpkChunkShift], tot);
  }
  if (active) {
    const int64_t r = ((int64_t)b * P.S + s) * P.n_out + o;
    P.r_vend[r] = v;
    P.r_k1[r] = k1;
    P.r_u1[r] = u1;
    P.r_A1[r] = A1;
    P.r_M[r] = M;
    P.r_Aseg[r] = Ap;
    P.r_nspk[r] = nspk;
    if (GAIN) {
      P.r_cnt[r] = pcnt;
      P.r_sum[r] = psum;
    }
  }
  if (g == 0 && lane == 0) P.r_mono[(int64_t)b * P.S + s] = mono;
}

// ------------------------------------------------------------------ 2. fix-up in time order

template <bool GAIN>
__global__ void __launch_bounds__(128) ffc_fixup(FloatLaunch P) {
  __shared__ float lut_all[4][kFloatLut * 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x * 4 + warp, b = blockIdx.y;
  float* lut_s = lut_all[warp];
  if (g < P.G) load_lut(P, g, lut_s, lane, 32);
  __syncwarp();
  if (g >= P.G) return;
  const int o = g * 32 + lane;
  const bool active = o < P.n_out;
  const float base = active ? P.decay_base[o] : 1.0f;
  const bool base_ok = base >= 0.0f && base <= 1.0f;  // then 0 <= A_k <= 1 on sorted times
  const float vth = P.vth, margin = P.margin;
  const int32_t n_eff = P.n_eff(b);
  uint32_t* swb = P.sw + (int64_t)b * P.sw_stride;
  int32_t* chunk = P.chunk_spikes + (int64_t)b * P.n_spk_chunks;

  float v_in = 0.0f;
  int32_t spk = 0, pcnt = 0;
  double psum = 0.0;
  for (int s = 0; s < P.S; ++s) {
    const int64_t r = ((int64_t)b * P.S + s) * P.n_out + o;
    float vend = 0.0f, u1 = 0.0f, A1 = 1.0f, M = -INFINITY, Aseg = 1.0f;
    int32_t k1 = -1, nspk = 0;
    if (active) {
      vend = P.r_vend[r];
      k1 = P.r_k1[r];
      u1 = P.r_u1[r];
      A1 = P.r_A1[r];
      M = P.r_M[r];
      Aseg = P.r_Aseg[r];
      nspk = P.r_nspk[r];
      if (GAIN) {
        pcnt += P.r_cnt[r];
        psum += (double)P.r_sum[r];
      }
    }
    const bool mono = P.r_mono[(int64_t)b * P.S + s] != 0;
    bool need = false;
    float v_out = vend;
    if (!active || s == 0 || v_in == 0.0f) {
      spk += nspk;  // the guess v = 0 was the true incoming state
    } else if (!(base_ok && mono)) {
      need = true;
    } else if (k1 < 0) {
      if (v_in <= 0.0f || M + v_in < vth - margin)
        v_out = fmaf(Aseg, v_in, vend);  // no fire in the true run either
      else
        need = true;
    } else if (v_in > 0.0f ? (M + v_in < vth - margin) : (u1 + A1 * v_in >= vth + margin)) {
      spk += nspk;  // the true run fires first at k1 too, and agrees from there on
    } else {
      need = true;
    }
    if (__any_sync(kFull, need)) {
      int32_t j0, j1;
      segment_bounds(P, n_eff, s, j0, j1);
      float tprev = j0 > 0 ? P.in.times[(int64_t)b * P.in.capacity + j0 - 1] : 0.0f;
      bool act = need;
      float v = v_in;
      int32_t delta = 0;  // true fires - guessed fires over the re-run events
      for (int32_t bs = j0; bs < j1 && __any_sync(kFull, act); bs += 32) {
        const Batch x = load_batch<GAIN>(P, b, bs, j1, tprev, lane);
        float bv[32];
        load_b<GAIN>(P, x, o, act, bv);
        const uint32_t old_l = lane < x.cnt ? swb[(int64_t)(bs + lane) * P.G + g] : 0u;
        uint32_t new_l = old_l;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if (e < x.cnt) {
            const uint32_t actm = __ballot_sync(kFull, act);
            if (actm) {
              const float a = decay_of(x, e, base, lut_s, lane);
              const uint32_t old = __shfl_sync(kFull, old_l, e);
              bool spike = false;
              if (act) {
                v = fmaf(a, v, bv[e]);
                spike = v >= vth;
                v = spike ? 0.0f : v;
                const bool guessed = (old >> lane) & 1u;
                delta += (int32_t)spike - (int32_t)guessed;
                if (spike && guessed) act = false;  // in step with the guess from here on
              }
              const uint32_t nw = (old & ~actm) | __ballot_sync(kFull, spike);
              new_l = lane == e ? nw : new_l;
            }
          }
        }
        if (lane < x.cnt && new_l != old_l) swb[(int64_t)(bs + lane) * P.G + g] = new_l;
        const int32_t d = warp_sum(lane < x.cnt ? __popc(new_l) - __popc(old_l) : 0);
        if (lane == 0 && d) atomicAdd(&chunk[bs >> kSpkChunkShift], d);
      }
      if (need) {
        spk += nspk + delta;
        v_out = act ? v : vend;
      }
    }
    v_in = v_out;
  }
  if (active) {
    P.v_final[(int64_t)b * P.n_out + o] = v_in;
    P.n_spk[(int64_t)b * P.n_out + o] = spk;
  }
  const int32_t tot = warp_sum(spk);
  // A neuron with spk <= max_extra_steps needs at most ceil(L/C) + spk <= max_steps steps.
  const bool cut = P.C > 1 && active && spk > P.max_steps - P.base_steps;
  const bool any_cut = __any_sync(kFull, cut);
  int32_t extra = 0;
  if (GAIN && active) extra = extra_steps_bound(pcnt, psum, P);
  extra = max(extra, __shfl_xor_sync(kFull, extra, 16));
  extra = max(extra, __shfl_xor_sync(kFull, extra, 8));
  extra = max(extra, __shfl_xor_sync(kFull, extra, 4));
  extra = max(extra, __shfl_xor_sync(kFull, extra, 2));
  extra = max(extra, __shfl_xor_sync(kFull, extra, 1));
  if (lane == 0) {
    if (tot) atomicAdd(&P.s_total[b], tot);
    if (GAIN) atomicMax(&P.needed[b], extra);
    P.exact[(int64_t)b * P.G + g] = any_cut;
  }
}

// ------------------------------------------------------------------ 3. exact step accounting

// float/scan.py:100-131 for the groups that ffc_fixup flagged: per neuron, the number of
// events in the open step (phase) and the steps used; a step ends at a fire or after C
// events, and once max_steps steps have ended the remaining events are dropped.
template <bool GAIN>
__global__ void __launch_bounds__(128) ffc_exact(FloatLaunch P) {
  __shared__ float lut_all[4][kFloatLut * 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x * 4 + warp, b = blockIdx.y;
  if (g >= P.G || !P.exact[(int64_t)b * P.G + g]) return;  // warp-uniform
  float* lut_s = lut_all[warp];
  load_lut(P, g, lut_s, lane, 32);
  __syncwarp();
  const int o = g * 32 + lane;
  const bool active = o < P.n_out;
  const float base = active ? P.decay_base[o] : 1.0f;
  const float vth = P.vth;
  const int32_t n_eff = P.n_eff(b);
  uint32_t* swb = P.sw + (int64_t)b * P.sw_stride;
  int32_t* chunk = P.chunk_spikes + (int64_t)b * P.n_spk_chunks;
  float tprev = 0.0f, v = 0.0f;
  int32_t phase = 0, steps = 0, spk = 0;
  bool run = active && P.max_steps > 0;
  for (int32_t bs = 0; bs < n_eff; bs += 32) {
    const Batch x = load_batch<GAIN>(P, b, bs, n_eff, tprev, lane);
    float bv[32];
    load_b<GAIN>(P, x, o, run, bv);
    const uint32_t old_l = lane < x.cnt ? swb[(int64_t)(bs + lane) * P.G + g] : 0u;
    uint32_t new_l = 0;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      if (e < x.cnt) {
        const float a = decay_of(x, e, base, lut_s, lane);
        bool spike = false;
        if (run) {
          v = fmaf(a, v, bv[e]);
          spike = v >= vth;
          v = spike ? 0.0f : v;
          ++phase;
          if (spike || phase == P.C) {
            ++steps;
            phase = 0;
          }
          run = steps < P.max_steps;
        }
        spk += spike;
        const uint32_t bal = __ballot_sync(kFull, spike);
        new_l = lane == e ? bal : new_l;
      }
    }
    if (lane < x.cnt && new_l != old_l) swb[(int64_t)(bs + lane) * P.G + g] = new_l;
    const int32_t d = warp_sum(lane < x.cnt ? __popc(new_l) - __popc(old_l) : 0);
    if (lane == 0 && d) atomicAdd(&chunk[bs >> kSpkChunkShift], d);
  }
  int32_t d_spk = 0;
  if (active) {
    P.v_final[(int64_t)b * P.n_out + o] = v;
    d_spk = spk - P.n_spk[(int64_t)b * P.n_out + o];
    P.n_spk[(int64_t)b * P.n_out + o] = spk;
  }
  d_spk = warp_sum(d_spk);
  if (lane == 0 && d_spk) atomicAdd(&P.s_total[b], d_spk);
}

// ------------------------------------------------------------------ launcher

#define FFC_LAUNCHED()                                    \
  do {                                                    \
    ++*launches;                                          \
    const cudaError_t e_ = cudaGetLastError();            \
    if (e_ != cudaSuccess) return e_;                     \
  } while (0)

cudaError_t float_fc_launch(const FloatLaunch& P, cudaStream_t st, int64_t* launches) {
  const int B = P.batch;
  ffc_transpose<<<dim3((P.n_in + 31) / 32, (P.n_out + 31) / 32), dim3(32, 8), 0, st>>>(
      P.w, P.wT, P.n_out, P.n_in);
  FFC_LAUNCHED();
  const int64_t nl = (int64_t)kFloatLut * P.n_out;
  ffc_lut<<<(unsigned)((nl + 255) / 256), 256, 0, st>>>(P.decay_base, P.lut, P.n_out);
  FFC_LAUNCHED();
  const bool gain = P.gain != nullptr;
  if (!gain) {
    const int hb = std::min((P.in.capacity + 255) / 256, 64);
    ffc_hist<<<dim3(hb, B), 256, 0, st>>>(P);
    FFC_LAUNCHED();
    ffc_bound<<<dim3((P.n_out + 127) / 128, B), 128, 0, st>>>(P);
    FFC_LAUNCHED();
  }
  const dim3 sg((P.S + kFloatSegWarps - 1) / kFloatSegWarps, P.G, B);
  const dim3 fg((P.G + 3) / 4, B);
  if (gain) {
    ffc_segment<true><<<sg, 32 * kFloatSegWarps, 0, st>>>(P);
    FFC_LAUNCHED();
    ffc_fixup<true><<<fg, 128, 0, st>>>(P);
    FFC_LAUNCHED();
    ffc_exact<true><<<fg, 128, 0, st>>>(P);
    FFC_LAUNCHED();
  } else {
    ffc_segment<false><<<sg, 32 * kFloatSegWarps, 0, st>>>(P);
    FFC_LAUNCHED();
    ffc_fixup<false><<<fg, 128, 0, st>>>(P);
    FFC_LAUNCHED();
    ffc_exact<false><<<fg, 128, 0, st>>>(P);
    FFC_LAUNCHED();
  }
  return cudaSuccess;
}

}  // namespace salt
