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
//  1. ffc_segment: every (segment, 32-neuron group) warp guesses the state at its segment's
//     start by a warm-up run from v = 0 over the events just before it (runs that fire at a
//     common event agree exactly from then on, so the guess is usually the exact float32 state),
//     then runs its segment from that guess v_start, writing one spike word per event and a
//     record per neuron: first spike (event, pre-reset value u1, decay product A1 up to it), the
//     largest value before it (M), the product of all decays (Aseg), the end state, the spike
//     count.
//  2. ffc_fixup: one warp per group walks the segments in order with the true incoming state
//     v_in.  A guess equal to v_in leaves nothing to do.  Otherwise, with d = v_in - v_start,
//     the true value before the guessed run's first spike is guess + A_k * d with 0 <= A_k <= 1,
//     so the records decide most segments outright: with d > 0 and M + d < v_th, or d < 0 and
//     u1 + A1 * d >= v_th, both runs fire first at the same event and agree from there on;
//     without any spike the end state is Aseg * d + guess.  Otherwise the lanes concerned re-run
//     the segment from v_in, rewriting their spike bits, until they fire at an event where the
//     guess also fired.
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
// number of events each source sent.  Block (x, b, z) adds sources z, z + gridDim.z, ... into
// the per-neuron totals.
__global__ void ffc_bound_partial(FloatLaunch P) {
  const int b = blockIdx.y;
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= P.n_out) return;
  const int32_t* h = P.hist + (int64_t)b * P.n_in;
  int32_t m = 0;
  double sum = 0.0;
  for (int s = blockIdx.z; s < P.n_in; s += gridDim.z) {
    const int32_t c = __ldg(&h[s]);
    if (c == 0) continue;
    const float w = __ldg(&P.wT[(int64_t)s * P.n_out + o]);
    if (w > 0.0f) {
      m += c;
      sum += (double)c * (double)w;
    }
  }
  if (m) {
    atomicAdd(&P.bcnt[(int64_t)b * P.n_out + o], m);
    atomicAdd(&P.bsum[(int64_t)b * P.n_out + o], sum);
  }
}

__global__ void ffc_bound(FloatLaunch P) {
  const int b = blockIdx.y;
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  int32_t extra = 0;
  if (o < P.n_out)
    extra = extra_steps_bound(P.bcnt[(int64_t)b * P.n_out + o], P.bsum[(int64_t)b * P.n_out + o],
                              P);
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

// Lane-parallel raw loads of one batch (lane e: event base + e, when before jend).
struct Raw {
  float t;
  int32_t src;
  float gain;
};

template <bool GAIN>
__device__ __forceinline__ Raw load_raw(const FloatLaunch& P, int b, int32_t base, int32_t jend,
                                        int lane) {
  Raw r{0.0f, 0, 1.0f};
  const int32_t j = base + lane;
  if (j < jend) {
    const int64_t row = (int64_t)b * P.in.capacity;
    r.t = P.in.times[row + j];
    r.src = (int32_t)jax_index(P.in.src[row + j], P.n_in);
    if (GAIN) r.gain = P.gain[row + j];
  }
  return r;
}

__device__ __forceinline__ Batch make_batch(const Raw& r, int32_t base, int32_t jend,
                                            float& tprev, int lane) {
  Batch x;
  x.src = r.src;
  x.gain = r.gain;
  float tp = __shfl_up_sync(kFull, r.t, 1);
  if (lane == 0) tp = tprev;
  x.cnt = min(32, jend - base);
  tprev = __shfl_sync(kFull, r.t, x.cnt - 1);
  x.dt = r.t - tp;
  x.row = decay_row(x.dt);
  return x;
}

template <bool GAIN>
__device__ __forceinline__ Batch load_batch(const FloatLaunch& P, int b, int32_t base,
                                            int32_t jend, float& tprev, int lane) {
  return make_batch(load_raw<GAIN>(P, b, base, jend, lane), base, jend, tprev, lane);
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

// powf for the rare gaps that the table does not hold; kept out of line so that the common
// path never evaluates it.
__device__ __noinline__ float decay_pow(float base, float dt) { return powf(base, dt); }

// a of event e for this lane's neuron.  The row is the same for all lanes, so the branch is
// warp-uniform.
__device__ __forceinline__ float decay_of(const Batch& x, int e, float base, const float* lut_s,
                                          int lane) {
  const int32_t row = __shfl_sync(kFull, x.row, e);
  if (row >= 0) return lut_s[(row << 5) + lane];
  return decay_pow(base, __shfl_sync(kFull, x.dt, e));
}

// The decay factors of the batch's 32 events for this lane's neuron, gathered before the
// recurrence so that its dependent chain holds no loads.
__device__ __forceinline__ void load_a(const Batch& x, float base, const float* lut_s, int lane,
                                       float (&av)[32]) {
  if (__any_sync(kFull, lane < x.cnt && x.row < 0)) {  // a gap beyond the table: rare
#pragma unroll
    for (int e = 0; e < 32; ++e) av[e] = decay_of(x, e, base, lut_s, lane);
  } else {  // every row is in the table
    const float* col = lut_s + lane;
    const int32_t off = x.row << 5;
#pragma unroll
    for (int e = 0; e < 32; ++e) av[e] = col[__shfl_sync(kFull, off, e)];
  }
}

// The speculative run over one batch: FULL (32 events) needs no per-event bound check; TRACK
// also keeps the decay product Ap and the batch's largest pre-reset value Mb (the exact first
// fire is recovered afterwards by first_fire).  wb[e * 32 + lane] holds event e's weight for
// this lane's neuron; bit e of the returned mask says whether this lane fired at event e.
template <bool TRACK, bool FULL, bool GAIN>
__device__ __forceinline__ uint32_t seg_batch(const Batch& x, const float (&av)[32],
                                              const float* wb, int lane, float vth, float& v,
                                              float& Ap, float& Mb) {
  uint32_t bits = 0;
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    if (FULL || e < x.cnt) {
      float w = wb[(e << 5) + lane];
      if (GAIN) w *= __shfl_sync(kFull, x.gain, e);
      v = fmaf(av[e], v, w);
      if (TRACK) {
        Ap *= av[e];
        Mb = fmaxf(Mb, v);
      }
      const bool spike = v >= vth;
      v = spike ? 0.0f : v;
      bits |= (uint32_t)spike << e;
    }
  }
  return bits;
}

// For lanes whose first fire lies in this batch (first), replays the batch from its start
// state (v0, A0) up to that fire: the largest value before it joins M, u1 is the value that
// fired and A1 the decay product up to it.  The replay repeats the same float operations, so
// it follows the batch's trajectory exactly.
template <bool GAIN>
__device__ __forceinline__ void first_fire(const Batch& x, const float (&av)[32], const float* wb,
                                           int lane, bool first, int estar, float v0, float A0,
                                           float& M, float& u1, float& A1) {
  float vv = v0, AA = A0, MM = M;
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    if (e < x.cnt) {
      float w = wb[(e << 5) + lane];
      if (GAIN) w *= __shfl_sync(kFull, x.gain, e);
      vv = fmaf(av[e], vv, w);
      AA *= av[e];
      if (first && e < estar) MM = fmaxf(MM, vv);
      if (first && e == estar) {
        u1 = vv;
        A1 = AA;
      }
    }
  }
  if (first) M = MM;
}

// 32 x 32 bit transpose across the warp: lane l's bit e becomes lane e's bit l.
__device__ __forceinline__ uint32_t transpose32(uint32_t x, int lane) {
  const uint32_t masks[5] = {0x0000ffffu, 0x00ff00ffu, 0x0f0f0f0fu, 0x33333333u, 0x55555555u};
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const int j = 16 >> i;
    const uint32_t m = masks[i];
    const uint32_t y = __shfl_xor_sync(kFull, x, j);
    x = (lane & j) ? ((x & ~m) | ((y & ~m) >> j)) : ((x & m) | ((y & m) << j));
  }
  return x;
}

// ---- asynchronous weight staging (cp.async)
__device__ __forceinline__ void cp_async16(float* smem, const float* gmem, int bytes) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async4(float* smem, const float* gmem, int bytes) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all_but_one() {
  asm volatile("cp.async.wait_group 1;\n" ::: "memory");
}

// Stages the batch's weight slices w[src_e][g*32 .. g*32+31] into wb[e*32 + k], zero for events
// past cnt and neurons past n_out, as one cp.async group.  VEC moves 16-byte pieces (needs
// n_out % 4 == 0 so that every piece is 16-byte aligned), otherwise 4-byte ones.
template <bool VEC>
__device__ __forceinline__ void stage_w(const FloatLaunch& P, const Raw& r, int cnt, int g,
                                        float* wb, int lane) {
  const int o0 = g * 32;
  if (VEC) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = lane + 32 * i, e = c >> 3, q = (c & 7) << 2;
      const int32_t s = __shfl_sync(kFull, r.src, e);
      const int bytes = e < cnt ? max(0, min(16, (P.n_out - o0 - q) * 4)) : 0;
      cp_async16(wb + e * 32 + q, bytes ? P.wT + (int64_t)s * P.n_out + o0 + q : P.wT, bytes);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int32_t s = __shfl_sync(kFull, r.src, e);
      const int bytes = (e < cnt && o0 + lane < P.n_out) ? 4 : 0;
      cp_async4(wb + e * 32 + lane, bytes ? P.wT + (int64_t)s * P.n_out + o0 + lane : P.wT,
                bytes);
    }
  }
  cp_async_commit();
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

// One warp per block (segment x, group y, sample z): blocks of one warp let the scheduler fill
// every SM evenly with the single wave of segments the host sized.  One pipelined pass covers
// the warm-up [jw, j0) and the segment [j0, j1): the weights of batch k + 1 are staged into
// shared memory (cp.async) and the events of batch k + 2 loaded while batch k runs.
template <bool GAIN, bool VEC>
__global__ void __launch_bounds__(32, kFloatSegBlocksPerSM) ffc_segment(FloatLaunch P) {
  __shared__ float lut_s[kFloatLut * 32];
  __shared__ __align__(16) float wbuf[2][32 * 32];
  const int g = blockIdx.y, b = blockIdx.z, s = blockIdx.x;
  const int lane = threadIdx.x;
  load_lut(P, g, lut_s, lane, 32);
  __syncwarp();
  const int o = g * 32 + lane;
  const bool active = o < P.n_out;
  const float base = active ? P.decay_base[o] : 1.0f;
  const float vth = P.vth;
  const int32_t n_eff = P.n_eff(b);
  int32_t j0, j1;
  segment_bounds(P, n_eff, s, j0, j1);
  uint32_t* swb = P.sw + (int64_t)b * P.sw_stride;
  int32_t* chunk = P.chunk_spikes + (int64_t)b * P.n_spk_chunks;

  // warm-up: from v = 0 over the (at most warm_max, at most half a segment) events before j0
  const int32_t warm = min(P.warm_max, ((P.seg_len(n_eff) >> 1) + 31) & ~31);
  const int32_t jw = j1 > j0 ? max(0, j0 - warm) : j0;
  float tprev = jw > 0 ? P.in.times[(int64_t)b * P.in.capacity + jw - 1] : 0.0f;
  float v = 0.0f, v_start = 0.0f;
  float Ap = 1.0f, M = -INFINITY, u1 = 0.0f, A1 = 1.0f, psum = 0.0f;
  int32_t k1 = -1, nspk = 0, pcnt = 0;
  bool mono = true;
  if (jw < j1) {
    Raw r_cur = load_raw<GAIN>(P, b, jw, j1, lane);
    stage_w<VEC>(P, r_cur, min(32, j1 - jw), g, wbuf[0], lane);
    Raw r_nxt = load_raw<GAIN>(P, b, jw + 32, j1, lane);
    int k = 0;
    for (int32_t bs = jw; bs < j1; bs += 32, ++k) {
      const Batch x = make_batch(r_cur, bs, j1, tprev, lane);
      if (bs + 32 < j1)
        stage_w<VEC>(P, r_nxt, min(32, j1 - bs - 32), g, wbuf[(k + 1) & 1], lane);
      else
        cp_async_commit();  // an empty group keeps the wait count uniform
      const Raw r_after = load_raw<GAIN>(P, b, bs + 64, j1, lane);
      float av[32];
      load_a(x, base, lut_s, lane, av);
      cp_async_wait_all_but_one();
      __syncwarp();
      const float* wb = wbuf[k & 1];
      if (bs == j0) v_start = v;
      if (bs < j0) {  // warm-up: state only
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if (e < x.cnt) {
            float w = wb[(e << 5) + lane];
            if (GAIN) w *= __shfl_sync(kFull, x.gain, e);
            v = fmaf(av[e], v, w);
            v = v >= vth ? 0.0f : v;
          }
        }
      } else {
        mono &= __all_sync(kFull, lane >= x.cnt || x.dt >= 0.0f);
        if (GAIN) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float w = wb[(e << 5) + lane] * __shfl_sync(kFull, x.gain, e);
            pcnt += w > 0.0f;
            psum += fmaxf(w, 0.0f);
          }
        }
        // Until every lane has fired once, track the first fire and the values before it.
        const bool track = __any_sync(kFull, active && k1 < 0);
        const float v0 = v, A0 = Ap;
        float Mb = -INFINITY;
        uint32_t bits;
        if (x.cnt == 32)
          bits = track ? seg_batch<true, true, GAIN>(x, av, wb, lane, vth, v, Ap, Mb)
                       : seg_batch<false, true, GAIN>(x, av, wb, lane, vth, v, Ap, Mb);
        else
          bits = track ? seg_batch<true, false, GAIN>(x, av, wb, lane, vth, v, Ap, Mb)
                       : seg_batch<false, false, GAIN>(x, av, wb, lane, vth, v, Ap, Mb);
        if (track) {
          const bool first = k1 < 0 && bits != 0;
          if (k1 < 0 && bits == 0) M = fmaxf(M, Mb);  // still silent: every value was before
          if (__any_sync(kFull, first)) {
            const int estar = __ffs(bits) - 1;
            first_fire<GAIN>(x, av, wb, lane, first, estar, v0, A0, M, u1, A1);
            if (first) k1 = bs + estar;
          }
        }
        nspk += __popc(bits);
        const uint32_t word = transpose32(bits, lane);  // lane e: the group's fires at event e
        if (lane < x.cnt) swb[(int64_t)(bs + lane) * P.G + g] = word;
        const int32_t tot = warp_sum(__popc(bits));
        if (lane == 0 && tot) atomicAdd(&chunk[bs >> kSpkChunkShift], tot);
      }
      __syncwarp();  // this buffer is restaged for batch k + 2
      r_cur = r_nxt;
      r_nxt = r_after;
    }
  }
  if (active) {
    const int64_t r = ((int64_t)b * P.S + s) * P.n_out + o;
    P.r_vstart[r] = v_start;
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
    float vstart = 0.0f, vend = 0.0f, u1 = 0.0f, A1 = 1.0f, M = -INFINITY, Aseg = 1.0f;
    int32_t k1 = -1, nspk = 0;
    if (active) {
      vstart = P.r_vstart[r];
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
    const float d = v_in - vstart;
    if (!active || v_in == vstart) {
      spk += nspk;  // the guess was the true incoming state
    } else if (!(base_ok && mono)) {
      need = true;  // no usable bound: re-run
    } else if (k1 < 0) {
      if (d <= 0.0f || M + d < vth - margin)
        v_out = fmaf(Aseg, d, vend);  // no fire in the true run either
      else
        need = true;
    } else if (d > 0.0f ? (M + d < vth - margin) : (u1 + A1 * d >= vth + margin)) {
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

// float/scan.py:67-116 for the groups that ffc_fixup flagged: per neuron, the number of
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

cudaError_t float_fc_launch(const FloatLaunch& P, cudaStream_t st, int64_t* launches,
                            cudaEvent_t seg_start, cudaEvent_t seg_stop) {
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
    const int split = std::max(1, std::min(P.n_in, 1184 / std::max(1, ((P.n_out + 127) / 128) * B)));
    ffc_bound_partial<<<dim3((P.n_out + 127) / 128, B, split), 128, 0, st>>>(P);
    FFC_LAUNCHED();
    ffc_bound<<<dim3((P.n_out + 127) / 128, B), 128, 0, st>>>(P);
    FFC_LAUNCHED();
  }
  const dim3 sg(P.S, P.G, B);
  const dim3 fg((P.G + 3) / 4, B);
  if (seg_start) {
    const cudaError_t e = cudaEventRecord(seg_start, st);
    if (e != cudaSuccess) return e;
  }
  const bool vec = P.n_out % 4 == 0;
  void* seg = gain ? (vec ? (void*)ffc_segment<true, true> : (void*)ffc_segment<true, false>)
                   : (vec ? (void*)ffc_segment<false, true> : (void*)ffc_segment<false, false>);
  // room for kFloatSegBlocksPerSM one-warp blocks of ~12 KB shared memory on every SM
  cudaError_t ce = cudaFuncSetAttribute(seg, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared);
  if (ce != cudaSuccess) return ce;
  FloatLaunch Pc = P;
  void* args[] = {&Pc};
  ce = cudaLaunchKernel(seg, sg, dim3(32), args, 0, st);
  if (ce != cudaSuccess) return ce;
  FFC_LAUNCHED();
  if (seg_stop) {
    const cudaError_t e = cudaEventRecord(seg_stop, st);
    if (e != cudaSuccess) return e;
  }
  if (gain) {
    ffc_fixup<true><<<fg, 128, 0, st>>>(P);
    FFC_LAUNCHED();
    ffc_exact<true><<<fg, 128, 0, st>>>(P);
    FFC_LAUNCHED();
  } else {
    ffc_fixup<false><<<fg, 128, 0, st>>>(P);
    FFC_LAUNCHED();
    ffc_exact<false><<<fg, 128, 0, st>>>(P);
    FFC_LAUNCHED();
  }
  return cudaSuccess;
}

}  // namespace salt
