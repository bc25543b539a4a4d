// Float conv layer and float per-step traces for B200 (sm_100a).
//
// Replaces ConvLayer.forward with FloatBackend (salt_core/layers/conv.py:124-149): the queue of
// build_conv_structure (connectivity/conv.py:128-172, the first max_queue_len candidates of each
// output position in event order, then the catch-up column and identity columns of :102-125),
// conv_float_values (:187-206: a = (1 - 1/tau)^Δt per position, b = w[oc, c, ky, kx] times the
// event gain on real columns), the chunked scan of float/scan.py:67-116 with process_chunk
// (float/affine.py:99-126), and the spike_step_upper_bound need (affine.py:57-88).  The output
// stream goes through the integer conv layer's compaction kernels (same per-event spike words).
//
// fconv_scan: one warp per (sample, output position, channel group); lanes are channels.  The warp
// walks the sample's events 32 at a time, keeps the ones whose receptive field holds its position
// (a ballot gives their queue columns in event order), and every lane advances its own chunked
// scan column by column.  The chunk is streamed: the prefix map (A, B) of the open chunk grows
// one column at a time (combine of affine.py:20-24, left fold), v_seq = A * v0 + B is tested
// against the threshold at every column, and a fire or a full chunk ends the step.  The
// reference composes a chunk with lax.associative_scan's tree, so for chunks of more than two
// columns the float32 roundings differ (results agree within the float tolerance); with
// chunk_size 1, the calibration setting, every operation is the reference's own.
//
// ffc_trace: the same streamed scan for FC layers (connectivity/fc.py:20-51: every neuron sees the
// whole stream, pads are identities), one thread per (sample, neuron); it produces the per-step
// trace and the potential ranges that calibration needs.
#include "salt_layers.cuh"

namespace salt {

// Float -> int keys whose integer order is the float order (for atomic max / min).
__device__ __forceinline__ int32_t float_key(float f) {
  const int32_t i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7fffffff;
}
__device__ __forceinline__ float key_float(int32_t k) {
  return __int_as_float(k >= 0 ? k : k ^ 0x7fffffff);
}

// One neuron's chunked scan, streamed column by column (float/scan.py:67-116).
struct ChunkLane {
  float v0 = 0.0f, A = 1.0f, B = 0.0f, vs = 0.0f;  // potential at the chunk start, prefix map
  float vmax = -INFINITY, vmin = INFINITY;         // over the potentials after each step
  float t0 = 0.0f;                                 // time of the open chunk's first column
  int32_t k = 0, steps = 0, p0 = 0;                // columns in the open chunk, steps, chunk start
  bool done = false;                               // max_steps steps taken

  // Per-step trace rows of this neuron (or null).
  float* v_steps = nullptr;
  float* event_ms = nullptr;
  uint8_t* spike_mask = nullptr;

  __device__ void end_step(float v, bool fire, float ms, int32_t max_steps) {
    if (v_steps) v_steps[steps] = v;
    if (event_ms) event_ms[steps] = ms;
    if (spike_mask) spike_mask[steps] = fire;
    vmax = fmaxf(vmax, v);
    vmin = fminf(vmin, v);
    v0 = v;
    A = 1.0f;
    B = 0.0f;
    k = 0;
    done = ++steps >= max_steps;
  }

  // Column col with map (a, b); t = the column's event time (NaN for a column that is idle in
  // the trace's sense).  Returns whether the neuron fired on this column.
  __device__ bool column(int32_t col, float a, float b, float t, float v_th, int32_t C,
                         int32_t max_steps) {
    if (k == 0) {
      p0 = col;
      t0 = t;
    }
    A = __fmul_rn(a, A);
    B = __fadd_rn(__fmul_rn(a, B), b);
    vs = __fadd_rn(__fmul_rn(A, v0), B);
    const bool fire = __fsub_rn(vs, v_th) >= 0.0f;  // atan_spike(v - v_th) forward
    if (fire) {
      end_step(__fmul_rn(1.0f - 1.0f, vs), true, t0, max_steps);  // soft reset (1 - s) * v
    } else if (++k == C) {
      end_step(vs, false, t0, max_steps);
    }
    return fire;
  }

  // After the last column that changes the prefix: the open chunk runs through identity maps
  // and ends silent; every later step is an identity step.  ms_at(p) gives the trace time of a
  // step that starts at column p.
  template <typename MsAt>
  __device__ void finish(int32_t next_col, int32_t C, int32_t max_steps, MsAt ms_at) {
    if (done) return;
    int32_t p = next_col;
    if (k > 0) {
      p = p0 + C;
      end_step(vs, false, t0, max_steps);
    }
    if (done) return;
    // identity steps: v stays; one range update covers them all
    vmax = fmaxf(vmax, v0);
    vmin = fminf(vmin, v0);
    if (v_steps || event_ms || spike_mask)
      for (; steps < max_steps; ++steps, p += C) {
        if (v_steps) v_steps[steps] = v0;
        if (event_ms) event_ms[steps] = ms_at(p);
        if (spike_mask) spike_mask[steps] = 0;
      }
    steps = max_steps;
    done = true;
  }
};

// spike_step_upper_bound (affine.py:57-71) minus base_scan_steps: m* = min(#b>0, floor(Σb+ / v_th)),
// steps = m* + ceil((L - m*) / C).
__device__ __forceinline__ int32_t extra_steps_bound(int32_t m_pos, double sum_pos, float v_th,
                                                     int32_t L, int32_t C, int32_t base_steps) {
  const float m_star = fminf((float)m_pos, floorf(__fdiv_rn((float)sum_pos, v_th)));
  const float steps = m_star + ceilf(__fdiv_rn((float)L - m_star, (float)C));
  return (int32_t)steps - base_steps;
}

template <bool GAIN>
__global__ void __launch_bounds__(kFConvThreads) fconv_scan(ConvLaunch P, FConvArgs X) {
  constexpr int W = kFConvThreads / 32;
  __shared__ float ev_t[W][32], ev_a[W][32], ev_g[W][GAIN ? 32 : 1];
  __shared__ int32_t ev_tap[W][32], ev_j[W][32], ev_slot[W][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  const int64_t unit = (int64_t)blockIdx.x * W + warp;
  if (unit >= (int64_t)P.n_sp * P.G) return;
  const int pos = (int)(unit / P.G), g = (int)(unit % P.G);
  const int oy0 = pos / P.w_out, ox0 = pos - (pos / P.w_out) * P.w_out;
  const int oc = g * P.lpu + lane;
  const bool act = lane < P.lpu && oc < P.oc;
  const int64_t neuron = (int64_t)oc * P.n_sp + pos;
  const int32_t E = P.in.capacity, n_eff = P.n_eff(b), n_in = P.in_nreal[b];
  const int32_t L = P.L, C = X.C;
  const int SWW = P.nslots * P.G;
  const uint32_t gmask = P.lpu == 32 ? 0xffffffffu : ((1u << P.lpu) - 1u);
  uint32_t* sw_b = P.sw + (int64_t)b * P.sw_stride;

  ChunkLane s;
  if (act && (X.v_steps || X.event_ms || X.spike_mask)) {
    const int64_t row = ((int64_t)b * P.n_neurons + neuron) * X.max_steps;
    if (X.v_steps) s.v_steps = X.v_steps + row;
    if (X.event_ms) s.event_ms = X.event_ms + row;
    if (X.spike_mask) s.spike_mask = X.spike_mask + row;
  }
  int32_t nr = 0, m_pos = 0, nspk = 0;
  double sum_pos = 0.0;
  float tprev = 0.0f, tlast = 0.0f;
  for (int32_t base = 0; base < n_eff; base += 32) {
    const int32_t j = base + lane;
    bool cand = false;
    int32_t tap = 0, slot = 0;
    if (j < n_eff) {
      int32_t c, y, x, oy_min, oy_lo, oy_hi, ox_min, ox_lo, ox_hi;
      P.decode(P.in.src[(int64_t)b * E + j], c, y, x);
      P.axis(y, P.h_out, oy_min, oy_lo, oy_hi);
      P.axis(x, P.w_out, ox_min, ox_lo, ox_hi);
      cand = oy0 >= oy_lo && oy0 <= oy_hi && ox0 >= ox_lo && ox0 <= ox_hi;
      if (cand) {
        const int ky = y + P.p - oy0 * P.s, kx = x + P.p - ox0 * P.s;  // inside the kernel
        tap = (c * P.k + ky) * P.k + kx;
        slot = (oy0 - oy_min) * P.ncand + (ox0 - ox_min);
      }
    }
    const uint32_t mask = __ballot_sync(0xffffffffu, cand);
    if (!mask) continue;
    const int m = __popc(mask);
    if (cand) {
      const int r = __popc(mask & ((1u << lane) - 1u));
      ev_t[warp][r] = P.in.times[(int64_t)b * E + j];
      ev_tap[warp][r] = tap;
      ev_j[warp][r] = j;
      ev_slot[warp][r] = slot;
      if (GAIN) ev_g[warp][r] = X.gain[(int64_t)b * E + j];
    }
    __syncwarp();
    const int mq = max(0, min(m, L - nr));  // candidates that get a queue column
    if (lane < mq) {  // Δt to the previous queued event (the first against t = 0)
      const float tp = lane ? ev_t[warp][lane - 1] : tprev;
      ev_a[warp][lane] = powf(X.base, __fsub_rn(ev_t[warp][lane], tp));
    }
    __syncwarp();
    for (int r = 0; r < mq; ++r) {
      float bv = 0.0f;
      if (act) {
        bv = X.wT[(int64_t)ev_tap[warp][r] * P.ocp + oc];
        if (GAIN) bv = __fmul_rn(bv, ev_g[warp][r]);
      }
      m_pos += bv > 0.0f;
      sum_pos += bv > 0.0f ? (double)bv : 0.0;
      bool fire = false;
      if (act && !s.done)
        fire = s.column(nr + r, ev_a[warp][r], bv, ev_t[warp][r], X.v_th, C, X.max_steps);
      nspk += fire;
      const uint32_t bits = __ballot_sync(0xffffffffu, fire) & gmask;
      if (lane == 0) {
        const int32_t jj = ev_j[warp][r];
        sw_b[(int64_t)jj * SWW + ev_slot[warp][r] * P.G + g] = bits;
        if (bits)
          atomicAdd(&P.chunk_spikes[(int64_t)b * P.n_spk_chunks + (jj >> kConvGroupShift)],
                    __popc(bits));
      }
    }
    if (lane >= mq && lane < m)  // candidates past the queue never fire here
      sw_b[(int64_t)ev_j[warp][lane] * SWW + ev_slot[warp][lane] * P.G + g] = 0u;
    if (mq > 0) tprev = tlast = ev_t[warp][mq - 1];
    nr += m;
    __syncwarp();
  }
  // catch-up column (conv.py:102-125): Δt = global last input time - this position's last real
  // event time (0 for a position without events), b = 0.  A fire here is a spike on an empty
  // queue entry: it sorts after every real spike (the integer path's tail spikes).
  int32_t tail = 0;
  int32_t next_col = min(nr, L);
  if (nr < L) {
    const float gl = P.in.time(b, (int32_t)jax_index((int64_t)n_in - 1, E), n_eff);
    const float a = powf(X.base, nr > 0 ? __fsub_rn(gl, tlast) : 0.0f);
    if (act && !s.done) tail = s.column(nr, a, 0.0f, __int_as_float(0x7fc00000), X.v_th, C,
                                        X.max_steps);
    next_col = nr + 1;
  }
  // trace time of an identity step starting at column p (trace.py:40-55 resolve_ms_conv)
  const float nan = __int_as_float(0x7fc00000);
  auto ms_at = [&](int32_t p) { return p >= nr ? nan : tlast; };
  if (act) s.finish(next_col, C, X.max_steps, ms_at);

  if (act) {
    X.v_final[(int64_t)b * P.n_neurons + neuron] = s.v0;
    P.tail_cnt[(int64_t)b * P.n_neurons + neuron] = tail;
    if (tail) atomicAdd(&P.tail_total[b], tail);
    atomicMax(&X.needed_extra[b],
              extra_steps_bound(m_pos, sum_pos, X.v_th, L, C, X.base_steps));
    if (X.vkey_max) {
      atomicMax(&X.vkey_max[(int64_t)b * P.oc + oc], float_key(s.vmax));
      atomicMin(&X.vkey_min[(int64_t)b * P.oc + oc], float_key(s.vmin));
    }
  }
  int32_t tot = nspk + tail;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
  if (lane == 0) {
    if (tot) atomicAdd(&P.s_total[b], tot);
    atomicMax(&P.needed[b], nr + 1);
  }
}

// Per-sample outputs: out n_real, stats, the potential ranges as floats.
__global__ void fconv_finish(ConvLaunch P, FConvArgs X, int32_t* out_nreal,
                             salt_float_conv_stats st, float* v_max, float* v_min) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (v_max && i < (int64_t)P.batch * P.oc) {
    v_max[i] = key_float(X.vkey_max[i]);
    v_min[i] = key_float(X.vkey_min[i]);
  }
  if (i >= P.batch) return;
  const int b = (int)i;
  const int32_t S = P.s_total[b], nq = P.needed[b], ex = X.needed_extra[b];
  if (out_nreal) out_nreal[b] = S;
  if (st.spike_count) st.spike_count[b] = S;
  if (st.needed_queue) st.needed_queue[b] = nq;
  if (st.needed_extra_steps) st.needed_extra_steps[b] = ex;
  if (st.fits) st.fits[b] = nq <= P.L && S <= P.M && ex <= P.max_extra;
}

// (oc, ic, k, k) -> (ic*k*k, ocp), zero-padded channels.
__global__ void fconv_transpose_w(const float* __restrict__ w, float* __restrict__ wT, int32_t oc,
                                  int32_t taps, int32_t ocp) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)taps * ocp) return;
  const int32_t t = (int32_t)(i / ocp), o = (int32_t)(i % ocp);
  wT[i] = o < oc ? w[(int64_t)o * taps + t] : 0.0f;
}

cudaError_t float_conv_launch(const ConvLaunch& P, const FConvArgs& X, const float* w,
                              float* wT, int32_t* out_nreal, const salt_float_conv_stats* st,
                              float* v_max, float* v_min, cudaStream_t stream) {
  const int32_t taps = P.ic * P.k * P.k;
  fconv_transpose_w<<<(unsigned)(((int64_t)taps * P.ocp + 255) / 256), 256, 0, stream>>>(
      w, wT, P.oc, taps, P.ocp);
  const int W = kFConvThreads / 32;
  const dim3 grid((unsigned)(((int64_t)P.n_sp * P.G + W - 1) / W), P.batch);
  if (X.gain)
    fconv_scan<true><<<grid, kFConvThreads, 0, stream>>>(P, X);
  else
    fconv_scan<false><<<grid, kFConvThreads, 0, stream>>>(P, X);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t nf = std::max<int64_t>(P.batch, v_max ? (int64_t)P.batch * P.oc : 0);
  fconv_finish<<<(unsigned)((nf + 255) / 256), 256, 0, stream>>>(
      P, X, out_nreal, st ? *st : salt_float_conv_stats{}, v_max, v_min);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ float FC traces

template <bool GAIN>
__global__ void ffc_trace(FTraceArgs T) {
  const int b = blockIdx.y;
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= T.n_out) return;
  const int32_t E = T.in.capacity, n_in = T.in_nreal[b];
  const int32_t n_eff = n_in < 0 ? 0 : (n_in < E ? n_in : E);
  const float base = T.decay_base[o];
  ChunkLane s;
  const int64_t row = ((int64_t)b * T.n_out + o) * T.max_steps;
  if (T.v_steps) s.v_steps = T.v_steps + row;
  if (T.event_ms) s.event_ms = T.event_ms + row;
  if (T.spike_mask) s.spike_mask = T.spike_mask + row;
  float tprev = 0.0f;
  int32_t col = 0;
  // fc.py:20-33: Δt to the previous entry (the first against t = 0); entries at or past n_real
  // are identities (1, 0), so the scan over them only finishes the open chunk
  for (; col < n_eff && !s.done; ++col) {
    const float t = T.in.time(b, col, n_eff);
    const float a = powf(base, __fsub_rn(t, tprev));
    tprev = t;
    float w = T.w[(int64_t)o * T.n_in + jax_index(T.in.source(b, col, n_eff), T.n_in)];
    if (GAIN) w = __fmul_rn(w, T.gain[(int64_t)b * E + col]);
    s.column(col, a, w, t, T.v_th, T.C, T.max_steps);
  }
  const float nan = __int_as_float(0x7fc00000);
  // trace.py:25-37 resolve_ms_fc: idle from n_real on, times clipped to the stream
  auto ms_at = [&](int32_t p) {
    return p >= n_in ? nan : T.in.time(b, p < E - 1 ? p : E - 1, n_eff);
  };
  s.finish(n_eff, T.C, T.max_steps, ms_at);
  if (T.v_final) T.v_final[(int64_t)b * T.n_out + o] = s.v0;
  if (T.v_max) {
    T.v_max[(int64_t)b * T.n_out + o] = s.vmax;
    T.v_min[(int64_t)b * T.n_out + o] = s.vmin;
  }
}

cudaError_t float_fc_trace_launch(const FTraceArgs& T, cudaStream_t stream) {
  const dim3 grid((unsigned)((T.n_out + 127) / 128), T.batch);
  if (T.gain)
    ffc_trace<true><<<grid, 128, 0, stream>>>(T);
  else
    ffc_trace<false><<<grid, 128, 0, stream>>>(T);
  return cudaGetLastError();
}

}  // namespace salt
