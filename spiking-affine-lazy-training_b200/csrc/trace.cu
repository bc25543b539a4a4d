// Per-column traces of the integer layer scan (the analysis path, not the hot path).
//
// Replaces QuantBackend.scan with trace=True (salt_core/quant/backend.py:31-53 calling
// run_layer_traced quant/scan.py:83-94) together with the event times of trace.py:25-55
// (resolve_ms_conv / resolve_ms_fc with pointer = column): for every neuron, the register after
// each of its L queue columns, whether it fired there and the time of the column's event, plus a
// per-neuron record of its first overflowing column (example/quant_run.py:189-214 reads those
// for overflow forensics).
//
// One thread per (sample, neuron) rebuilds that neuron's queue straight from the stream: the
// real events whose receptive field holds the neuron, in event order (the stable lexsort of
// connectivity/conv.py:71), the first L of them queued (:57-99), then the catch-up column and
// identity columns of the three Δt regimes (:102-125).  The hot fused kernels never build these
// (n, L) arrays; this path exists for the few samples a user inspects.
#include "salt_layers.cuh"

namespace salt {

// Output pointers of a trace (any may be null).
struct TraceOut {
  int32_t* v_steps;       // (B, n, L)
  uint8_t* spike_mask;    // (B, n, L)
  float* event_ms;        // (B, n, L)
  salt_neuron_trace rec;  // (B, n) each
};

struct ColumnSink {
  const TraceOut& o;
  int64_t base;   // (b * n + neuron) * L
  int64_t nidx;   // b * n + neuron
  int32_t V = 0, vmin = 0, vmax = 0, spikes = 0, first = -1, v_before = 0, v_after = 0;
  int32_t spiked_first = 0;
  float t_first = 0.0f;

  __device__ ColumnSink(const TraceOut& out, int64_t b_, int64_t n_, int64_t n, int32_t L)
      : o(out), base((b_ * n + n_) * L), nidx(b_ * n + n_) {}

  // One column: decay code a (identity when ident), weight code q, event time (NaN if idle).
  __device__ void step(int32_t col, int32_t a, bool ident, int32_t q, bool has_vth, int32_t vth,
                       const QuantCfg& qc, float ms) {
    int32_t u;
    bool ovf;
    const int32_t prev = V;
    const int32_t w = quant_step(V, a, ident, q, qc, u, ovf);
    const bool spike = has_vth && w >= vth;
    V = spike ? 0 : w;
    vmin = min(vmin, u);
    vmax = max(vmax, u);
    spikes += spike;
    if (ovf && first < 0) {
      first = col;
      v_before = prev;
      v_after = V;
      spiked_first = spike;
      t_first = ms;
    }
    if (o.v_steps) o.v_steps[base + col] = V;
    if (o.spike_mask) o.spike_mask[base + col] = spike;
    if (o.event_ms) o.event_ms[base + col] = ms;
  }

  __device__ void finish() {
    const salt_neuron_trace& r = o.rec;
    if (r.first_overflow) r.first_overflow[nidx] = first;
    if (r.v_before) r.v_before[nidx] = v_before;
    if (r.v_after) r.v_after[nidx] = v_after;
    if (r.spiked) r.spiked[nidx] = spiked_first;
    if (r.time_ms) r.time_ms[nidx] = t_first;
    if (r.v_min) r.v_min[nidx] = vmin;
    if (r.v_max) r.v_max[nidx] = vmax;
    if (r.v_final) r.v_final[nidx] = V;
    if (r.spike_count) r.spike_count[nidx] = spikes;
  }
};

__global__ void conv_trace_kernel(ConvLaunch P, TraceOut out) {
  const int b = blockIdx.y;
  const int64_t neuron = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (neuron >= P.n_neurons) return;
  const int oc = (int)(neuron / P.n_sp);
  const int pos = (int)(neuron - (int64_t)oc * P.n_sp);
  const int oy = pos / P.w_out, ox = pos - oy * P.w_out;
  const int32_t L = P.L, E = P.in.capacity, n_in = P.in_nreal[b];
  const int32_t n_eff = P.n_eff(b);
  const int64_t row = b;
  const int32_t vth = P.has_vth ? P.vth[neuron] : 0;
  const float nan = __int_as_float(0x7fc00000);
  ColumnSink sink(out, b, neuron, P.n_neurons, L);
  int32_t nr = 0;           // real events of this position (all of them, even beyond L)
  float t_prev = 0.0f;      // time of the previous queued event (column 0 against t = 0)
  float t_last = 0.0f;      // time of the last queued real event
  for (int32_t j = 0; j < n_eff; ++j) {
    const int32_t s = P.in.src[row * E + j];
    const int32_t c = floordiv(s, P.hw_in);       // connectivity/conv.py:32-43
    const int32_t rem = floormod(s, P.hw_in);
    const int32_t y = rem / P.w_in, x = rem - (rem / P.w_in) * P.w_in;
    const int32_t ky = y + P.p - oy * P.s, kx = x + P.p - ox * P.s;
    if (ky < 0 || ky >= P.k || kx < 0 || kx >= P.k) continue;
    if (nr < L) {
      const float t = P.in.times[row * E + j];
      const int32_t dt = dt_from_times(t, t_prev);
      const int32_t cc = (int32_t)jax_index(c, P.ic);
      const int32_t q = P.q[(((int64_t)oc * P.ic + cc) * P.k + ky) * P.k + kx];
      sink.step(nr, decay_code(dt, P.lut, P.qc.lut_len), dt == 0, q, P.has_vth, vth, P.qc, t);
      t_prev = t;
      t_last = t;
    }
    ++nr;
  }
  if (nr < L) {
    // catch-up column: Δt = global last input time - this position's last real event time
    // (zero for an empty position); weight code 0
    const float global_last = P.in.time(row, (int32_t)jax_index((int64_t)n_in - 1, E), n_eff);
    const int32_t dt = nr > 0 ? dt_from_times(global_last, t_last) : 0;
    sink.step(nr, decay_code(dt, P.lut, P.qc.lut_len), dt == 0, 0, P.has_vth, vth, P.qc, nan);
    for (int32_t col = nr + 1; col < L; ++col)  // identity columns
      sink.step(col, 0, true, 0, P.has_vth, vth, P.qc, nan);
  }
  sink.finish();
}

__global__ void fc_trace_kernel(FCLaunch P, TraceOut out) {
  const int b = blockIdx.y;
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= P.n_out) return;
  const int32_t L = P.in.capacity, n_in = P.in_nreal[b], n_eff = P.n_eff(b);
  const int32_t vth = P.has_vth ? P.vth[o] : 0;
  const float nan = __int_as_float(0x7fc00000);
  ColumnSink sink(out, b, o, P.n_out, L);
  float t_prev = 0.0f;
  for (int32_t j = 0; j < L; ++j) {
    // connectivity/fc.py:20-33: Δt against the previous entry (the first against t = 0), pads
    // masked to Δt = 0 and weight 0
    const float t = P.in.time(b, j, n_eff);
    const bool real = j < n_in;
    const int32_t dt = real ? dt_from_times(t, t_prev) : 0;
    t_prev = t;
    // P.qT holds the weight codes in the caller's (n_out, n_in) layout on this path
    const int32_t q =
        real ? P.qT[(int64_t)o * P.n_in + jax_index(P.in.source(b, j, n_eff), P.n_in)] : 0;
    sink.step(j, decay_code(dt, P.lut, P.qc.lut_len), dt == 0, q, P.has_vth, vth, P.qc,
              real ? t : nan);
  }
  sink.finish();
}

cudaError_t conv_trace_launch(const ConvLaunch& P, const salt_neuron_trace* rec, int32_t* v_steps,
                              uint8_t* spike_mask, float* event_ms, cudaStream_t st) {
  TraceOut o{v_steps, spike_mask, event_ms, rec ? *rec : salt_neuron_trace{}};
  conv_trace_kernel<<<dim3((unsigned)((P.n_neurons + 127) / 128), P.batch), 128, 0, st>>>(P, o);
  return cudaGetLastError();
}

cudaError_t fc_trace_launch(const FCLaunch& P, const salt_neuron_trace* rec, int32_t* v_steps,
                            uint8_t* spike_mask, float* event_ms, cudaStream_t st) {
  TraceOut o{v_steps, spike_mask, event_ms, rec ? *rec : salt_neuron_trace{}};
  fc_trace_kernel<<<dim3((unsigned)((P.n_out + 127) / 128), P.batch), 128, 0, st>>>(P, o);
  return cudaGetLastError();
}

}  // namespace salt
