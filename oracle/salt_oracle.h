/*
 * CPU oracle for the SALT integer event-driven forward — TEST INFRASTRUCTURE ONLY.
 *
 * A literal, single-sample restatement of the reference's JAX code path
 *   salt_core/quant/fixed_point.py, salt_core/quant/codes.py (apply_decay_table_int),
 *   salt_core/quant/scan.py, salt_core/connectivity/{conv,fc}.py, salt_core/stream.py,
 *   salt_core/layers/{conv,fc}.py forward, salt_core/capacity.py fits.
 * It builds the reference's dense (n, L) queue arrays, scans every one of the L columns for
 * every neuron, selects spikes in jnp.nonzero row-major order and stable-sorts them by the
 * global event index, exactly as the reference does.  It is deliberately NOT shaped like the
 * GPU kernels so that it checks them independently.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use this library.
 * The product path never links or calls it.
 */
#ifndef SALT_ORACLE_H
#define SALT_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { SO_ROUND = 0, SO_TRUNCATE = 1 };
enum { SO_WRAP = 0, SO_SATURATE = 1 };

/* Quantised per-layer parameters (salt_core/quant/params.py:9-21). */
typedef struct {
  const int32_t *q;        /* conv: (oc, ic, k, k); fc: (n_out, n_in) */
  const int32_t *lut;      /* decay_table_int, lut_len entries */
  int32_t lut_len;
  const int32_t *vth;      /* per-neuron integer threshold, or NULL = never fires */
  int32_t f_a, f_V, i_V;
  int32_t round_mode;      /* SO_ROUND / SO_TRUNCATE */
  int32_t overflow_mode;   /* SO_WRAP / SO_SATURATE */
} so_quant_params;

typedef struct {
  int32_t ic, h_in, w_in, oc, k, s, p;
  int32_t max_queue_len, max_out_spikes, max_extra_steps;
} so_conv_geom;

typedef struct {
  int32_t n_in, n_out;
  int32_t max_out_spikes, max_extra_steps;
} so_fc_geom;

/* Output of one layer for one sample.  Arrays are caller-allocated:
 *   v_final, vmin, vmax: n_neurons
 *   spike_mask, overflowed: n_neurons * L (may be NULL)
 *   out_times, out_src: max_out_spikes
 */
typedef struct {
  int32_t *v_final, *vmin, *vmax;
  uint8_t *spike_mask, *overflowed;
  float *out_times;
  int32_t *out_src;
  int32_t n_real_out;      /* total spikes (not clipped to max_out_spikes) */
  int32_t spike_count;     /* same as n_real_out (sum of spike_mask) */
  int32_t needed_queue;    /* conv: max(n_real per position) + 1; fc: 0 */
  int32_t any_overflow;
  int32_t vmin_all, vmax_all;
  int32_t fits;
  /* trace (quant/scan.py:83-94 run_layer_traced, trace.py:25-55 resolve_ms_*), may be NULL:
   *   v_steps  (n_neurons, L) register value after each column (after the reset)
   *   event_ms (n_neurons, L) time of the column's event, NaN for columns at or past n_real */
  int32_t *v_steps;
  float *event_ms;
} so_layer_out;

/* fixed_point.py:32-44, :47-65, :68-90 */
int32_t so_round_shift(int32_t x, int32_t shift_bits, int32_t round_mode);
int32_t so_wide_mul_shift(int32_t a, int32_t v, int32_t shift_bits, int32_t round_mode);
int32_t so_fit_to_bits(int32_t x, int32_t total_bits, int32_t overflow_mode, int32_t *overflowed);

/* quant/scan.py:22-52 — one event update; returns v_final and writes the other results. */
int32_t so_process_event(int32_t v0, int32_t a, int32_t is_identity, int32_t q, int32_t has_vth,
                         int32_t vth, int32_t f_a, int32_t f_V, int32_t i_V, int32_t round_mode,
                         int32_t overflow_mode, int32_t *is_spiked, int32_t *overflowed,
                         int32_t *v_unfitted);

/* quant/codes.py:87-105 */
void so_apply_decay_table(const float *delta_t, int64_t n, const int32_t *lut, int32_t lut_len,
                          int32_t *a_int, uint8_t *is_identity);

/* quant/scan.py:97-132 over (n, L) inputs. spike_mask/overflowed may be NULL. */
void so_run_layer(const int32_t *a_int, const uint8_t *is_identity, const int32_t *q_int,
                  const int32_t *vth, int32_t n, int32_t L, int32_t f_a, int32_t f_V, int32_t i_V,
                  int32_t round_mode, int32_t overflow_mode, uint8_t *spike_mask,
                  uint8_t *overflowed, int32_t *v_final, int32_t *vmin, int32_t *vmax);

/* connectivity/conv.py:128-172 (+ :57-125). Outputs (n_sp, L) arrays and n_real (n_sp). */
int so_conv_structure(const so_conv_geom *g, const float *times, const int32_t *src, int32_t E_len,
                      int32_t n_in, int32_t *l2g, int32_t *n_real, float *delta_t, int32_t *tap_c,
                      int32_t *tap_ky, int32_t *tap_kx);

/* connectivity/conv.py:57-99 _compress_candidates: (n_flat, j_flat) candidates -> per-position
 * queues l2g (n_sp, L) (empty = n_events) and n_real (n_sp). */
int so_compress_candidates(const int32_t *n_flat, const int32_t *j_flat, int64_t C, int32_t n_sp,
                           int32_t L, int32_t n_events, int32_t *l2g, int32_t *n_real);
/* connectivity/conv.py:102-125 _delta_t_three_regimes on (n, L) gathered times. */
void so_delta_t_regimes(const float *t_gathered, const int32_t *n_real, float global_last,
                        int32_t n, int32_t L, float *delta_t);
/* stream.py:49-100 extract_output_events_{fc,conv}: spike grid (n, steps) with the queue column
 * of every step (event_idx, NULL = the step itself), optional local_to_global_j (rows, L) tiled
 * over neurons (NULL = the column is the global index, FC), into a max_out stream. */
void so_extract_output_events(const uint8_t *mask, const int32_t *event_idx, int32_t n,
                              int32_t steps, const int32_t *l2g, int32_t l2g_rows, int32_t L,
                              const float *times, int32_t E_len, int32_t max_out, float *out_times,
                              int32_t *out_src, int32_t *n_real_out);

/* Whole layers (layers/conv.py:124-149, layers/fc.py:84-101 with QuantBackend). */
int so_conv_forward(const so_conv_geom *g, const so_quant_params *qp, const float *times,
                    const int32_t *src, int32_t E_len, int32_t n_in, so_layer_out *out);
int so_fc_forward(const so_fc_geom *g, const so_quant_params *qp, const float *times,
                  const int32_t *src, int32_t E_len, int32_t n_in, so_layer_out *out);

/* Multi-threaded batch driver used only as the timed CPU baseline: runs a chain of layers over
 * B samples with `threads` workers (one sample per task).  kinds[l]: 0 conv, 1 fc.
 * Writes the last layer's v_final (B, n_last) and per-(sample, layer) spike counts. */
typedef struct {
  int32_t kind;
  so_conv_geom conv;
  so_fc_geom fc;
  so_quant_params qp;
} so_layer_spec;

int so_network_batch(const so_layer_spec *layers, int32_t n_layers, const float *times,
                     const int32_t *src, const int32_t *n_real, int32_t B, int32_t E_len,
                     int32_t threads, int32_t *v_final_last, int32_t *spike_counts,
                     int32_t *fits);

/* ---------------------------------------------------------------- float chunked scan
 * FCLayer.forward with FloatBackend (layers/fc.py:84-106 -> build_fc_structure
 * connectivity/fc.py:20-33, fc_float_values :36-51, float/scan.py:34-50 run_layer,
 * float/affine.py:99-126 process_chunk, extract_output_events_fc stream.py:67-81,
 * extra_steps_upper_bound float/affine.py:57-88).  Float32 throughout, as XLA computes it:
 * each chunk's maps are composed in lax.associative_scan's odd/even recursion order.
 * decay_base[i] = float32(1 - 1/tau_i): one entry per neuron (the reference's scalar tau is the
 * case where all entries are equal). */
typedef struct {
  int32_t n_in, n_out, chunk_size, max_out_spikes, max_extra_steps;
  float v_th;
} so_float_fc_geom;

typedef struct {
  float *v_final;            /* (n_out) */
  uint8_t *spike_mask;       /* (n_out, max_steps) or NULL */
  int32_t *spike_event_idx;  /* (n_out, max_steps) or NULL */
  float *out_times;          /* (max_out_spikes) */
  int32_t *out_src;          /* (max_out_spikes) */
  float *out_gain;           /* (max_out_spikes) */
  int32_t n_real_out;        /* spikes in the layer (not clipped to max_out_spikes) */
  int32_t extra_steps_needed;
  int32_t fits;
  float *v_steps;            /* (n_out, max_steps) potential after each step, or NULL */
  float *event_ms;           /* (n_out, max_steps) trace.py resolve_ms_fc, or NULL */
} so_float_out;

/* max_steps = ceil(L / chunk_size) + max_extra_steps (layers/fc.py:128-130).  gain may be NULL
 * (all ones).  threads > 1 splits the neurons over worker threads. */
int so_float_fc_forward(const so_float_fc_geom *g, const float *w, const float *decay_base,
                        const float *times, const int32_t *src, const float *gain, int32_t L,
                        int32_t n_real, int32_t threads, so_float_out *out);

/* ConvLayer.forward with FloatBackend (layers/conv.py:124-149): build_conv_structure, then
 * conv_float_values (connectivity/conv.py:187-206: a = decay_base ** Δt per position, b = the
 * weight tap times the event gain on real columns), the chunked scan of float/scan.py:67-116 and
 * extract_output_events_conv (stream.py:84-100).  w is (oc, ic, k, k); gain may be NULL (ones).
 * max_steps = ceil(L / chunk_size) + max_extra_steps.  The per-step arrays (spike_mask,
 * spike_event_idx = queue column, v_steps, event_ms = trace.py:40-55) may be NULL. */
typedef struct {
  so_conv_geom conv;
  int32_t chunk_size;
  float v_th;
} so_float_conv_geom;

typedef struct {
  float *v_final;            /* (n_neurons) */
  uint8_t *spike_mask;       /* (n_neurons, max_steps) or NULL */
  int32_t *spike_event_idx;  /* (n_neurons, max_steps) or NULL */
  float *v_steps;            /* (n_neurons, max_steps) or NULL */
  float *event_ms;           /* (n_neurons, max_steps) or NULL */
  float *out_times;          /* (max_out_spikes) */
  int32_t *out_src;
  float *out_gain;
  int32_t n_real_out, needed_queue, extra_steps_needed, fits;
} so_float_conv_out;

int so_float_conv_forward(const so_float_conv_geom *g, const float *w, float decay_base,
                          const float *times, const int32_t *src, const float *gain,
                          int32_t E_len, int32_t n_in, so_float_conv_out *out);

/* Float64 yardstick of a float FC layer (test infrastructure): the layer's sequential semantics
 * (v = a*v + b with fire-and-reset at every event, a = base^dt with base = float32(1 - 1/tau)
 * widened to double; the step accounting of float/scan.py:67-116: a step ends at a fire or
 * after chunk_size events, events after max_steps steps are dropped) in double precision.
 * Outputs per neuron: v_final (double) and first_near, the first event at which the value came
 * within `near` of v_th (E_len when never).  gain may be NULL (all ones). */
int so_float_seq64(int32_t n_in, int32_t n_out, const float *w, const float *decay_base,
                   const float *times, const int32_t *src, const float *gain, int32_t E_len,
                   int32_t n_real, int32_t chunk_size, int32_t max_extra_steps, double v_th,
                   double near, double *v_final, int32_t *first_near);

/* lax.associative_scan(combine, maps) of float/affine.py:20-24 over n maps (exposed for tests). */
int so_affine_scan(const float *a, const float *b, int64_t n, float *out_a, float *out_b);

#ifdef __cplusplus
}
#endif
#endif
