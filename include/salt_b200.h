/*
 * salt_b200 — C ABI of the B200 (sm_100a) implementation of SALT's integer event-driven
 * forward pass and its float chunked affine scan.
 *
 * The reference (Salt-Shio/Spiking-Affine-Lazy-Training) is pure Python/JAX; it has no C
 * interface.  Each entry point below replaces one reference Python call (cited per entry);
 * a host binding (ctypes here, a jax.ffi custom-call handler or cgo elsewhere) passes plain
 * device pointers and sizes.  No torch, JAX or C++ types cross this boundary.
 *
 * Conventions
 *   - All array pointers are DEVICE pointers unless a comment says "host".
 *   - Batch-major layouts: a stream is (batch, capacity) row-major; per-neuron arrays are
 *     (batch, n_neurons) with neuron = oc * h_out * w_out + oy * w_out + ox for conv layers
 *     (salt_core/layers/conv.py:104-112).
 *   - Every call is asynchronous on `stream` (a cudaStream_t) and returns a status; argument
 *     errors are reported before anything is enqueued.  Capacity overflow is NOT an error: it
 *     is reported through `fits` / `needed_queue` / `n_real`, as salt_core/capacity.py:60-63.
 *   - Streams written by this library do not materialise their pad entries: entries at or
 *     beyond min(n_real, capacity) are pads whose time is 1e12 and source 0
 *     (salt_core/stream.py:42-45).  `virtual_pads = 1` tells a consumer to read them that way.
 */
#ifndef SALT_B200_H
#define SALT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t salt_status;
enum {
  SALT_OK = 0,
  SALT_BAD_ARG = 1,          /* invalid geometry, bit widths, sizes or null pointers */
  SALT_CUDA_ERROR = 2,       /* a CUDA runtime call failed; see salt_last_error() */
  SALT_NO_DEVICE = 3,        /* no sm_100 device is visible */
  SALT_WORKSPACE_TOO_SMALL = 4
};

enum { SALT_ROUND = 0, SALT_TRUNCATE = 1 };  /* salt_core/quant/fixed_point.py:20-23 */
enum { SALT_WRAP = 0, SALT_SATURATE = 1 };   /* salt_core/quant/fixed_point.py:26-29 */

/* Fixed-point settings of one quantised layer (salt_core/quant/params.py:9-21). */
typedef struct {
  int32_t f_a, f_V, i_V;   /* f_a <= 15, i_V + f_V <= 30 (fixed_point.py:15-17) */
  int32_t round_mode;      /* SALT_ROUND / SALT_TRUNCATE (network-wide in the reference) */
  int32_t overflow_mode;   /* SALT_WRAP / SALT_SATURATE */
  int32_t lut_len;         /* length of decay_table_int */
  int32_t has_vth;         /* 0: v_th_int is None, the layer never fires */
  int32_t q_bits;          /* 8 / 16 when every weight code fits int8 / int16, else 32; lets
                              the kernels stage narrower weights in shared memory */
  int32_t needs_tail;      /* 1 when some v_th_int <= 0 or some decay code is outside
                              [0, 2^f_a): only then can catch-up/identity/pad columns fire, and
                              the kernels must walk them (salt_core/quant/scan.py:65-80 applies
                              every column).  Setting it when not needed is always correct. */
} salt_quant_desc;

/* ConvLayer geometry and capacity (salt_core/layers/conv.py:23-99). */
typedef struct {
  int32_t ic, h_in, w_in, oc, k, s, p;
  int32_t max_queue_len, max_out_spikes, max_extra_steps;
} salt_conv_desc;

/* FCLayer geometry and capacity (salt_core/layers/fc.py:23-41). */
typedef struct {
  int32_t n_in, n_out;
  int32_t max_out_spikes, max_extra_steps;
} salt_fc_desc;

/* Input event stream of a layer: (batch, capacity) times/sources plus n_real per sample.
 * salt_core/stream.py:16-21 EventStream (event_gain is identically 1 on the integer path). */
typedef struct {
  const float *times;
  const int32_t *src;
  const int32_t *n_real;
  int32_t capacity;
  int32_t virtual_pads;
} salt_stream_in;

/* Output stream of a layer, capacity = the layer's max_out_spikes.  n_real[b] is the total
 * spike count (not clipped), exactly as stream.py:61 reports it. */
typedef struct {
  float *times;
  int32_t *src;
  int32_t *n_real;
} salt_stream_out;

/* Per-sample diagnostics of one layer (batch entries each).  Any pointer may be NULL.
 *   spike_count  LayerDiag.spike_count (layers/base.py:73-79)
 *   needed_queue LayerDiag.needed["max_queue_len"] = max n_real + 1 (layers/conv.py:137-141)
 *   overflowed   any(QuantLayerResult.overflowed) (example/quant_run.py:88-89)
 *   vmin / vmax  min/max of v_unfitted_min/max over neurons (example/quant_run.py:90-93)
 *   fits         Capacity.fits (capacity.py:60-63) */
typedef struct {
  int32_t *spike_count, *needed_queue, *overflowed, *vmin, *vmax, *fits;
} salt_layer_stats;

/* ---------------------------------------------------------------- conv layer
 * Replaces ConvLayer.forward with QuantBackend (salt_core/layers/conv.py:124-149 calling
 * build_conv_structure connectivity/conv.py:128-172, QuantBackend.scan quant/backend.py:31-53,
 * extract_output_events_conv stream.py:84-100, _layer_diag layers/base.py:73-79).
 *   q    (oc, ic, k, k) int32 weight codes      lut (lut_len) int32 decay_table_int
 *   vth  (oc*h_out*w_out) int32, or NULL when has_vth == 0
 *   v_final (batch, n_neurons) int32 register values after the queue (QuantLayerResult.v_final)
 * The workspace must be at least salt_conv_layer_workspace_size() bytes, 256-byte aligned. */
salt_status salt_conv_layer_workspace_size(const salt_conv_desc *layer, const salt_quant_desc *quant,
                                           int32_t batch, int32_t in_capacity, size_t *bytes);
salt_status salt_conv_layer_forward(const salt_conv_desc *layer, const salt_quant_desc *quant,
                                    const int32_t *q, const int32_t *lut, const int32_t *vth,
                                    int32_t batch, const salt_stream_in *in, salt_stream_out *out,
                                    int32_t *v_final, const salt_layer_stats *stats,
                                    void *workspace, size_t workspace_bytes, void *stream);

/* Size of the library's fixed device scratch (64 MiB), the largest conv workspace that
 * salt_conv_layer_forward_noalloc accepts. */
#define SALT_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)

/* salt_conv_layer_forward without a caller workspace, for callers that cannot allocate device
 * memory at call time (a plugin host that hands out no scratch buffers, a loop that must not
 * call cudaMalloc).  No counterpart in the reference: there JAX owns every buffer.
 *   - Same arguments, results and errors as salt_conv_layer_forward minus the workspace; the
 *     layer's scratch lives in a fixed SALT_NOALLOC_SCRATCH_BYTES device array inside the
 *     library, and the call allocates no device memory.
 *   - A layer whose salt_conv_layer_workspace_size exceeds SALT_NOALLOC_SCRATCH_BYTES is
 *     rejected with SALT_WORKSPACE_TOO_SMALL before anything is enqueued.
 *   - Nothing has to start at zero: every call clears the counters it uses, on `stream`.
 *   - The first call on a device does a one-time setup (it looks up the scratch's device
 *     address, which loads the module holding it); make that first call before any stream
 *     capture.  The address is kept for the life of the process: a context reset
 *     (cudaDeviceReset) reloads the library's device code and leaves the kept address stale, so
 *     do not call this entry point on a device after resetting it.
 *   - All calls on one device share the one scratch: calls that may overlap in time (other
 *     streams, other host threads) race and corrupt each other's results.  Order them on one
 *     stream, or with events. */
salt_status salt_conv_layer_forward_noalloc(const salt_conv_desc *layer,
                                            const salt_quant_desc *quant, const int32_t *q,
                                            const int32_t *lut, const int32_t *vth, int32_t batch,
                                            const salt_stream_in *in, salt_stream_out *out,
                                            int32_t *v_final, const salt_layer_stats *stats,
                                            void *stream);

/* ---------------------------------------------------------------- traces
 * Replace QuantBackend.scan with trace=True (salt_core/quant/backend.py:31-53 ->
 * run_layer_traced quant/scan.py:83-94) and the event times of salt_core/trace.py:25-55: for
 * every neuron of every sample, the register after each of its L queue columns (conv: L =
 * max_queue_len; fc: L = the input stream capacity), whether it fired there and the time of the
 * column's event (NaN for columns at or past the neuron's real events).  v_steps / spike_mask /
 * event_ms are (batch, n_neurons, L) or NULL.  per_neuron (optional, each pointer optional,
 * (batch, n_neurons) each) gives the first overflowing column (-1: none) with the register before
 * and after it, whether that column fired and its event time — the fields example/quant_run.py
 * (overflow_events, :189-214) reports — plus the unfitted extremes, v_final and the spike count.
 * An analysis path: one thread per neuron rebuilds its queue from the stream. */
typedef struct {
  int32_t *first_overflow;
  int32_t *v_before, *v_after;
  int32_t *spiked;
  float *time_ms;
  int32_t *v_min, *v_max;
  int32_t *v_final, *spike_count;
} salt_neuron_trace;

salt_status salt_conv_layer_trace(const salt_conv_desc *layer, const salt_quant_desc *quant,
                                  const int32_t *q, const int32_t *lut, const int32_t *vth,
                                  int32_t batch, const salt_stream_in *in, int32_t *v_steps,
                                  uint8_t *spike_mask, float *event_ms,
                                  const salt_neuron_trace *per_neuron, void *stream);
salt_status salt_fc_layer_trace(const salt_fc_desc *layer, const salt_quant_desc *quant,
                                const int32_t *q, const int32_t *lut, const int32_t *vth,
                                int32_t batch, const salt_stream_in *in, int32_t *v_steps,
                                uint8_t *spike_mask, float *event_ms,
                                const salt_neuron_trace *per_neuron, void *stream);

/* ---------------------------------------------------------------- fc layer
 * Replaces FCLayer.forward with QuantBackend (salt_core/layers/fc.py:84-101 calling
 * build_fc_structure connectivity/fc.py:20-33, fc_weight_codes :54-61, QuantBackend.scan,
 * extract_output_events_fc stream.py:67-81).
 *   q (n_out, n_in) int32 weight codes; vth (n_out) or NULL; v_final (batch, n_out). */
salt_status salt_fc_layer_workspace_size(const salt_fc_desc *layer, const salt_quant_desc *quant,
                                         int32_t batch, int32_t in_capacity, size_t *bytes);
salt_status salt_fc_layer_forward(const salt_fc_desc *layer, const salt_quant_desc *quant,
                                  const int32_t *q, const int32_t *lut, const int32_t *vth,
                                  int32_t batch, const salt_stream_in *in, salt_stream_out *out,
                                  int32_t *v_final, const salt_layer_stats *stats,
                                  void *workspace, size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------- dense scan
 * Replaces quant.scan.run_layer (salt_core/quant/scan.py:65-80, :97-132) on materialised
 * (n, L) queues — the Backend.scan plug-in point of salt_core/backend.py:64-74.
 *   a_int (n, L) int32, is_identity (n, L) uint8, q_int (n, L) int32, vth (n) or NULL
 *   spike_mask / overflowed (n, L) uint8 (may be NULL); v_final, vmin, vmax (n) int32. */
salt_status salt_quant_scan_dense(const salt_quant_desc *quant, int32_t n, int32_t L,
                                  const int32_t *a_int, const uint8_t *is_identity,
                                  const int32_t *q_int, const int32_t *vth, uint8_t *spike_mask,
                                  uint8_t *overflowed, int32_t *v_final, int32_t *vmin,
                                  int32_t *vmax, void *stream);

/* The same scan with trace=True (run_layer_traced, salt_core/quant/scan.py:83-94, as
 * QuantBackend.scan calls it, salt_core/quant/backend.py:41-43): v_steps (n, L) int32 receives
 * the register after each column (after a spike's reset); its last column equals v_final. */
salt_status salt_quant_scan_dense_trace(const salt_quant_desc *quant, int32_t n, int32_t L,
                                        const int32_t *a_int, const uint8_t *is_identity,
                                        const int32_t *q_int, const int32_t *vth,
                                        uint8_t *spike_mask, uint8_t *overflowed,
                                        int32_t *v_final, int32_t *vmin, int32_t *vmax,
                                        int32_t *v_steps, void *stream);

/* ---------------------------------------------------------------- network plan
 * A native runtime object that chains layers on the device (salt_core/network.py:93-122
 * run_network, vmapped over the batch as Network.apply_batched :179-183) with every
 * intermediate stream kept in the workspace, optionally replayed as one CUDA graph.
 * Layer parameters are HOST pointers copied to the device at creation. */
typedef struct {
  int32_t kind;            /* 0 conv, 1 fc */
  salt_conv_desc conv;
  salt_fc_desc fc;
  salt_quant_desc quant;
  const int32_t *q_host;   /* weight codes (layout as above) */
  const int32_t *lut_host;
  const int32_t *vth_host; /* per-neuron thresholds, NULL when has_vth == 0 */
} salt_layer_spec;

typedef struct salt_network salt_network;

salt_status salt_network_create(const salt_layer_spec *layers, int32_t n_layers,
                                salt_network **out);
salt_status salt_network_destroy(salt_network *net);
salt_status salt_network_workspace_size(const salt_network *net, int32_t batch,
                                        int32_t in_capacity, size_t *bytes);
/* Runs every layer.  Outputs (device, may be NULL except logits):
 *   logits      (batch, n_last) int32: v_final of the last layer (register values)
 *   spike_count (n_layers, batch) int32, overflowed (n_layers, batch) int32,
 *   vmin/vmax   (n_layers, batch) int32, needed_queue (n_layers, batch) int32,
 *   fits        (batch) int32: AND of Capacity.fits over layers (network.py:116-119). */
salt_status salt_network_forward(salt_network *net, int32_t batch, const salt_stream_in *in,
                                 int32_t *logits, int32_t *spike_count, int32_t *overflowed,
                                 int32_t *vmin, int32_t *vmax, int32_t *needed_queue,
                                 int32_t *fits, void *workspace, size_t workspace_bytes,
                                 void *stream);
/* Part of a forward (no reference counterpart: lets a caller overlap the input transfer with the
 * first layer): layers [layer_begin, layer_end) on rows [row0, row0 + rows) of a batch-`batch`
 * forward planned for first-layer input capacity in_capacity, with that forward's workspace and
 * full-batch output arrays (same layouts as salt_network_forward; only the rows' entries are
 * written).  layer_begin == 0 reads `in` (rows rows, capacity in_capacity); otherwise the part
 * reads what layer layer_begin - 1 left in the workspace for these rows, so parts run in layer
 * order on one stream.  logits and fits are written when layer_end is the last layer.  Running
 * layer 0 on row slices and then the remaining layers on all rows gives the results of
 * salt_network_forward. */
salt_status salt_network_forward_part(salt_network *net, int32_t batch, int32_t in_capacity,
                                      int32_t row0, int32_t rows, int32_t layer_begin,
                                      int32_t layer_end, const salt_stream_in *in,
                                      int32_t *logits, int32_t *spike_count, int32_t *overflowed,
                                      int32_t *vmin, int32_t *vmax, int32_t *needed_queue,
                                      int32_t *fits, void *workspace, size_t workspace_bytes,
                                      void *stream);
/* Number of kernel launches the last salt_network_forward enqueued (for launch accounting). */
int32_t salt_network_last_launch_count(const salt_network *net);
/* Kernel timing of the forwards enqueued while profiling is on: CUDA events are recorded on the
 * launching stream around every conv layer's fused bucket+scan kernel (the dominant kernel) and
 * around every whole layer.  salt_network_profile_read synchronises on those events and writes,
 * per layer, the summed milliseconds of the fused kernel (fused_ms, 0 for FC layers) and of the
 * whole layer (layer_ms), and the number of timed forwards (launches); reset clears them. */
salt_status salt_network_set_profiling(salt_network *net, int32_t enable);
salt_status salt_network_profile_read(salt_network *net, float *fused_ms, float *layer_ms,
                                      int32_t *launches, int32_t reset);

/* ---------------------------------------------------------------- float FC layer
 * Replaces FCLayer.forward with FloatBackend (salt_core/layers/fc.py:84-106 calling
 * build_fc_structure connectivity/fc.py:20-33, fc_float_values :36-51, FloatBackend.scan
 * float/backend.py:16-31 -> float.scan.run_layer float/scan.py:34-50 over process_chunk
 * float/affine.py:99-126, extract_output_events_fc stream.py:67-81, extra_steps_upper_bound
 * float/affine.py:57-88) — the forward values.
 *   w (n_out, n_in) float32 as FCLayer holds it; decay_base (n_out) = float32(1 - 1/tau) per
 *   neuron (all equal for the reference's scalar tau; per-neuron values extend it).
 *   in_gain (batch, capacity) event gains or NULL for all ones (the forward s_spike of an upstream
 *   float layer is 1).  v_final (batch, n_out).  The output stream's gains are 1 for every real
 *   entry and are not written.
 *   stats (optional, each pointer optional): spike_count (batch) = Σ spike_mask;
 *   needed_extra_steps (batch) = LayerDiag.needed["max_extra_steps"]; fits (batch).
 * v_th must be > 0 (a threshold <= 0 fires on padding, which only the reference's fixed step
 * count bounds).  Float results follow the reference within float32 rounding: the scan runs the
 * recurrence v = a*v + b in event order, where the reference composes each chunk's maps first. */
typedef struct {
  int32_t n_in, n_out;
  int32_t chunk_size;       /* FCLayer.chunk_size */
  int32_t max_out_spikes;   /* FCLayer.max_out_spikes */
  int32_t max_extra_steps;  /* FCLayer.max_extra_steps */
  float v_th;               /* FCLayer.v_th */
} salt_float_fc_desc;

typedef struct {
  int32_t *spike_count;
  int32_t *needed_extra_steps;
  int32_t *fits;
} salt_float_layer_stats;

salt_status salt_float_fc_layer_workspace_size(const salt_float_fc_desc *layer, int32_t batch,
                                               int32_t in_capacity, int32_t has_gain,
                                               size_t *bytes);
salt_status salt_float_fc_layer_forward(const salt_float_fc_desc *layer, const float *w,
                                        const float *decay_base, int32_t batch,
                                        const salt_stream_in *in, const float *in_gain,
                                        salt_stream_out *out, float *v_final,
                                        const salt_float_layer_stats *stats, void *workspace,
                                        size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------- float conv layer
 * Replaces ConvLayer.forward with FloatBackend (salt_core/layers/conv.py:124-149): the queue of
 * build_conv_structure (connectivity/conv.py:128-172), conv_float_values (:187-206), the chunked
 * scan (float/scan.py:67-116, float/affine.py:99-126), spike_step_upper_bound's need
 * (affine.py:57-88) and extract_output_events_conv (stream.py:84-100).  The float forward of the
 * quantisation pipeline: with chunk_size 1 it is the calibration forward of
 * example/quant_run.py:30-44.  w is (oc, ic, k, k) float32; decay_base = float32(1 - 1/tau);
 * in_gain (batch, capacity) may be NULL (all ones).  The output stream's real entries carry gain
 * 1 (the forward value of s_spike), so it has no gain array.  v_th must be finite and > 0. */
typedef struct {
  int32_t ic, h_in, w_in, oc, k, s, p;
  int32_t max_queue_len;    /* ConvLayer.max_queue_len */
  int32_t max_out_spikes;   /* ConvLayer.max_out_spikes */
  int32_t max_extra_steps;  /* ConvLayer.max_extra_steps */
  int32_t chunk_size;       /* ConvLayer.chunk_size */
  float v_th;               /* ConvLayer.v_th */
} salt_float_conv_desc;

typedef struct {
  int32_t *spike_count;         /* (batch) spikes, not clipped to max_out_spikes */
  int32_t *needed_queue;        /* (batch) largest real taps of a position + 1 */
  int32_t *needed_extra_steps;  /* (batch) */
  int32_t *fits;                /* (batch) every need within its knob */
} salt_float_conv_stats;

/* Per-step traces of a float layer (run_layer_traced, float/scan.py:53-64, with trace.py:13-55)
 * and its potential ranges (quant/calibrate.py:16-36 reduces v_steps to these); any pointer may
 * be NULL.  max_steps = ceil(L / chunk_size) + max_extra_steps, L = max_queue_len (conv) or the
 * input capacity (FC).  Ranges are over every step and, for conv layers, every position of a
 * channel; an FC neuron is its own channel. */
typedef struct {
  float *v_steps;       /* (batch, n_neurons, max_steps) potential after each step */
  float *event_ms;      /* (batch, n_neurons, max_steps) first event time of the step; NaN idle */
  uint8_t *spike_mask;  /* (batch, n_neurons, max_steps) */
  float *v_max;         /* (batch, channels) */
  float *v_min;         /* (batch, channels) */
} salt_float_trace;

salt_status salt_float_conv_layer_workspace_size(const salt_float_conv_desc *layer, int32_t batch,
                                                 int32_t in_capacity, size_t *bytes);
salt_status salt_float_conv_layer_forward(const salt_float_conv_desc *layer, const float *w,
                                          float decay_base, int32_t batch,
                                          const salt_stream_in *in, const float *in_gain,
                                          salt_stream_out *out, float *v_final,
                                          const salt_float_conv_stats *stats,
                                          const salt_float_trace *trace, void *workspace,
                                          size_t workspace_bytes, void *stream);

/* Per-step traces and potential ranges of a float FC layer (FCLayer.forward with FloatBackend and
 * trace=True, salt_core/layers/fc.py:84-106); v_final (batch, n_out) may be NULL.  The layer's
 * output stream comes from salt_float_fc_layer_forward. */
salt_status salt_float_fc_layer_trace(const salt_float_fc_desc *layer, const float *w,
                                      const float *decay_base, int32_t batch,
                                      const salt_stream_in *in, const float *in_gain,
                                      float *v_final, const salt_float_trace *trace, void *stream);

/* ---------------------------------------------------------------- stream transfer
 * No reference counterpart (the reference's input lives in XLA buffers): copies a batch of event
 * streams from PINNED host memory to the device, moving each sample's row only up to
 * min(n_real, capacity).  host_times / host_src: (batch, host_pitch) rows in page-locked memory
 * (cudaHostAlloc / cudaMallocHost / cudaHostRegister; rejected with SALT_BAD_ARG otherwise);
 * n_real: (batch) DEVICE array (copy it first); dev_times / dev_src: (batch, capacity) device
 * rows, whose pad entries are left as they were.  Exact whenever no layer reads pad entries: true
 * unless the first layer has needs_tail set (then copy the full rows instead). */
salt_status salt_stream_h2d_real(const float *host_times, const int32_t *host_src,
                                 int64_t host_pitch, const int32_t *n_real, int32_t batch,
                                 int32_t capacity, float *dev_times, int32_t *dev_src,
                                 void *stream);

/* Optional timing of the float FC layers that the calling thread enqueues: with profiling on,
 * CUDA events are recorded on the launching stream around each layer's speculative segment
 * kernel (the dominant kernel) and around the whole layer.  salt_float_fc_profile_read
 * synchronises on them and writes the summed milliseconds and the number of timed layers;
 * reset clears the sums. */
salt_status salt_float_fc_set_profiling(int32_t enable);
salt_status salt_float_fc_profile_read(float *segment_ms, float *layer_ms, int32_t *layers,
                                       int32_t reset);

/* ---------------------------------------------------------------- runtime plumbing
 * No reference counterpart: under JAX, XLA owns the buffers, streams and executables.  A host
 * that calls this library without XLA (the Python package, a C or cgo caller) takes device
 * memory, pinned host memory, streams, events and graph replay from these thin wrappers of the
 * CUDA runtime, so that nothing else on the host side needs a GPU framework.
 *   - salt_malloc / salt_free: stream-ordered device memory (cudaMallocAsync / cudaFreeAsync on
 *     `stream`; the device's default pool keeps freed memory cached for reuse).  A pointer may
 *     be used on another stream only after that stream waits for `stream`.
 *   - salt_host_alloc / salt_host_free: page-locked host memory, mapped into the device's address
 *     space (what salt_stream_h2d_real reads).
 *   - salt_memcpy_async: any direction (cudaMemcpyDefault: unified addressing tells host from
 *     device); salt_memset_async: bytes.
 *   - streams are created non-blocking (no implicit ordering with the legacy default stream,
 *     which is `stream` = NULL).
 *   - salt_graph_*: records everything enqueued on `stream` between begin and end (a
 *     non-default stream; nothing may synchronise meanwhile) and replays it with one launch. */
salt_status salt_malloc(size_t bytes, void *stream, void **ptr);
salt_status salt_free(void *ptr, void *stream);
salt_status salt_host_alloc(size_t bytes, void **ptr);
salt_status salt_host_free(void *ptr);
salt_status salt_memcpy_async(void *dst, const void *src, size_t bytes, void *stream);
salt_status salt_memset_async(void *ptr, int32_t value, size_t bytes, void *stream);
salt_status salt_device_count(int32_t *count);
salt_status salt_set_device(int32_t device);
salt_status salt_get_device(int32_t *device);
salt_status salt_device_synchronize(void);
salt_status salt_stream_create(void **stream);
/* A non-blocking stream whose blocks the scheduler prefers (the device's greatest priority):
 * for transfers that must overlap a kernel already filling the GPU. */
salt_status salt_stream_create_high_priority(void **stream);
salt_status salt_stream_destroy(void *stream);
salt_status salt_stream_synchronize(void *stream);
salt_status salt_stream_wait_event(void *stream, void *event);
salt_status salt_event_create(int32_t timing, void **event);
salt_status salt_event_destroy(void *event);
salt_status salt_event_record(void *event, void *stream);
salt_status salt_event_synchronize(void *event);
/* *done = 1 when the work before the event's last record has finished, else 0 (no waiting). */
salt_status salt_event_query(void *event, int32_t *done);
salt_status salt_event_elapsed_ms(void *start, void *stop, float *ms);
salt_status salt_graph_begin_capture(void *stream);
salt_status salt_graph_end_capture(void *stream, void **graph_exec);
salt_status salt_graph_launch(void *graph_exec, void *stream);
salt_status salt_graph_destroy(void *graph_exec);

/* Library facts and errors (host). */
const char *salt_last_error(void);
const char *salt_version(void);
/* Kernel launches enqueued by this thread since the last reset (for launch accounting). */
int64_t salt_launch_counter(int32_t reset);

#ifdef __cplusplus
}
#endif
#endif /* SALT_B200_H */
