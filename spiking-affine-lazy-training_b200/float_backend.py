"""FloatB200Backend: the float forward (FloatBackend) of FC and conv layers on B200.

Mirrors FCLayer.forward / ConvLayer.forward with FloatBackend (salt_core/layers/fc.py:84-106,
layers/conv.py:124-149, float/backend.py:16-31, float/scan.py:34-116, float/affine.py:57-126,
connectivity/conv.py:128-206, stream.py:67-100) for the forward values:
``FloatLayerResult.v_final``, the output EventStream (gain 1 on every real entry, the forward value
of s_spike) and LayerDiag with the reference's ``needed``.  FC layers run
``salt_float_fc_layer_forward``, conv layers ``salt_float_conv_layer_forward`` (libsalt_b200,
include/salt_b200.h); no CPU fallback.  ``trace=True`` adds the per-step LayerForwardTrace
(trace.py:13-55) and ``v_range=True`` each layer's per-(sample, channel) potential extremes over all
steps, which calibration (quant/calibrate.py) reduces to M.

Extension beyond the reference API: an FC layer's ``tau`` may be given per neuron (an (n_out,)
array overriding FCLayer.tau); neurons are independent, so each neuron behaves as a one-neuron
layer with its own tau.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np

from . import _lib
from .capacity import LayerDiag
from .device import (DeviceArray, DeviceStream, empty, ptr, require_cuda, stream_handle, to_device,
                     workspace, zeros)
from .layers import LayerOutput, is_conv
from .stream import EventStream
from .trace import LayerForwardTrace



class FloatLayerResult(NamedTuple):
    """Forward values of float/scan.py:15-22, batched.  The per-step arrays of the reference
    (spike_mask, spike_event_idx, s_spike, s_value of shape (n, max_steps)) carry no more than the
    output stream does in a forward pass (s_spike = s_value = spike_mask there), so the layer
    returns the stream instead; spike_count = Σ spike_mask."""
    v_final: np.ndarray
    spike_count: np.ndarray


class NetworkOutput(NamedTuple):
    """salt_core/network.py:57-67 for a chain of float layers, batched.  traces: per layer a
    LayerForwardTrace (trace=True); v_ranges: per layer (v_max, v_min), each (B, channels)
    (v_range=True)."""
    results: tuple
    diags: tuple
    traces: tuple | None
    fits: np.ndarray
    streams: tuple = ()
    v_ranges: tuple = ()

    @property
    def last(self):
        return self.results[-1]


class _FloatRun(NamedTuple):
    out: DeviceStream
    v_final: DeviceArray
    # FC (3, B): spike_count, needed_extra_steps, fits;
    # conv (4, B): spike_count, needed_queue, needed_extra_steps, fits
    stats: DeviceArray
    trace: tuple | None = None    # (spike_mask, v_steps, event_ms), each (B, n, max_steps)
    v_range: tuple | None = None  # (v_max, v_min), each (B, channels)


def decay_base(tau, n_out: int) -> np.ndarray:
    """float32(1 - 1/tau) per neuron: the base that create_affine_maps (float/affine.py:27-31)
    raises to the Δt power (a Python-float base meeting a float32 array becomes float32)."""
    t = np.broadcast_to(np.asarray(tau, dtype=np.float64), (n_out,))
    if np.any(~np.isfinite(t)) or np.any(t == 0):
        raise ValueError("tau must be finite and non-zero")
    return np.ascontiguousarray((1.0 - 1.0 / t).astype(np.float32))


def _check_vth(layer) -> None:
    if not float(layer.v_th) > 0.0 or not np.isfinite(float(layer.v_th)):
        raise ValueError(f"float layer {layer.name}: v_th must be finite and > 0 (a threshold "
                         "<= 0 fires on pad and identity entries)")


def float_desc(layer) -> _lib.FloatFCDesc:
    if is_conv(layer):
        raise TypeError("float_desc takes FC layers; conv layers use float_conv_desc")
    _check_vth(layer)
    return _lib.FloatFCDesc(int(layer.n_in), int(layer.n_out), int(layer.chunk_size),
                            int(layer.max_out_spikes), int(layer.max_extra_steps),
                            float(layer.v_th))


def float_conv_desc(layer) -> _lib.FloatConvDesc:
    _check_vth(layer)
    return _lib.FloatConvDesc(int(layer.ic), int(layer.h_in), int(layer.w_in), int(layer.oc),
                              int(layer.k), int(layer.s), int(layer.p), int(layer.max_queue_len),
                              int(layer.max_out_spikes), int(layer.max_extra_steps),
                              int(layer.chunk_size), float(layer.v_th))


def max_steps(layer, in_capacity: int) -> int:
    """Scan steps (layers/conv.py:175-177, layers/fc.py:128-130)."""
    L = int(layer.max_queue_len) if is_conv(layer) else int(in_capacity)
    return -(-L // int(layer.chunk_size)) + int(layer.max_extra_steps)


def _unit_gains(stream: EventStream) -> bool:
    g = np.asarray(stream.event_gain, dtype=np.float32)
    t = np.asarray(stream.event_times)
    n = np.atleast_1d(np.asarray(stream.n_real_events)).astype(np.int64)
    if g.ndim == 1:
        g, t = g[None], t[None]
    real = np.arange(g.shape[1])[None, :] < n[:, None]
    return bool(np.all(np.where(real, g, 1.0) == 1.0))


class _TraceBuffers:
    """Device outputs of salt_float_trace for one layer."""

    def __init__(self, B: int, n: int, steps: int, channels: int, trace: bool, v_range: bool):
        self.trace = trace
        self.v_range = v_range
        z = None
        self.spike_mask = empty((B, n, steps), np.uint8) if trace else z
        self.v_steps = empty((B, n, steps), np.float32) if trace else z
        self.event_ms = empty((B, n, steps), np.float32) if trace else z
        self.v_max = empty((B, channels), np.float32) if v_range else z
        self.v_min = empty((B, channels), np.float32) if v_range else z
        self.struct = _lib.FloatTrace(ptr(self.v_steps), ptr(self.event_ms), ptr(self.spike_mask),
                                      ptr(self.v_max), ptr(self.v_min))

    @property
    def any(self) -> bool:
        return self.trace or self.v_range

    def outputs(self):
        tr = (self.spike_mask, self.v_steps, self.event_ms) if self.trace else None
        vr = (self.v_max, self.v_min) if self.v_range else None
        return tr, vr


class FloatLayerPlan:
    """One float FC layer prepared for repeated batched forwards: weights, decay bases, output
    buffers and the workspace live on the device; each forward is one C-ABI call on the current
    stream over a device-resident stream of the planned shape (plus the trace kernel when trace
    or v_range is asked for)."""

    def __init__(self, layer, w, batch: int, in_capacity: int, *, tau=None, gain: bool = False,
                 trace: bool = False, v_range: bool = False):
        require_cuda()
        self.layer, self.batch, self.capacity, self.gain = layer, int(batch), int(in_capacity), gain
        self.desc = float_desc(layer)
        n = int(layer.n_out)
        self.w = to_device(np.asarray(w, dtype=np.float32).reshape(n, int(layer.n_in)), np.float32)
        self.base = to_device(decay_base(layer.tau if tau is None else tau, n), np.float32)
        B, M = self.batch, int(layer.max_out_spikes)
        self.out_t = empty((B, M), np.float32)
        self.out_s = empty((B, M), np.int32)
        self.out_n = empty((B,), np.int32)
        self.v_final = empty((B, n), np.float32)
        self.stats = zeros((3, B), np.int32)
        self._st = _lib.FloatLayerStats(*[ptr(self.stats[i]) for i in range(3)])
        self._sout = _lib.StreamOut(ptr(self.out_t), ptr(self.out_s), ptr(self.out_n))
        self._tb = _TraceBuffers(B, n, max_steps(layer, self.capacity), n, trace, v_range)
        nbytes = ctypes.c_size_t(0)
        _lib.check(_lib.lib().salt_float_fc_layer_workspace_size(
            _lib.byref(self.desc), B, self.capacity, int(gain), _lib.byref(nbytes)))
        self.ws_bytes = nbytes.value
        self.ws = workspace(self.ws_bytes)

    def forward_device(self, dstream: DeviceStream, gain: "DeviceArray | None" = None
                       ) -> _FloatRun:
        if (dstream.batch, dstream.capacity) != (self.batch, self.capacity):
            raise ValueError(f"stream shape {(dstream.batch, dstream.capacity)} does not match the "
                             f"plan's {(self.batch, self.capacity)}")
        if (gain is not None) != self.gain:
            raise ValueError("gain given to a plan built without it, or missing")
        sin = _lib.StreamIn(ptr(dstream.times), ptr(dstream.src), ptr(dstream.n_real),
                            self.capacity, int(dstream.virtual_pads))
        lib = _lib.lib()
        _lib.check(lib.salt_float_fc_layer_forward(
            _lib.byref(self.desc), ptr(self.w), ptr(self.base), self.batch, _lib.byref(sin),
            ptr(gain), _lib.byref(self._sout), ptr(self.v_final), _lib.byref(self._st),
            ptr(self.ws), self.ws_bytes, stream_handle()))
        if self._tb.any:
            _lib.check(lib.salt_float_fc_layer_trace(
                _lib.byref(self.desc), ptr(self.w), ptr(self.base), self.batch, _lib.byref(sin),
                ptr(gain), None, _lib.byref(self._tb.struct), stream_handle()))
        tr, vr = self._tb.outputs()
        return _FloatRun(DeviceStream(self.out_t, self.out_s, self.out_n, True), self.v_final,
                         self.stats, tr, vr)


class FloatConvPlan:
    """One float conv layer prepared for repeated batched forwards (salt_float_conv_layer_forward),
    the conv counterpart of FloatLayerPlan.  tau is the layer's scalar ConvLayer.tau."""

    def __init__(self, layer, w, batch: int, in_capacity: int, *, gain: bool = False,
                 trace: bool = False, v_range: bool = False):
        require_cuda()
        self.layer, self.batch, self.capacity, self.gain = layer, int(batch), int(in_capacity), gain
        self.desc = float_conv_desc(layer)
        n = int(layer.n_neurons)
        self.w = to_device(np.asarray(w, dtype=np.float32).reshape(layer.weight_shape), np.float32)
        self.base = float(decay_base(layer.tau, 1)[0])
        B, M = self.batch, int(layer.max_out_spikes)
        self.out_t = empty((B, M), np.float32)
        self.out_s = empty((B, M), np.int32)
        self.out_n = empty((B,), np.int32)
        self.v_final = empty((B, n), np.float32)
        self.stats = zeros((4, B), np.int32)
        self._st = _lib.FloatConvStats(*[ptr(self.stats[i]) for i in range(4)])
        self._sout = _lib.StreamOut(ptr(self.out_t), ptr(self.out_s), ptr(self.out_n))
        self._tb = _TraceBuffers(B, n, max_steps(layer, self.capacity), int(layer.oc), trace,
                                 v_range)
        nbytes = ctypes.c_size_t(0)
        _lib.check(_lib.lib().salt_float_conv_layer_workspace_size(
            _lib.byref(self.desc), B, self.capacity, _lib.byref(nbytes)))
        self.ws_bytes = nbytes.value
        self.ws = workspace(self.ws_bytes)

    def forward_device(self, dstream: DeviceStream, gain: "DeviceArray | None" = None
                       ) -> _FloatRun:
        if (dstream.batch, dstream.capacity) != (self.batch, self.capacity):
            raise ValueError(f"stream shape {(dstream.batch, dstream.capacity)} does not match the "
                             f"plan's {(self.batch, self.capacity)}")
        if (gain is not None) != self.gain:
            raise ValueError("gain given to a plan built without it, or missing")
        sin = _lib.StreamIn(ptr(dstream.times), ptr(dstream.src), ptr(dstream.n_real),
                            self.capacity, int(dstream.virtual_pads))
        _lib.check(_lib.lib().salt_float_conv_layer_forward(
            _lib.byref(self.desc), ptr(self.w), ctypes.c_float(self.base), self.batch,
            _lib.byref(sin), ptr(gain), _lib.byref(self._sout), ptr(self.v_final),
            _lib.byref(self._st), _lib.byref(self._tb.struct) if self._tb.any else None,
            ptr(self.ws), self.ws_bytes, stream_handle()))
        tr, vr = self._tb.outputs()
        return _FloatRun(DeviceStream(self.out_t, self.out_s, self.out_n, True), self.v_final,
                         self.stats, tr, vr)


def set_profiling(enable: bool) -> None:
    """Time each float FC layer this thread enqueues (segment kernel and whole layer)."""
    _lib.check(_lib.lib().salt_float_fc_set_profiling(int(bool(enable))))


def profile_read(reset: bool = True) -> tuple[float, float, int]:
    """(segment kernel ms, whole layer ms, layers timed) summed since the last reset."""
    seg, lay, n = ctypes.c_float(0), ctypes.c_float(0), ctypes.c_int32(0)
    _lib.check(_lib.lib().salt_float_fc_profile_read(_lib.byref(seg), _lib.byref(lay),
                                                     _lib.byref(n), int(bool(reset))))
    return float(seg.value), float(lay.value), int(n.value)


def _first(x):
    return x[0] if isinstance(x, tuple) else x


@dataclass(frozen=True)
class FloatB200Backend:
    """FloatBackend's drop-in for FC and conv layers (forward values) on B200."""

    def compile(self, layer, w, batch: int, in_capacity: int, *, tau=None, gain: bool = False,
                trace: bool = False, v_range: bool = False):
        if is_conv(layer):
            if tau is not None:
                raise ValueError("conv layers take their scalar ConvLayer.tau")
            return FloatConvPlan(layer, w, batch, in_capacity, gain=gain, trace=trace,
                                 v_range=v_range)
        return FloatLayerPlan(layer, w, batch, in_capacity, tau=tau, gain=gain, trace=trace,
                              v_range=v_range)

    def forward_layer_device(self, layer, w, dstream: DeviceStream, *, tau=None,
                             gain: "DeviceArray | None" = None, trace: bool = False,
                             v_range: bool = False) -> _FloatRun:
        """One batched layer on device-resident streams; gain (B, capacity) or None (ones)."""
        plan = self.compile(layer, w, dstream.batch, dstream.capacity, tau=tau,
                            gain=gain is not None, trace=trace, v_range=v_range)
        return plan.forward_device(dstream, gain)

    @staticmethod
    def _host_layer(layer, run: _FloatRun, n_in: np.ndarray):
        stats = run.stats.numpy()
        S = stats[0].astype(np.int32)
        result = FloatLayerResult(v_final=run.v_final.numpy(), spike_count=S)
        n = int(layer.n_neurons) if is_conv(layer) else int(layer.n_out)
        denom = np.float32(n) * np.maximum(n_in, 1).astype(np.float32)
        if is_conv(layer):
            needed = {"max_queue_len": stats[1].astype(np.int32), "max_out_spikes": S,
                      "max_extra_steps": stats[2].astype(np.int32)}
            fits = stats[3] != 0
        else:
            needed = {"max_out_spikes": S, "max_extra_steps": stats[1].astype(np.int32)}
            fits = stats[2] != 0
        diag = LayerDiag(spike_count=S, firing_rate=S.astype(np.float32) / denom, needed=needed)
        return result, diag, fits

    @staticmethod
    def _host_trace(run: _FloatRun):
        if run.trace is None:
            return None
        mask, v, ms = (t.numpy() for t in run.trace)
        return LayerForwardTrace(spike_mask=mask.astype(bool), v_steps=v, event_ms=ms)

    @staticmethod
    def _single(result, diag, stream, trace):
        result = FloatLayerResult(result.v_final[0], result.spike_count[0])
        diag = LayerDiag(diag.spike_count[0], diag.firing_rate[0],
                         {k: v[0] for k, v in diag.needed.items()})
        if stream is not None:
            stream = EventStream(stream.event_times[0], stream.event_source_idx[0],
                                 stream.event_gain[0], stream.n_real_events[0])
        if trace is not None:
            trace = LayerForwardTrace(trace.spike_mask[0], trace.v_steps[0], trace.event_ms[0])
        return result, diag, stream, trace

    def forward_layer(self, layer, w, in_stream: EventStream, *, tau=None, trace: bool = False
                      ) -> LayerOutput:
        """FCLayer / ConvLayer .forward(w, in_stream, backend=FLOAT, trace=trace), batched or
        single sample."""
        single = np.ndim(in_stream.event_times) == 1
        dstream = DeviceStream.from_host(in_stream)
        gain = None
        if not _unit_gains(in_stream):
            g = np.asarray(in_stream.event_gain, dtype=np.float32)
            gain = to_device(g[None] if single else g, np.float32)
        run = self.forward_layer_device(layer, w, dstream, tau=tau, gain=gain, trace=trace)
        n_in = np.atleast_1d(np.asarray(in_stream.n_real_events)).astype(np.int64)
        result, diag, _ = self._host_layer(layer, run, n_in)
        stream = run.out.to_host()  # gains: 1 on every entry
        tr = self._host_trace(run)
        if single:
            result, diag, stream, tr = self._single(result, diag, stream, tr)
        return LayerOutput(stream=stream, result=result, diag=diag, trace=tr)

    def run_network(self, layers, weights, input_stream: EventStream, *, taus=None,
                    trace: bool = False, v_range: bool = False, keep_streams: bool = False
                    ) -> NetworkOutput:
        """network.py:93-122 for a chain of float FC and conv layers; the intermediate streams
        stay on the device (their gains are 1).  taus: optional per-layer tau overrides (FC
        layers).  trace=True: per-layer LayerForwardTrace; v_range=True: per-layer (v_max, v_min)
        per (sample, channel)."""
        single = np.ndim(input_stream.event_times) == 1
        cur = DeviceStream.from_host(input_stream)
        gain = None
        if not _unit_gains(input_stream):
            g = np.asarray(input_stream.event_gain, dtype=np.float32)
            gain = to_device(g[None] if single else g, np.float32)
        runs = []
        for i, (layer, w) in enumerate(zip(layers, weights)):
            tau = None if taus is None else taus[i]
            run = self.forward_layer_device(layer, w, cur, tau=tau, gain=gain, trace=trace,
                                            v_range=v_range)
            runs.append(run)
            cur, gain = run.out, None
        results, diags, fits, streams, traces, ranges = [], [], None, [], [], []
        prev = np.atleast_1d(np.asarray(input_stream.n_real_events)).astype(np.int64)
        for layer, run in zip(layers, runs):
            r, d, f = self._host_layer(layer, run, prev)
            prev = r.spike_count.astype(np.int64)
            tr = self._host_trace(run)
            st = run.out.to_host() if keep_streams else None
            vr = tuple(t.numpy() for t in run.v_range) if v_range else None
            if single:
                r, d, st, tr = self._single(r, d, st, tr)
                f = f[0]
                vr = tuple(a[0] for a in vr) if vr is not None else None
            results.append(r)
            diags.append(d)
            fits = f if fits is None else (fits & f)
            if keep_streams:
                streams.append(st)
            traces.append(tr)
            if v_range:
                ranges.append(vr)
        return NetworkOutput(tuple(results), tuple(diags), tuple(traces) if trace else None, fits,
                             tuple(streams), tuple(ranges))

    def readout(self, result, params):
        """float/backend.py:33-35: the float path is already at physical scale."""
        return result
