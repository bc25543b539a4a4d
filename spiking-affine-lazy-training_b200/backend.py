"""QuantB200Backend: the B200 integer backend behind the reference's Backend protocol.

Two entry levels, both on the CUDA kernels of libsalt_b200 (no CPU fallback):

* ``scan(layer, structure, params, event_gain, *, trace)`` and ``readout(result, params)`` —
  exactly the plug-in point of salt_core/backend.py:64-74 (QuantBackend.scan,
  salt_core/quant/backend.py:31-63).  ``scan`` takes the reference's materialised (n, L) queue
  (layer.neuron_delta_t / layer.gather_weight_codes) and runs the integer recurrence on the GPU.
* ``forward_layer`` / ``run_network`` / ``compile`` — the fused per-layer pipeline (fan-out,
  stable bucketing, recurrence, compaction, diagnostics) that replaces ConvLayer.forward /
  FCLayer.forward / run_network (salt_core/layers/conv.py:124-149, layers/fc.py:84-101,
  network.py:93-122) without materialising any (n, L) array.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np

from . import _lib
from .capacity import LayerDiag
from .device import (DeviceArray, DeviceStream, empty, ptr, require_cuda, stream_handle,
                     to_device, workspace, zeros)
from .layers import LayerOutput, is_conv
from .quant import (OverflowMode, RoundMode, apply_decay_table_int, check_bit_widths,
                    check_weight_codes, weight_bits)
from .stream import EventStream

class QuantLayerResult(NamedTuple):
    """Per-layer integer result (salt_core/quant/scan.py:55-62), batched.

    The fused pipeline keeps the reference's per-neuron v_final and reduces the per-column
    fields the way example/quant_run.py:86-93 consumes them: ``overflowed`` is any() over
    (neuron, column), ``v_unfitted_min/max`` are min/max over neurons.  The output spikes are
    the layer's EventStream.  ``scan`` (the dense plug-in) returns the full per-column fields.
    """
    v_final: np.ndarray
    spike_count: np.ndarray
    overflowed: np.ndarray
    v_unfitted_min: np.ndarray
    v_unfitted_max: np.ndarray


class DenseQuantLayerResult(NamedTuple):
    """salt_core/quant/scan.py:55-62 field for field (from ``scan``)."""
    spike_mask: np.ndarray
    spike_event_idx: np.ndarray
    v_final: np.ndarray
    overflowed: np.ndarray
    v_unfitted_min: np.ndarray
    v_unfitted_max: np.ndarray


class ScanOutput(NamedTuple):
    """salt_core/backend.py:27-33"""
    result: DenseQuantLayerResult
    spike_gain: np.ndarray
    extra_steps_needed: np.ndarray
    v_steps: np.ndarray | None
    pointer_steps: np.ndarray | None


class NetworkOutput(NamedTuple):
    """salt_core/network.py:57-67, batched (leading batch axis on every array)."""
    results: tuple
    diags: tuple
    traces: tuple | None
    fits: np.ndarray
    streams: tuple = ()   # each layer's output EventStream (host), when requested

    @property
    def last(self):
        return self.results[-1]


def _round_code(mode) -> int:
    return 0 if RoundMode(mode) is RoundMode.ROUND else 1


def _overflow_code(mode) -> int:
    return 0 if OverflowMode(mode) is OverflowMode.WRAP else 1


def _vth_array(params, n: int) -> np.ndarray | None:
    if params.v_th_int is None:
        return None
    v = np.asarray(params.v_th_int)
    if not np.issubdtype(v.dtype, np.integer):
        v = v.astype(np.int64)
    return np.ascontiguousarray(np.broadcast_to(v.astype(np.int32), (n,)))


def quant_desc(params, round_mode, n_neurons: int) -> tuple[_lib.QuantDesc, np.ndarray | None]:
    """salt_quant_desc for one layer, with the same argument checks as the reference."""
    check_weight_codes(params.q)
    check_bit_widths(int(params.f_a), int(params.f_V), int(params.i_V))
    lut = np.asarray(params.decay_table_int)
    vth = _vth_array(params, n_neurons)
    d = _lib.QuantDesc()
    d.f_a, d.f_V, d.i_V = int(params.f_a), int(params.f_V), int(params.i_V)
    d.round_mode = _round_code(round_mode)
    d.overflow_mode = _overflow_code(getattr(params, "overflow_mode", OverflowMode.WRAP))
    d.lut_len = int(lut.shape[0])
    d.has_vth = vth is not None
    d.q_bits = weight_bits(params.q)
    tail = vth is not None and bool(np.any(vth <= 0))
    if lut.size:
        tail = tail or bool(np.any((lut < 0) | (lut >= (1 << d.f_a))))
    d.needs_tail = int(tail)
    return d, vth


def conv_desc(layer) -> _lib.ConvDesc:
    d = _lib.ConvDesc()
    for f in ("ic", "h_in", "w_in", "oc", "k", "s", "p", "max_queue_len", "max_out_spikes",
              "max_extra_steps"):
        setattr(d, f, int(getattr(layer, f)))
    return d


def fc_desc(layer) -> _lib.FCDesc:
    d = _lib.FCDesc()
    for f in ("n_in", "n_out", "max_out_spikes", "max_extra_steps"):
        setattr(d, f, int(getattr(layer, f)))
    return d


class _LayerRun(NamedTuple):
    out: DeviceStream
    v_final: DeviceArray
    stats: DeviceArray      # (6, B): spike_count, needed_queue, overflowed, vmin, vmax, fits


@dataclass(frozen=True)
class QuantB200Backend:
    """Integer backend on B200 (QuantBackend's drop-in).  round_mode is network-wide, as in
    salt_core/quant/backend.py:23-29."""
    round_mode: RoundMode | str = RoundMode.ROUND

    # ------------------------------------------------------------ fused pipeline (device)
    def forward_layer_device(self, layer, params, dstream: DeviceStream) -> _LayerRun:
        require_cuda()
        lib = _lib.lib()
        B, E = dstream.batch, dstream.capacity
        n = layer.n_neurons
        qd, vth = quant_desc(params, self.round_mode, n)
        q_dev = to_device(np.asarray(params.q).reshape(layer.weight_shape), np.int32)
        lut_dev = to_device(np.asarray(params.decay_table_int, dtype=np.int32).reshape(-1),
                            np.int32) if qd.lut_len else None
        vth_dev = to_device(vth, np.int32) if vth is not None else None
        M = int(layer.max_out_spikes)
        out_t = empty((B, M), np.float32)
        out_s = empty((B, M), np.int32)
        out_n = empty((B,), np.int32)
        v_final = empty((B, n), np.int32)
        stats = zeros((6, B), np.int32)
        sin = _lib.StreamIn(ptr(dstream.times), ptr(dstream.src), ptr(dstream.n_real), E,
                            int(dstream.virtual_pads))
        sout = _lib.StreamOut(ptr(out_t), ptr(out_s), ptr(out_n))
        st = _lib.LayerStats(*[ptr(stats[i]) for i in range(6)])
        nbytes = ctypes.c_size_t(0)
        if is_conv(layer):
            d = conv_desc(layer)
            _lib.check(lib.salt_conv_layer_workspace_size(_lib.byref(d), _lib.byref(qd), B, E,
                                                          _lib.byref(nbytes)))
            ws = workspace(nbytes.value)
            _lib.check(lib.salt_conv_layer_forward(
                _lib.byref(d), _lib.byref(qd), ptr(q_dev), ptr(lut_dev), ptr(vth_dev), B,
                _lib.byref(sin), _lib.byref(sout), ptr(v_final), _lib.byref(st), ptr(ws),
                nbytes.value, stream_handle()))
        else:
            d = fc_desc(layer)
            _lib.check(lib.salt_fc_layer_workspace_size(_lib.byref(d), _lib.byref(qd), B, E,
                                                        _lib.byref(nbytes)))
            ws = workspace(nbytes.value)
            _lib.check(lib.salt_fc_layer_forward(
                _lib.byref(d), _lib.byref(qd), ptr(q_dev), ptr(lut_dev), ptr(vth_dev), B,
                _lib.byref(sin), _lib.byref(sout), ptr(v_final), _lib.byref(st), ptr(ws),
                nbytes.value, stream_handle()))
        # Temporaries (weights, workspace) may be released now: their memory is freed in stream
        # order on this stream, after these kernels.
        return _LayerRun(DeviceStream(out_t, out_s, out_n, True), v_final, stats)

    def trace_layer_device(self, layer, params, dstream: DeviceStream, *, dense: bool = True,
                           per_neuron: bool = True) -> dict:
        """Per-column trace of one layer over a device stream (salt_conv_layer_trace /
        salt_fc_layer_trace): dense (B, n, L) v_steps / spike_mask / event_ms and per-neuron
        first-overflow records, as device arrays keyed by field name."""
        require_cuda()
        lib = _lib.lib()
        B, E = dstream.batch, dstream.capacity
        n = layer.n_neurons
        conv = is_conv(layer)
        L = int(layer.max_queue_len) if conv else E
        qd, vth = quant_desc(params, self.round_mode, n)
        q_dev = to_device(np.asarray(params.q).reshape(layer.weight_shape), np.int32)
        lut_dev = to_device(np.asarray(params.decay_table_int, dtype=np.int32).reshape(-1),
                            np.int32) if qd.lut_len else None
        vth_dev = to_device(vth, np.int32) if vth is not None else None
        out = {}
        if dense:
            out["v_steps"] = empty((B, n, L), np.int32)
            out["spike_mask"] = empty((B, n, L), np.uint8)
            out["event_ms"] = empty((B, n, L), np.float32)
        rec = None
        if per_neuron:
            names = [f for f, _ in _lib.NeuronTrace._fields_]
            for f in names:
                out[f] = empty((B, n), np.float32 if f == "time_ms" else np.int32)
            rec = _lib.NeuronTrace(*[ptr(out[f]) for f in names])
        sin = _lib.StreamIn(ptr(dstream.times), ptr(dstream.src), ptr(dstream.n_real), E,
                            int(dstream.virtual_pads))
        desc = conv_desc(layer) if conv else fc_desc(layer)
        fn = lib.salt_conv_layer_trace if conv else lib.salt_fc_layer_trace
        _lib.check(fn(_lib.byref(desc), _lib.byref(qd), ptr(q_dev), ptr(lut_dev), ptr(vth_dev), B,
                      _lib.byref(sin), ptr(out.get("v_steps")), ptr(out.get("spike_mask")),
                      ptr(out.get("event_ms")), _lib.byref(rec) if rec is not None else None,
                      stream_handle()))
        return out

    @staticmethod
    def _layer_trace(tr: dict):
        from .trace import LayerForwardTrace
        return LayerForwardTrace(spike_mask=tr["spike_mask"].numpy().astype(bool),
                                 v_steps=tr["v_steps"].numpy(),
                                 event_ms=tr["event_ms"].numpy())

    # ------------------------------------------------------------ host-level API
    @staticmethod
    def _host_layer(layer, run: _LayerRun, n_in: np.ndarray) -> tuple:
        stats = run.stats.numpy()
        v_final = run.v_final.numpy()
        S = stats[0].astype(np.int32)
        result = QuantLayerResult(v_final=v_final, spike_count=S, overflowed=stats[2] != 0,
                                  v_unfitted_min=stats[3].copy(), v_unfitted_max=stats[4].copy())
        denom = np.float32(layer.n_neurons) * np.maximum(n_in, 1).astype(np.float32)
        needed = {"max_out_spikes": S, "max_extra_steps": np.zeros_like(S)}
        if is_conv(layer):
            needed = {"max_queue_len": stats[1].astype(np.int32), **needed}
        diag = LayerDiag(spike_count=S, firing_rate=S.astype(np.float32) / denom, needed=needed)
        return result, diag, stats[5] != 0

    def forward_layer(self, layer, params, in_stream: EventStream, *, trace: bool = False
                      ) -> LayerOutput:
        """ConvLayer.forward / FCLayer.forward with QuantBackend (batched or single sample).
        trace=True adds the per-column trajectories (LayerForwardTrace) from the trace kernels."""
        single = np.ndim(in_stream.event_times) == 1
        dstream = DeviceStream.from_host(in_stream)
        run = self.forward_layer_device(layer, params, dstream)
        tr = self._layer_trace(self.trace_layer_device(layer, params, dstream, per_neuron=False)
                               ) if trace else None
        n_in = np.atleast_1d(np.asarray(in_stream.n_real_events)).astype(np.int64)
        result, diag, _ = self._host_layer(layer, run, n_in)
        stream = run.out.to_host()
        if single:
            result = QuantLayerResult(*(np.asarray(f)[0] for f in result))
            diag = LayerDiag(diag.spike_count[0], diag.firing_rate[0],
                             {k: v[0] for k, v in diag.needed.items()})
            stream = EventStream(stream.event_times[0], stream.event_source_idx[0],
                                 stream.event_gain[0], stream.n_real_events[0])
            if tr is not None:
                tr = type(tr)(*(f[0] for f in tr))
        return LayerOutput(stream=stream, result=result, diag=diag, trace=tr)

    def run_network(self, layers, weights, input_stream: EventStream, *, trace: bool = False,
                    keep_streams: bool = False) -> NetworkOutput:
        """network.py:93-122 on the device; intermediate streams never leave the GPU.
        trace=True also returns each layer's LayerForwardTrace (network.py:93-122)."""
        single = np.ndim(input_stream.event_times) == 1
        cur = DeviceStream.from_host(input_stream)
        runs, n_ins, traces = [], [], []
        n_in = np.atleast_1d(np.asarray(input_stream.n_real_events)).astype(np.int64)
        for layer, p in zip(layers, weights):
            if trace:
                traces.append(self._layer_trace(self.trace_layer_device(layer, p, cur,
                                                                        per_neuron=False)))
            run = self.forward_layer_device(layer, p, cur)
            runs.append((run, n_in, run.out if keep_streams else None))
            cur = run.out
            n_in = None  # filled from the device stats below
        results, diags, fits, streams = [], [], None, []
        prev_S = np.atleast_1d(np.asarray(input_stream.n_real_events)).astype(np.int64)
        for layer, (run, _, keep) in zip(layers, runs):
            r, d, f = self._host_layer(layer, run, prev_S)
            prev_S = r.spike_count.astype(np.int64)
            results.append(r)
            diags.append(d)
            fits = f if fits is None else (fits & f)
            if keep is not None:
                streams.append(keep.to_host())
        out = NetworkOutput(tuple(results), tuple(diags), tuple(traces) if trace else None, fits,
                            tuple(streams))
        if single:
            out = NetworkOutput(
                tuple(QuantLayerResult(*(np.asarray(f)[0] for f in r)) for r in out.results),
                tuple(LayerDiag(d.spike_count[0], d.firing_rate[0],
                                {k: v[0] for k, v in d.needed.items()}) for d in out.diags),
                tuple(type(t)(*(f[0] for f in t)) for t in traces) if trace else None,
                out.fits[0],
                tuple(EventStream(s.event_times[0], s.event_source_idx[0], s.event_gain[0],
                                  s.n_real_events[0]) for s in out.streams))
        return out

    def readout(self, result, params):
        """salt_core/quant/backend.py:55-63: v_final -> v * 2^-f_V * s_c (float32)."""
        v = (np.asarray(result.v_final).astype(np.float32) * np.float32(2.0 ** -params.f_V)
             * np.asarray(params.scale, dtype=np.float32))
        return result._replace(v_final=v)

    # ------------------------------------------------------------ Backend.scan plug-in
    def scan(self, layer, structure, params, event_gain, *, trace: bool) -> ScanOutput:
        """salt_core/quant/backend.py:31-53 on materialised queues, integer scan on the GPU.
        The layer supplies the queue's Δt and weight codes through its ScanLayer accessors
        (neuron_delta_t, gather_weight_codes); event_gain is unused (the integer path's gain is
        1).  trace=True adds v_steps, the register after every column, and pointer_steps, the
        column index (quant/backend.py:41-43)."""
        check_weight_codes(params.q)
        delta_t = np.asarray(layer.neuron_delta_t(structure), dtype=np.float32)
        a_int, is_identity = apply_decay_table_int(delta_t, params.decay_table_int)
        q_int = np.asarray(layer.gather_weight_codes(structure, params.q), dtype=np.int32)
        res = self.scan_dense(a_int, is_identity, q_int, params.v_th_int, f_a=params.f_a,
                              f_V=params.f_V, i_V=params.i_V,
                              overflow_mode=getattr(params, "overflow_mode", "wrap"),
                              trace=trace)
        v_steps = None
        if trace:
            res, v_steps = res
        return ScanOutput(result=res, spike_gain=np.ones_like(res.spike_mask, dtype=np.float32),
                          extra_steps_needed=np.zeros((), np.int32), v_steps=v_steps,
                          pointer_steps=res.spike_event_idx if trace else None)

    def scan_dense(self, a_int, is_identity, q_int, v_th_int, *, f_a, f_V, i_V,
                   overflow_mode="wrap", trace: bool = False):
        """quant/scan.py:65-80 run_layer on the GPU; with trace=True, run_layer_traced
        (:83-94): returns (result, v_steps (n, L))."""
        require_cuda()
        check_bit_widths(int(f_a), int(f_V), int(i_V))
        a = np.ascontiguousarray(a_int, dtype=np.int32)
        n, L = a.shape
        from .quant import QuantizedLayerParams
        qd, vth = quant_desc(QuantizedLayerParams(np.zeros(1, np.int32), np.zeros(0, np.int32),
                                                  v_th_int, 1.0, f_a, f_V, i_V, overflow_mode),
                             self.round_mode, n)
        a_d = to_device(a, np.int32)
        id_d = to_device(np.asarray(is_identity, dtype=np.uint8), np.uint8)
        q_d = to_device(np.asarray(q_int), np.int32)
        vth_d = to_device(vth, np.int32) if vth is not None else None
        mask = empty((n, L), np.uint8)
        ovf = empty((n, L), np.uint8)
        vf, lo, hi = (empty((n,), np.int32) for _ in range(3))
        args = (_lib.byref(qd), n, L, ptr(a_d), ptr(id_d), ptr(q_d), ptr(vth_d), ptr(mask),
                ptr(ovf), ptr(vf), ptr(lo), ptr(hi))
        steps = None
        if trace:
            steps = empty((n, L), np.int32)
            _lib.check(_lib.lib().salt_quant_scan_dense_trace(*args, ptr(steps),
                                                              stream_handle()))
        else:
            _lib.check(_lib.lib().salt_quant_scan_dense(*args, stream_handle()))
        m = mask.numpy().astype(bool)
        res = DenseQuantLayerResult(spike_mask=m,
                                    spike_event_idx=np.broadcast_to(np.arange(L), (n, L)),
                                    v_final=vf.numpy(), overflowed=ovf.numpy() != 0,
                                    v_unfitted_min=lo.numpy(), v_unfitted_max=hi.numpy())
        return (res, steps.numpy()) if trace else res

    # ------------------------------------------------------------ compiled network
    def compile(self, layers, weights, batch: int, in_capacity: int):
        """A native network plan (C++ runtime object) for repeated batched forwards."""
        from .plan import NetworkPlan
        return NetworkPlan(list(layers), list(weights), batch, in_capacity, self.round_mode)


_DEFAULT = None


def default_backend() -> QuantB200Backend:
    global _DEFAULT
    if _DEFAULT is None:
        _DEFAULT = QuantB200Backend()
    return _DEFAULT
