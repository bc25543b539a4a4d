"""FloatB200Backend: the float chunked affine scan of FC layers on B200.

Mirrors FCLayer.forward with FloatBackend (salt_core/layers/fc.py:84-106, float/backend.py:16-31,
float/scan.py:34-50, float/affine.py:99-126, stream.py:67-81) for the forward values:
``FloatLayerResult.v_final``, the output EventStream (gain 1 on every real entry, the forward value
of s_spike) and LayerDiag with the reference's ``needed`` (max_out_spikes, max_extra_steps).
Computed by ``salt_float_fc_layer_forward`` (libsalt_b200, include/salt_b200.h); no CPU fallback.

Extension beyond the reference API: ``tau`` may be given per neuron (an (n_out,) array
overriding FCLayer.tau); neurons are independent, so each neuron behaves as a one-neuron layer
with its own tau.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np

from . import _lib
from .capacity import LayerDiag
from .device import DeviceStream, current_stream, ptr, require_cuda, to_device, workspace
from .layers import LayerOutput, is_conv
from .stream import EventStream

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


class FloatLayerResult(NamedTuple):
    """Forward values of float/scan.py:10-16, batched.  The per-step arrays of the reference
    (spike_mask, spike_event_idx, s_spike, s_value of shape (n, max_steps)) carry no more than the
    output stream does in a forward pass (s_spike = s_value = spike_mask there), so the layer
    returns the stream instead; spike_count = Σ spike_mask."""
    v_final: np.ndarray
    spike_count: np.ndarray


class NetworkOutput(NamedTuple):
    """salt_core/network.py:157-167 for a chain of float FC layers, batched."""
    results: tuple
    diags: tuple
    traces: tuple | None
    fits: np.ndarray
    streams: tuple = ()

    @property
    def last(self):
        return self.results[-1]


class _FloatRun(NamedTuple):
    out: DeviceStream
    v_final: "torch.Tensor"
    stats: "torch.Tensor"   # (3, B): spike_count, needed_extra_steps, fits


def decay_base(tau, n_out: int) -> np.ndarray:
    """float32(1 - 1/tau) per neuron: the base that create_affine_maps (float/affine.py:27-31)
    raises to the Δt power (a Python-float base meeting a float32 array becomes float32)."""
    t = np.broadcast_to(np.asarray(tau, dtype=np.float64), (n_out,))
    if np.any(~np.isfinite(t)) or np.any(t == 0):
        raise ValueError("tau must be finite and non-zero")
    return np.ascontiguousarray((1.0 - 1.0 / t).astype(np.float32))


def float_desc(layer) -> _lib.FloatFCDesc:
    if is_conv(layer):
        raise NotImplementedError("the B200 float path covers FC layers (float conv layers are "
                                  "not built)")
    if not float(layer.v_th) > 0.0 or not np.isfinite(float(layer.v_th)):
        raise ValueError("float FC layer: v_th must be finite and > 0 (a threshold <= 0 fires on "
                         "pad entries)")
    return _lib.FloatFCDesc(int(layer.n_in), int(layer.n_out), int(layer.chunk_size),
                            int(layer.max_out_spikes), int(layer.max_extra_steps),
                            float(layer.v_th))


def _unit_gains(stream: EventStream) -> bool:
    g = np.asarray(stream.event_gain, dtype=np.float32)
    t = np.asarray(stream.event_times)
    n = np.atleast_1d(np.asarray(stream.n_real_events)).astype(np.int64)
    if g.ndim == 1:
        g, t = g[None], t[None]
    real = np.arange(g.shape[1])[None, :] < n[:, None]
    return bool(np.all(np.where(real, g, 1.0) == 1.0))


class FloatLayerPlan:
    """One float FC layer prepared for repeated batched forwards: weights, decay bases, output
    buffers and the workspace live on the device; each forward is one C-ABI call on the current
    stream over a device-resident stream of the planned shape."""

    def __init__(self, layer, w, batch: int, in_capacity: int, *, tau=None, gain: bool = False):
        require_cuda()
        self.layer, self.batch, self.capacity, self.gain = layer, int(batch), int(in_capacity), gain
        self.desc = float_desc(layer)
        n = int(layer.n_out)
        self.w = to_device(np.asarray(w, dtype=np.float32).reshape(n, int(layer.n_in)), np.float32)
        self.base = to_device(decay_base(layer.tau if tau is None else tau, n), np.float32)
        B, M = self.batch, int(layer.max_out_spikes)
        self.out_t = torch.empty((B, M), dtype=torch.float32, device="cuda")
        self.out_s = torch.empty((B, M), dtype=torch.int32, device="cuda")
        self.out_n = torch.empty((B,), dtype=torch.int32, device="cuda")
        self.v_final = torch.empty((B, n), dtype=torch.float32, device="cuda")
        self.stats = torch.zeros((3, B), dtype=torch.int32, device="cuda")
        self._st = _lib.FloatLayerStats(*[ptr(self.stats[i]) for i in range(3)])
        self._sout = _lib.StreamOut(ptr(self.out_t), ptr(self.out_s), ptr(self.out_n))
        nbytes = ctypes.c_size_t(0)
        _lib.check(_lib.lib().salt_float_fc_layer_workspace_size(
            _lib.byref(self.desc), B, self.capacity, int(gain), _lib.byref(nbytes)))
        self.ws_bytes = nbytes.value
        self.ws = workspace(self.ws_bytes)

    def forward_device(self, dstream: DeviceStream, gain: "torch.Tensor | None" = None
                       ) -> _FloatRun:
        if (dstream.batch, dstream.capacity) != (self.batch, self.capacity):
            raise ValueError(f"stream shape {(dstream.batch, dstream.capacity)} does not match the "
                             f"plan's {(self.batch, self.capacity)}")
        if (gain is not None) != self.gain:
            raise ValueError("gain given to a plan built without it, or missing")
        sin = _lib.StreamIn(ptr(dstream.times), ptr(dstream.src), ptr(dstream.n_real),
                            self.capacity, int(dstream.virtual_pads))
        _lib.check(_lib.lib().salt_float_fc_layer_forward(
            _lib.byref(self.desc), ptr(self.w), ptr(self.base), self.batch, _lib.byref(sin),
            ptr(gain), _lib.byref(self._sout), ptr(self.v_final), _lib.byref(self._st),
            ptr(self.ws), self.ws_bytes, current_stream()))
        return _FloatRun(DeviceStream(self.out_t, self.out_s, self.out_n, True), self.v_final,
                         self.stats)


def set_profiling(enable: bool) -> None:
    """Time each float layer this thread enqueues (segment kernel and whole layer)."""
    _lib.check(_lib.lib().salt_float_fc_set_profiling(int(bool(enable))))


def profile_read(reset: bool = True) -> tuple[float, float, int]:
    """(segment kernel ms, whole layer ms, layers timed) summed since the last reset."""
    seg, lay, n = ctypes.c_float(0), ctypes.c_float(0), ctypes.c_int32(0)
    _lib.check(_lib.lib().salt_float_fc_profile_read(_lib.byref(seg), _lib.byref(lay),
                                                     _lib.byref(n), int(bool(reset))))
    return float(seg.value), float(lay.value), int(n.value)


@dataclass(frozen=True)
class FloatB200Backend:
    """FloatBackend's drop-in for FC layers (forward values) on B200."""

    def compile(self, layer, w, batch: int, in_capacity: int, *, tau=None, gain: bool = False
                ) -> FloatLayerPlan:
        return FloatLayerPlan(layer, w, batch, in_capacity, tau=tau, gain=gain)

    def forward_layer_device(self, layer, w, dstream: DeviceStream, *, tau=None,
                             gain: "torch.Tensor | None" = None) -> _FloatRun:
        """One batched layer on device-resident streams; gain (B, capacity) or None (ones)."""
        plan = FloatLayerPlan(layer, w, dstream.batch, dstream.capacity, tau=tau,
                              gain=gain is not None)
        return plan.forward_device(dstream, gain)

    @staticmethod
    def _host_layer(layer, run: _FloatRun, n_in: np.ndarray):
        stats = run.stats.cpu().numpy()
        S = stats[0].astype(np.int32)
        result = FloatLayerResult(v_final=run.v_final.cpu().numpy(), spike_count=S)
        denom = np.float32(layer.n_out) * np.maximum(n_in, 1).astype(np.float32)
        diag = LayerDiag(spike_count=S, firing_rate=S.astype(np.float32) / denom,
                         needed={"max_out_spikes": S, "max_extra_steps": stats[1].astype(np.int32)})
        return result, diag, stats[2] != 0

    def forward_layer(self, layer, w, in_stream: EventStream, *, tau=None, trace: bool = False
                      ) -> LayerOutput:
        """FCLayer.forward(w, in_stream, backend=FLOAT) (batched or single sample)."""
        if trace:
            raise NotImplementedError("trace=True (per-step trajectories) is not part of the B200 "
                                      "float path")
        single = np.ndim(in_stream.event_times) == 1
        dstream = DeviceStream.from_host(in_stream)
        gain = None
        if not _unit_gains(in_stream):
            g = np.asarray(in_stream.event_gain, dtype=np.float32)
            gain = to_device(g[None] if single else g, np.float32)
        run = self.forward_layer_device(layer, w, dstream, tau=tau, gain=gain)
        n_in = np.atleast_1d(np.asarray(in_stream.n_real_events)).astype(np.int64)
        result, diag, _ = self._host_layer(layer, run, n_in)
        stream = run.out.to_host()  # gains: 1 on every entry
        if single:
            result = FloatLayerResult(result.v_final[0], result.spike_count[0])
            diag = LayerDiag(diag.spike_count[0], diag.firing_rate[0],
                             {k: v[0] for k, v in diag.needed.items()})
            stream = EventStream(stream.event_times[0], stream.event_source_idx[0],
                                 stream.event_gain[0], stream.n_real_events[0])
        return LayerOutput(stream=stream, result=result, diag=diag, trace=None)

    def run_network(self, layers, weights, input_stream: EventStream, *, taus=None,
                    trace: bool = False, keep_streams: bool = False) -> NetworkOutput:
        """network.py:93-122 for a chain of float FC layers; the intermediate streams stay on
        the device (their gains are 1).  taus: optional per-layer tau overrides."""
        if trace:
            raise NotImplementedError("trace=True is not part of the B200 float path")
        single = np.ndim(input_stream.event_times) == 1
        cur = DeviceStream.from_host(input_stream)
        gain = None
        if not _unit_gains(input_stream):
            g = np.asarray(input_stream.event_gain, dtype=np.float32)
            gain = to_device(g[None] if single else g, np.float32)
        runs = []
        for i, (layer, w) in enumerate(zip(layers, weights)):
            tau = None if taus is None else taus[i]
            run = self.forward_layer_device(layer, w, cur, tau=tau, gain=gain)
            runs.append(run)
            cur, gain = run.out, None
        results, diags, fits, streams = [], [], None, []
        prev = np.atleast_1d(np.asarray(input_stream.n_real_events)).astype(np.int64)
        for layer, run in zip(layers, runs):
            r, d, f = self._host_layer(layer, run, prev)
            prev = r.spike_count.astype(np.int64)
            results.append(r)
            diags.append(d)
            fits = f if fits is None else (fits & f)
            if keep_streams:
                streams.append(run.out.to_host())
        out = NetworkOutput(tuple(results), tuple(diags), None, fits, tuple(streams))
        if single:
            out = NetworkOutput(
                tuple(FloatLayerResult(r.v_final[0], r.spike_count[0]) for r in out.results),
                tuple(LayerDiag(d.spike_count[0], d.firing_rate[0],
                                {k: v[0] for k, v in d.needed.items()}) for d in out.diags),
                None, out.fits[0],
                tuple(EventStream(s.event_times[0], s.event_source_idx[0], s.event_gain[0],
                                  s.n_real_events[0]) for s in out.streams))
        return out

    def readout(self, result, params):
        """float/backend.py:33-35: the float path is already at physical scale."""
        return result
