"""NetworkPlan: the native network runtime object of libsalt_b200 (salt_network_*).

Parameters are uploaded once; every intermediate stream lives in one workspace; a forward is a
fixed sequence of kernel launches on the caller's stream with no host synchronisation, so it can
be timed with CUDA events or replayed from a CUDA graph.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .backend import conv_desc, fc_desc, quant_desc
from .device import (Event, Graph, Stream, current_stream, empty, pinned_empty, ptr, require_cuda,
                     stream_handle, to_device, use_stream, workspace)
from .layers import is_conv


class NetworkPlan:
    def __init__(self, layers, weights, batch: int, in_capacity: int, round_mode="round"):
        require_cuda()
        self.layers, self.batch, self.in_capacity = list(layers), int(batch), int(in_capacity)
        lib = _lib.lib()
        specs = (_lib.LayerSpec * len(self.layers))()
        self._host = []
        for i, (layer, p) in enumerate(zip(self.layers, weights)):
            qd, vth = quant_desc(p, round_mode, layer.n_neurons)
            q = np.ascontiguousarray(np.asarray(p.q).reshape(layer.weight_shape), dtype=np.int32)
            lut = np.ascontiguousarray(np.asarray(p.decay_table_int), dtype=np.int32)
            self._host += [q, lut, vth]
            spec = specs[i]
            if is_conv(layer):
                spec.kind, spec.conv = 0, conv_desc(layer)
            else:
                spec.kind, spec.fc = 1, fc_desc(layer)
            spec.quant = qd
            spec.q_host = q.ctypes.data
            spec.lut_host = lut.ctypes.data if lut.size else None
            spec.vth_host = vth.ctypes.data if vth is not None else None
        self._net = ctypes.c_void_p()
        _lib.check(lib.salt_network_create(specs, len(self.layers), ctypes.byref(self._net)))
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.salt_network_workspace_size(self._net, self.batch, self.in_capacity,
                                                   ctypes.byref(nbytes)))
        self.workspace_bytes = nbytes.value
        self._ws = workspace(self.workspace_bytes)
        nl, B = len(self.layers), self.batch
        self.n_out = self.layers[-1].n_neurons
        self.logits = empty((B, self.n_out), np.int32)
        self.stats = empty((5, nl, B), np.int32)
        self.fits = empty((B,), np.int32)
        self._graph = None

    def forward_device(self, times, src, n_real, virtual_pads: bool = False):
        """Enqueue one batched forward on the current stream (inputs already on the device).
        Returns (logits, stats, fits) device arrays; stats rows are spike_count, overflowed,
        vmin, vmax, needed_queue, each (n_layers, B)."""
        sin = _lib.StreamIn(ptr(times), ptr(src), ptr(n_real), int(times.shape[1]),
                            int(virtual_pads))
        s = self.stats
        _lib.check(_lib.lib().salt_network_forward(
            self._net, self.batch, _lib.byref(sin), ptr(self.logits), ptr(s[0]), ptr(s[1]),
            ptr(s[2]), ptr(s[3]), ptr(s[4]), ptr(self.fits), ptr(self._ws),
            self.workspace_bytes, stream_handle()))
        return self.logits, self.stats, self.fits

    def forward_part(self, times, src, n_real, row0: int, rows: int, layer_begin: int,
                     layer_end: int, virtual_pads: bool = False):
        """Layers [layer_begin, layer_end) on rows [row0, row0 + rows) of this plan's batch
        (salt_network_forward_part).  With layer_begin == 0 the inputs are that row slice
        (rows, in_capacity); later parts read what the previous layer left in the workspace, so
        parts are enqueued in layer order.  Outputs land in the full-batch (logits, stats, fits)
        returned by forward_device; logits and fits only when layer_end is the last layer."""
        sin = None
        if layer_begin == 0:
            sin = _lib.StreamIn(ptr(times), ptr(src), ptr(n_real), int(times.shape[1]),
                                int(virtual_pads))
        s = self.stats
        _lib.check(_lib.lib().salt_network_forward_part(
            self._net, self.batch, self.in_capacity, int(row0), int(rows), int(layer_begin),
            int(layer_end), _lib.byref(sin) if sin is not None else None, ptr(self.logits),
            ptr(s[0]), ptr(s[1]), ptr(s[2]), ptr(s[3]), ptr(s[4]), ptr(self.fits), ptr(self._ws),
            self.workspace_bytes, stream_handle()))
        return self.logits, self.stats, self.fits

    def capture(self, times, src, n_real, virtual_pads: bool = False):
        """Records forward_device on these device buffers as a CUDA graph and returns its replay
        function: one launch per forward instead of one per kernel (launch-bound batches gain,
        large ones do not).  Refill the same buffers between replays; the results appear in the
        arrays forward_device returns.  Profiling must be off while capturing."""
        side = Stream()
        side.wait_stream(current_stream())
        with use_stream(side):   # first call outside the capture: kernel attributes set
            self.forward_device(times, src, n_real, virtual_pads)
        current_stream().wait_stream(side)
        with Graph.capture(side) as graph:
            self.forward_device(times, src, n_real, virtual_pads)
        self._graph = (graph, side)   # kept alive with the plan
        return lambda: graph.replay(current_stream())

    def set_profiling(self, enable: bool) -> None:
        _lib.check(_lib.lib().salt_network_set_profiling(self._net, int(bool(enable))))

    def profile_read(self, reset: bool = True):
        """(fused-kernel ms summed per layer, whole-layer ms summed per layer, timed forwards)."""
        nl = len(self.layers)
        fused = np.zeros(nl, np.float32)
        whole = np.zeros(nl, np.float32)
        n = np.zeros(nl, np.int32)
        _lib.check(_lib.lib().salt_network_profile_read(
            self._net, fused.ctypes.data_as(ctypes.c_void_p), whole.ctypes.data_as(ctypes.c_void_p),
            n.ctypes.data_as(ctypes.c_void_p), int(bool(reset))))
        return fused, whole, n

    def last_launch_count(self) -> int:
        return int(_lib.lib().salt_network_last_launch_count(self._net))

    def __call__(self, raw):
        """Host in, host out (the end-to-end path): returns (logits, spike_count, fits) numpy."""
        t = to_device(np.asarray(raw.event_times, dtype=np.float32), np.float32)
        s = to_device(np.asarray(raw.source_idx), np.int32)
        n = to_device(np.asarray(raw.n_real_events), np.int32)
        logits, stats, fits = self.forward_device(t, s, n)
        return logits.numpy(), stats[0].numpy().T, fits.numpy() != 0

    def close(self) -> None:
        if self._net:
            _lib.lib().salt_network_destroy(self._net)
            self._net = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class OverlappedForward:
    """Consecutive batches with two in flight: two network plans (each with its own workspace)
    on two streams take the batches in turn, and batch k+1's layers start as soon as batch k's
    second-to-last layer is done, so batch k's last layer — a membrane readout whose time is one
    sample's chain, with most of the GPU idle — runs beside batch k+1's first layers.  Every batch
    is computed in full; only the idle tail of one overlaps the head of the next.

    submit() enqueues one batch (device inputs, read-only) after the work already on the caller's
    current stream and returns (logits, stats, fits, done): the outputs of the plan that took it
    and an event recorded when they are final.  A plan's outputs are overwritten two submissions
    later; pass `wait` events (e.g. a collective that reads the logits) that its next batch must
    wait for.  join() makes the current stream wait for everything submitted."""

    def __init__(self, layers, weights, batch: int, in_capacity: int, round_mode="round"):
        require_cuda()
        self.plans = [NetworkPlan(layers, weights, batch, in_capacity, round_mode) for _ in range(2)]
        self.streams = [Stream(), Stream()]
        self.entry = [Event(), Event()]       # the caller's stream reached the submission
        self.head_done = [Event(), Event()]   # a batch's layers but the last are done
        self.done = [Event(), Event()]
        self.n_layers = len(self.plans[0].layers)
        self.batch = int(batch)
        self._waits = [[], []]
        self._k = 0
        self._launches = 0

    def submit(self, times, src, n_real, wait=()):
        i = self._k % 2
        plan, st = self.plans[i], self.streams[i]
        st.wait_event(self.entry[i].record(current_stream()))   # inputs ready
        for ev in list(self._waits[i]) + list(wait):
            st.wait_event(ev)
        self._waits[i] = []
        if self._k > 0:
            st.wait_event(self.head_done[1 - i])             # the previous batch's head is done
        nl, B = self.n_layers, self.batch
        with use_stream(st):
            if nl > 1:
                plan.forward_part(times, src, n_real, 0, B, 0, nl - 1)
                launches = plan.last_launch_count()
                self.head_done[i].record(st)
                plan.forward_part(None, None, None, 0, B, nl - 1, nl)
                launches += plan.last_launch_count()
            else:
                plan.forward_device(times, src, n_real)
                launches = plan.last_launch_count()
                self.head_done[i].record(st)
        self._launches = launches
        self.done[i].record(st)
        self._k += 1
        return plan.logits, plan.stats, plan.fits, self.done[i]

    def hold(self, event) -> None:
        """The plan that took the last batch starts its next batch only after `event` (a reader of
        its outputs, e.g. the logits all-gather)."""
        self._waits[(self._k - 1) % 2].append(event)

    def join(self) -> None:
        for ev in self.done:
            current_stream().wait_event(ev)

    def set_profiling(self, enable: bool) -> None:
        for p in self.plans:
            p.set_profiling(enable)

    def profile_read(self, reset: bool = True):
        """Per-layer fused-kernel ms, whole-layer ms and timed forwards, summed over both plans."""
        parts = [p.profile_read(reset) for p in self.plans]
        return tuple(sum(x[j] for x in parts) for j in range(3))

    def last_launch_count(self) -> int:
        """Kernel launches of the last submission."""
        return self._launches

    def close(self) -> None:
        for st in self.streams:
            st.synchronize()
        for p in self.plans:
            p.close()


class PipelinedForward:
    """Host in, host out, with the transfer overlapped: the batch's first `slice_layers` layers
    run as `chunks` row slices, each starting as soon as its rows are on the device, while the
    next slice is copied on a second (high-priority) stream into its own device buffer; the
    remaining layers then run on the whole batch (salt_network_forward_part).  Calls enqueued
    back to back overlap too: the buffers form a ring of two per slice, so a slice's copy waits
    only for the first layer that read its buffer two calls earlier.  Each sample's row is copied only up to its n_real (salt_stream_h2d_real)
    unless the first layer may fire on pad entries (needs_tail), in which case whole rows are
    copied.

    Host arrays should be pinned numpy arrays (device.pinned_empty / pinned_copy): times (B, E)
    float32, src (B, E) int32, n_real (B,) int32; the real-event gather requires pinned rows.
    Returns pinned (logits (B, n_out) int32, fits (B,) int32) filled in place; with sync=False
    the call returns once everything is enqueued, and the buffers hold the results when the
    current stream reaches the end of the call (the next call reuses them).

    overlap=True keeps two calls in flight: two plans on two streams of this object take the
    calls in turn, and a call's layers start once the previous call's layers but the last are
    done (the last layer, a readout with most of the GPU idle, runs beside the next call's first
    layers).  The caller's current stream then does not wait for a call: `done` is the event
    recorded when the last call's results are on the host, `plan` the plan that computed them
    (its device outputs stay valid until two calls later, or longer with hold()), and join()
    makes the current stream wait for every call."""

    def __init__(self, layers, weights, batch: int, in_capacity: int, chunks: int = 4,
                 round_mode="round", slice_layers: int = 1, overlap: bool = False):
        require_cuda()
        if batch % chunks:
            raise ValueError(f"batch {batch} is not a multiple of chunks {chunks}")
        self.batch, self.chunks, self.sub = int(batch), int(chunks), int(batch) // int(chunks)
        self.capacity = int(in_capacity)
        self.overlap = bool(overlap)
        self.plans = [NetworkPlan(layers, weights, self.batch, self.capacity, round_mode)
                      for _ in range(2 if self.overlap else 1)]
        self.plan = self.plans[0]
        self.n_layers = len(self.plan.layers)
        if self.overlap:
            self._streams = [Stream(), Stream()]
            self._entry = [Event(), Event()]
            self._head_done = [Event(), Event()]
            self._done = [Event(), Event()]
            self._waits = [[], []]
        self.done = None
        # layers run per slice as the slice arrives; the rest run once on the whole batch
        self.slice_layers = max(1, min(int(slice_layers), self.n_layers))
        qd, _ = quant_desc(weights[0], round_mode, layers[0].n_neurons)
        self.full_rows = bool(qd.needs_tail)
        E, sub = self.capacity, self.sub
        # a ring of two device buffers per slice: a slice's copy waits only for the first layer
        # that read its buffer two calls earlier, so calls enqueued back to back keep the copy
        # stream busy (a one-slice call's copy overlaps the previous call's whole forward)
        nbuf = 2 * self.chunks
        self._calls = 0
        self._t = [empty((sub, E), np.float32) for _ in range(nbuf)]
        self._s = [empty((sub, E), np.int32) for _ in range(nbuf)]
        self._n = [empty((sub,), np.int32) for _ in range(nbuf)]
        # the gather kernel of the copy stream must get SM slots while a layer fills the GPU
        self._copy = Stream(high_priority=True)
        self._ready = [Event() for _ in range(nbuf)]
        self._free = [Event() for _ in range(nbuf)]
        self._used = [False] * nbuf   # buffer i was handed to a forward (this or an earlier call)
        self.logits = pinned_empty((batch, self.plan.n_out), np.int32)
        self.fits = pinned_empty((batch,), np.int32)

    def h2d_bytes(self, n_real_host) -> int:
        """Bytes one call moves host -> device for these event counts."""
        n = np.minimum(np.maximum(np.asarray(n_real_host), 0), self.capacity)
        rows = n.size * self.capacity if self.full_rows else int(n.sum())
        return int(rows * 8 + n.size * 4)

    def wait_for(self, event) -> None:
        """Orders this object's transfers after `event` (e.g. the start of a timed region)."""
        self._copy.wait_event(event)

    def hold(self, event) -> None:
        """overlap=True: the plan of the last call takes its next call only after `event` (a
        reader of its device outputs, e.g. a logits all-gather)."""
        self._waits[(self._calls - 1) % 2].append(event)

    def join(self) -> None:
        """Makes the current stream wait for every call enqueued so far."""
        if self.overlap:
            for ev in self._done:
                current_stream().wait_event(ev)

    def __call__(self, times_h, src_h, n_real_h, sync: bool = True, out=None):
        """out = (logits (B, n_out) int32, fits (B,) int32) pinned host arrays to receive this
        call's results instead of the object's own buffers (calls enqueued back to back with
        sync=False then keep their results apart)."""
        lib = _lib.lib()
        call = self._calls
        self._calls += 1
        if self.overlap:
            j = call % 2
            plan, compute = self.plans[j], self._streams[j]
            compute.wait_event(self._entry[j].record(current_stream()))
            for ev in self._waits[j]:
                compute.wait_event(ev)
            self._waits[j] = []
            if call > 0:   # the previous call's layers but its last are done
                compute.wait_event(self._head_done[1 - j])
        else:
            plan, compute = self.plans[0], current_stream()
        self.plan = plan
        with use_stream(compute):
            out = self._enqueue(lib, plan, compute, call, times_h, src_h, n_real_h, out)
        if self.overlap:
            self.done = self._done[call % 2].record(compute)
        if sync:
            compute.synchronize()
        return out

    def _enqueue(self, lib, plan, compute, call, times_h, src_h, n_real_h, out):
        sub, E = self.sub, self.capacity
        per_slice, nl = self.slice_layers, self.n_layers
        base = (call % 2) * self.chunks
        for k in range(self.chunks):
            i = base + k
            rows = slice(k * sub, (k + 1) * sub)
            copy = self._copy
            if self._used[i]:   # the forward that last read buffer i, in any call
                copy.wait_event(self._free[i])
            self._n[i].copy_from(n_real_h[rows], stream=copy)
            if self.full_rows:
                self._t[i].copy_from(times_h[rows], stream=copy)
                self._s[i].copy_from(src_h[rows], stream=copy)
            else:
                _lib.check(lib.salt_stream_h2d_real(
                    ptr(times_h[rows]), ptr(src_h[rows]), ctypes.c_int64(times_h.shape[1]),
                    ptr(self._n[i]), sub, E, ptr(self._t[i]), ptr(self._s[i]), copy.ptr))
            self._ready[i].record(copy)
            compute.wait_event(self._ready[i])
            plan.forward_part(self._t[i], self._s[i], self._n[i], k * sub, sub, 0, per_slice)
            self._free[i].record(compute)
            self._used[i] = True
        # the remaining layers on the whole batch; with overlap, the last one after head_done
        head_end = max(per_slice, nl - 1) if self.overlap else nl
        if per_slice < head_end:
            plan.forward_part(None, None, None, 0, self.batch, per_slice, head_end)
        if self.overlap:
            self._head_done[call % 2].record(compute)
        if head_end < nl:
            plan.forward_part(None, None, None, 0, self.batch, head_end, nl)
        logits_h, fits_h = out if out is not None else (self.logits, self.fits)
        plan.logits.copy_to(logits_h, sync=False, stream=compute)
        plan.fits.copy_to(fits_h, sync=False, stream=compute)
        return logits_h, fits_h

    def close(self) -> None:
        self._copy.synchronize()   # no copy still writes into the buffers about to be freed
        for st in (self._streams if self.overlap else []):
            st.synchronize()
        current_stream().synchronize()
        for plan in self.plans:
            plan.close()
