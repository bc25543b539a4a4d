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
from .device import current_stream, ptr, require_cuda, to_device, workspace
from .layers import is_conv

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


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
        self.logits = torch.empty((B, self.n_out), dtype=torch.int32, device="cuda")
        self.stats = torch.empty((5, nl, B), dtype=torch.int32, device="cuda")
        self.fits = torch.empty((B,), dtype=torch.int32, device="cuda")

    def forward_device(self, times, src, n_real, virtual_pads: bool = False):
        """Enqueue one batched forward on the current stream (inputs already on the device).
        Returns (logits, stats, fits) device tensors; stats rows are spike_count, overflowed,
        vmin, vmax, needed_queue, each (n_layers, B)."""
        sin = _lib.StreamIn(ptr(times), ptr(src), ptr(n_real), int(times.shape[1]),
                            int(virtual_pads))
        s = self.stats
        _lib.check(_lib.lib().salt_network_forward(
            self._net, self.batch, _lib.byref(sin), ptr(self.logits), ptr(s[0]), ptr(s[1]),
            ptr(s[2]), ptr(s[3]), ptr(s[4]), ptr(self.fits), ptr(self._ws),
            self.workspace_bytes, current_stream()))
        return self.logits, self.stats, self.fits

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
        return logits.cpu().numpy(), stats[0].cpu().numpy().T, fits.cpu().numpy() != 0

    def close(self) -> None:
        if self._net:
            _lib.lib().salt_network_destroy(self._net)
            self._net = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
