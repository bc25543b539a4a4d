"""Per-channel membrane ranges for quantisation (salt_core/quant/calibrate.py:16-55) and the
calibration forward of example/quant_run.py:30-44 on the B200 float path.

``v_range_per_channel`` / ``merge_v_ranges`` / ``v_abs_max_per_channel`` are the reference's
host functions over per-step traces.  ``calibrate_v_abs_max`` runs the float forward with
chunk_size 1 on the GPU, which reduces each layer's per-step potentials to per-(sample, channel)
extremes on the device, so no (n, steps) trace is materialised.
"""
from __future__ import annotations

from collections.abc import Sequence

import numpy as np

VRange = tuple[np.ndarray, np.ndarray]


def _steps(trace) -> np.ndarray:
    return np.asarray(getattr(trace, "v_steps", trace))


def v_range_per_channel(layers: Sequence, traces: Sequence) -> list[VRange]:
    """calibrate.py:16-36: each layer's per-channel (v_max, v_min) over neurons and steps of one
    sample's traces ((n, steps) arrays or objects with ``v_steps``).  Every layer must run with
    chunk_size 1 (the traces hold only chunk-end values otherwise): ValueError."""
    not_one = [l.name for l in layers if l.chunk_size != 1]
    if not_one:
        raise ValueError(f"membrane ranges need chunk_size=1; these layers differ: {not_one}")
    ranges = []
    for layer, trace in zip(layers, traces):
        v = _steps(trace)
        v_max = layer.unflatten_neurons(v.max(axis=1))
        v_min = layer.unflatten_neurons(v.min(axis=1))
        ranges.append((v_max.reshape(v_max.shape[0], -1).max(axis=1),
                       v_min.reshape(v_min.shape[0], -1).min(axis=1)))
    return ranges


def merge_v_ranges(per_sample: Sequence[Sequence[VRange]]) -> list[VRange]:
    """calibrate.py:39-52: maximum of maxima, minimum of minima; at least one entry."""
    if not per_sample:
        raise ValueError("per_sample needs at least one entry")
    merged = []
    for i in range(len(per_sample[0])):
        merged.append((np.max([s[i][0] for s in per_sample], axis=0),
                       np.min([s[i][1] for s in per_sample], axis=0)))
    return merged


def v_abs_max_per_channel(v_ranges: Sequence[VRange]) -> list[np.ndarray]:
    """calibrate.py:55-57: M = max(v_max, |v_min|) per channel."""
    return [np.maximum(v_max, np.abs(v_min)) for v_max, v_min in v_ranges]


def calibrate_v_abs_max(network, weights, raw, batch_size: int, *, backend=None
                        ) -> list[np.ndarray]:
    """example/quant_run.py:30-44: every sample of raw (InputEvents) through the float forward in
    batches; per layer and channel the largest |v| over all samples, neurons and steps.  Each
    layer must have chunk_size 1 (ValueError otherwise)."""
    from .float_backend import FloatB200Backend
    layers = list(network.layers)
    not_one = [l.name for l in layers if l.chunk_size != 1]
    if not_one:
        raise ValueError(f"membrane ranges need chunk_size=1; these layers differ: {not_one}")
    backend = backend or FloatB200Backend()
    n = np.asarray(raw.event_times).shape[0]
    per_batch = []
    for start in range(0, n, batch_size):
        sl = slice(start, start + batch_size)
        from .network import InputEvents
        part = InputEvents(np.asarray(raw.event_times)[sl], np.asarray(raw.source_idx)[sl],
                           np.asarray(raw.n_real_events)[sl])
        out = backend.run_network(layers, weights, network.input_stream(part), v_range=True)
        per_batch.append([(vr[0].max(axis=0), vr[1].min(axis=0)) for vr in out.v_ranges])
    return v_abs_max_per_channel(merge_v_ranges(per_batch))
