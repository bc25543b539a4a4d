"""Per-step trajectories of a forward (salt_core/trace.py:13-81).

``forward_layer(..., trace=True)`` and ``run_network(..., trace=True)`` on the B200 integer
backend fill ``LayerOutput.trace`` with a LayerForwardTrace computed by the trace kernels
(``salt_conv_layer_trace`` / ``salt_fc_layer_trace``); the fused forward itself never builds
these (n, L) arrays.
"""
from __future__ import annotations

from typing import NamedTuple, TypedDict

import numpy as np


class LayerForwardTrace(NamedTuple):
    """trace.py:13-22: (n, L) per neuron and queue column (leading batch axis when batched).

    spike_mask: the forward's spike mask.  v_steps: the register after each column (after the
    reset); the last column equals v_final.  event_ms: the time of each column's event, NaN for
    idle columns (at or past the neuron's real events)."""
    spike_mask: np.ndarray
    v_steps: np.ndarray
    event_ms: np.ndarray


class TraceSummary(TypedDict):
    """trace.py:58-66"""
    n: int
    steps: int
    total_spikes: int
    fired: np.ndarray
    idle_frac: float
    v_range: tuple[float, float]
    nonfinite_v: int


def summarize_trace_scalars(trace: LayerForwardTrace) -> TraceSummary:
    """trace.py:69-81: one sample's one layer as scalars."""
    sm = np.asarray(trace.spike_mask)
    vs = np.asarray(trace.v_steps)
    ms = np.asarray(trace.event_ms)
    n, steps = sm.shape
    return {"n": n, "steps": steps, "total_spikes": int(sm.sum()),
            "fired": np.where(sm.sum(axis=1) > 0)[0], "idle_frac": float(np.isnan(ms).mean()),
            "v_range": (float(np.nanmin(vs)), float(np.nanmax(vs))),
            "nonfinite_v": int(np.sum(~np.isfinite(vs)))}
