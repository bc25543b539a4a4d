"""Network container and run_network (salt_core/network.py), on the B200 backend."""
from __future__ import annotations

import math
from collections import Counter
from collections.abc import Sequence
from dataclasses import dataclass, replace
from typing import NamedTuple

import numpy as np

from .layers import ConvLayer, FCLayer
from .stream import EventStream

_MAX_EVENT_TIME = 2 ** 31  # network.py:23


class InputEvents(NamedTuple):
    """network.py:26-54.  Single sample: (E,) arrays and a scalar; batched: (B, E), (B,)."""
    event_times: np.ndarray
    source_idx: np.ndarray
    n_real_events: np.ndarray

    @staticmethod
    def checked(event_times, source_idx, n_real_events) -> "InputEvents":
        """Host check of the real events' times (network.py:33-54): integer ms in
        [0, 2^31), non-decreasing.  Raises ValueError otherwise."""
        times = np.asarray(event_times)
        n_real = np.asarray(n_real_events)
        is_real = np.arange(times.shape[-1]) < n_real[..., None]
        real_times = times[is_real]
        if not np.all(real_times == np.floor(real_times)):
            raise ValueError("event times must be integer milliseconds")
        if real_times.size and (np.any(real_times < 0) or np.any(real_times >= _MAX_EVENT_TIME)):
            raise ValueError(f"event times must lie in [0, 2^31), got [{real_times.min()}, "
                             f"{real_times.max()}]")
        both_real = is_real[..., 1:]
        if np.any(np.diff(times, axis=-1)[both_real] < 0):
            raise ValueError("real event times must be non-decreasing")
        return InputEvents(event_times, source_idx, n_real_events)


def _check_connected(out_shape, in_shape, out_name, in_name) -> None:
    """network.py:70-84"""
    out_shape, in_shape = tuple(out_shape), tuple(in_shape)
    connected = (math.prod(out_shape) == in_shape[0]) if len(in_shape) == 1 else out_shape == in_shape
    if connected:
        return
    if len(out_shape) < len(in_shape):
        raise ValueError(f"{out_name} output {out_shape} has no spatial shape; {in_name} needs "
                         f"{in_shape}")
    raise ValueError(f"{out_name} output {out_shape} does not connect to {in_name} input {in_shape}")


def check_layer_connections(layers: Sequence) -> None:
    """network.py:87-90"""
    for prev, nxt in zip(layers, layers[1:]):
        _check_connected(prev.output_shape, nxt.input_shape, prev.name, nxt.name)


def input_stream(raw: InputEvents) -> EventStream:
    """network.py:165-171: source_idx as int32, event_gain all ones."""
    t = np.asarray(raw.event_times, dtype=np.float32)
    return EventStream(t, np.asarray(raw.source_idx, dtype=np.int32), np.ones_like(t),
                       np.asarray(raw.n_real_events, dtype=np.int32))


def run_network(layers: Sequence, weights: Sequence, input_stream: EventStream, *, backend=None,
                trace: bool = False, keep_streams: bool = False):
    """network.py:93-122 — chain the layers; fits = AND of every layer's Capacity.fits."""
    from .backend import default_backend
    check_layer_connections(layers)
    return (backend or default_backend()).run_network(layers, weights, input_stream, trace=trace,
                                                      keep_streams=keep_streams)


@dataclass(frozen=True)
class Network:
    """network.py:125-187"""
    input_shape: tuple[int, ...]
    layers: tuple

    def __post_init__(self) -> None:
        object.__setattr__(self, "input_shape", tuple(int(v) for v in self.input_shape))
        object.__setattr__(self, "layers", tuple(self.layers))
        if not self.layers:
            raise ValueError("layers must not be empty")
        _check_connected(self.input_shape, self.layers[0].input_shape, "input",
                         self.layers[0].name)
        check_layer_connections(self.layers)

    @classmethod
    def build(cls, input_shape: Sequence[int], specs: Sequence) -> "Network":
        shape = tuple(int(v) for v in input_shape)
        counts: Counter = Counter()
        layers = []
        for spec in specs:
            counts[spec.name_prefix] += 1
            layer = spec.build(shape, spec.name or f"{spec.name_prefix}{counts[spec.name_prefix]}")
            layers.append(layer)
            shape = layer.output_shape
        return cls(input_shape=input_shape, layers=layers)

    def init(self, seed: int = 0) -> tuple:
        rng = np.random.default_rng(seed)
        return tuple(layer.init_weight(rng) for layer in self.layers)

    def input_stream(self, raw: InputEvents) -> EventStream:
        return input_stream(raw)

    def apply(self, weights, raw: InputEvents, *, backend=None, trace: bool = False,
              keep_streams: bool = False):
        return run_network(self.layers, weights, self.input_stream(raw), backend=backend,
                           trace=trace, keep_streams=keep_streams)

    def apply_batched(self, weights, raw_batch: InputEvents, *, backend=None, trace: bool = False,
                      keep_streams: bool = False):
        """Batched forward (the reference vmaps apply over axis 0, network.py:179-183)."""
        if np.ndim(raw_batch.event_times) != 2:
            raise ValueError("apply_batched expects (B, E) event arrays")
        return run_network(self.layers, weights, self.input_stream(raw_batch), backend=backend,
                           trace=trace, keep_streams=keep_streams)

    def replace_layers(self, layers) -> "Network":
        return replace(self, layers=tuple(layers))
