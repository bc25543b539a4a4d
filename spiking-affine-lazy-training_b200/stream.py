"""Inter-layer event streams (salt_core/stream.py:16-21) and their device-resident form."""
from __future__ import annotations

from typing import NamedTuple

import numpy as np

PAD_TIME = np.float32(1e12)  # salt_core/stream.py:13 _PAD_TIME


class EventStream(NamedTuple):
    """salt_core/stream.py:16-21.  The first n_real_events entries are real, the rest pads.

    Single sample: arrays (E,) and a scalar n_real_events; batched: (B, E) and (B,).
    """
    event_times: np.ndarray       # float32 integer ms, non-decreasing; pads are 1e12
    event_source_idx: np.ndarray  # int32 flat index of the emitting neuron
    event_gain: np.ndarray        # float32; identically 1 on the integer path
    n_real_events: np.ndarray     # int32, may exceed the stream length (truncation)


def sample(stream: EventStream, i: int) -> EventStream:
    """Sample i of a batched stream."""
    return EventStream(stream.event_times[i], stream.event_source_idx[i], stream.event_gain[i],
                       np.int32(stream.n_real_events[i]))
