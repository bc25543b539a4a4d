"""Capacity knobs and per-layer diagnostics (salt_core/capacity.py)."""
from __future__ import annotations

import math
from collections.abc import Iterator, Mapping
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np


class LayerDiag(NamedTuple):
    """salt_core/capacity.py:13-22.  Batched: every value has a leading batch axis."""
    spike_count: np.ndarray
    firing_rate: np.ndarray
    needed: dict


def reduce_over_batch(diag: LayerDiag) -> LayerDiag:
    """capacity.py:25-32"""
    return LayerDiag(spike_count=np.mean(diag.spike_count), firing_rate=np.mean(diag.firing_rate),
                     needed={k: np.max(v) for k, v in diag.needed.items()})


class Capacity(Mapping):
    """capacity.py:35-63 — knob name -> capacity, immutable."""

    def __init__(self, **knobs: int):
        self._knobs = {k: int(v) for k, v in knobs.items()}

    def __getitem__(self, knob: str) -> int:
        return self._knobs[knob]

    def __iter__(self) -> Iterator[str]:
        return iter(self._knobs)

    def __len__(self) -> int:
        return len(self._knobs)

    def __repr__(self) -> str:
        return f"Capacity({', '.join(f'{k}={v}' for k, v in self._knobs.items())})"

    def replace(self, **knobs: int) -> "Capacity":
        unknown = set(knobs) - set(self._knobs)
        if unknown:
            raise KeyError(f"unknown knobs {sorted(unknown)}, have {list(self._knobs)}")
        return Capacity(**{**self._knobs, **knobs})

    def fits(self, diag: LayerDiag) -> np.ndarray:
        """Every knob holds diag.needed; per sample when diag is batched (capacity.py:60-63)."""
        return np.all(np.stack([np.asarray(diag.needed[k]) <= v for k, v in self._knobs.items()]),
                      axis=0)


def _grow(observed: int, factor: float) -> int:
    return int(math.ceil(int(observed) * factor))


def base_scan_steps(queue_len: int, chunk_size: int) -> int:
    """salt_core/float/affine.py:73-75"""
    return -(-queue_len // chunk_size)


def safe_extra_steps(queue_len: int, chunk_size: int) -> int:
    """salt_core/float/affine.py:78-80"""
    return queue_len - base_scan_steps(queue_len, chunk_size)


@dataclass(frozen=True)
class GrowthPolicy:
    """capacity.py:71-124 — growth/shrink of a layer's capacities (host-side policy)."""
    max_queue_len_grow_factor: float = 1.5
    out_grow_factor: float = 1.5
    max_extra_steps_grow_factor: float = 1.5
    out_shrink_threshold: float = 0.5
    max_extra_steps_shrink_threshold: float = 0.5

    def _grow_factor(self, knob: str) -> float:
        return {"max_queue_len": self.max_queue_len_grow_factor,
                "max_out_spikes": self.out_grow_factor,
                "max_extra_steps": self.max_extra_steps_grow_factor}[knob]

    def grown(self, capacity: Capacity, needed: Mapping, chunk_size: int) -> Capacity:
        new = {k: _grow(needed[k], self._grow_factor(k)) if int(needed[k]) > v else v
               for k, v in capacity.items()}
        if ("max_queue_len" in new and "max_extra_steps" in new
                and new["max_queue_len"] != capacity["max_queue_len"]):
            new["max_extra_steps"] = safe_extra_steps(new["max_queue_len"], chunk_size)
        return Capacity(**new)


def grown_to_fit(layers, policies: Mapping, diags) -> list:
    """capacity.py:153-164 — layers whose needs exceed their capacity, grown; diags reduced."""
    out = []
    for layer, diag in zip(layers, diags):
        cap = layer.capacity
        if cap is None:
            out.append(layer)
            continue
        new = policies[layer.name].grown(cap, diag.needed, layer.chunk_size)
        out.append(layer if new == cap else layer.with_capacity(new))
    return out
