"""Layer descriptions: ConvLayer / FCLayer and their specs (salt_core/layers/{conv,fc}.py).

The fields, derived geometry and capacity knobs mirror the reference.  ``forward`` runs the
whole per-layer pipeline (queue construction, integer scan, compaction, diagnostics) on the GPU
through the backend; there is no per-layer JAX structure object.
"""
from __future__ import annotations

import math
from collections.abc import Mapping
from dataclasses import dataclass, field, replace
from typing import Any, ClassVar, NamedTuple

import numpy as np

from .capacity import Capacity, LayerDiag, base_scan_steps, safe_extra_steps


def uniform_init(rng: np.random.Generator, shape, fan_in: int, init_k: float) -> np.ndarray:
    """layers/base.py:18-21 with a numpy generator instead of a JAX key."""
    limit = init_k / math.sqrt(float(fan_in))
    return rng.uniform(-limit, limit, size=shape).astype(np.float32)


class ConvQueueStructure(NamedTuple):
    """A conv layer's materialised queue (salt_core/connectivity/conv.py:46-54), one row per
    output position oy*w_out+ox, shared by every output channel; the input of the dense
    Backend.scan plug-in.  Built by the caller (the reference builds it with XLA)."""
    local_to_global_j: np.ndarray  # (n_spatial, L) int32; empty columns hold n_events
    n_real_events: np.ndarray      # (n_spatial,) int32; may exceed L
    delta_t: np.ndarray            # (n_spatial, L) float32 integer ms
    tap_c: np.ndarray              # (n_spatial, L) int32, clamped kernel coordinates
    tap_ky: np.ndarray
    tap_kx: np.ndarray
    n_input_events: int = 0


class FCQueueStructure(NamedTuple):
    """An FC layer's queue (salt_core/connectivity/fc.py:13-17): every neuron sees the stream."""
    delta_t: np.ndarray            # (E,) float32; pads 0
    source_idx: np.ndarray         # (E,) int
    n_real_events: int


def _jax_take(n: int, idx) -> np.ndarray:
    """Gather indices as XLA resolves them: negative ones wrap once, then clamp into [0, n)."""
    idx = np.asarray(idx, dtype=np.int64)
    return np.clip(np.where(idx < 0, idx + n, idx), 0, n - 1)


class LayerOutput(NamedTuple):
    """layers/base.py:65-70"""
    stream: Any       # EventStream (host) of the layer's output spikes
    result: Any       # QuantLayerResult
    diag: LayerDiag
    trace: Any = None


def _check_leading_axis(values, expected: int, what: str) -> None:
    if np.ndim(values) == 0 or np.shape(values)[0] != expected:
        raise ValueError(f"axis 0 must have length {what}={expected}, got shape "
                         f"{np.shape(values)}")


@dataclass(frozen=True)
class ConvLayer:
    """salt_core/layers/conv.py:23-187.  Output geometry (h_in + 2p - k) // s + 1."""
    name: str
    ic: int
    h_in: int
    w_in: int
    oc: int
    k: int
    s: int
    p: int
    init_k: float
    tau: float = 16.0
    v_th: float = 1.0
    alpha: float = 2.0
    chunk_size: int = 1
    max_queue_len: int = 128
    max_out_spikes: int = 8192
    max_extra_steps: int | None = None

    def __post_init__(self) -> None:
        if self.h_out < 1 or self.w_out < 1:
            raise ValueError(f"{self.name}: degenerate geometry {self.h_in}x{self.w_in}, k={self.k}"
                             f" s={self.s} p={self.p} -> {self.h_out}x{self.w_out}")
        if self.max_extra_steps is None:
            object.__setattr__(self, "max_extra_steps",
                               safe_extra_steps(self.max_queue_len, self.chunk_size))

    @property
    def h_out(self) -> int:
        return (self.h_in + 2 * self.p - self.k) // self.s + 1

    @property
    def w_out(self) -> int:
        return (self.w_in + 2 * self.p - self.k) // self.s + 1

    @property
    def n_neurons(self) -> int:
        return self.oc * self.h_out * self.w_out

    @property
    def input_shape(self) -> tuple[int, ...]:
        return (self.ic, self.h_in, self.w_in)

    @property
    def output_shape(self) -> tuple[int, ...]:
        return (self.oc, self.h_out, self.w_out)

    @property
    def fan_in(self) -> int:
        return self.ic * self.k * self.k

    @property
    def weight_shape(self) -> tuple[int, ...]:
        return (self.oc, self.ic, self.k, self.k)

    @property
    def capacity(self) -> Capacity:
        return Capacity(max_queue_len=self.max_queue_len, max_out_spikes=self.max_out_spikes,
                        max_extra_steps=self.max_extra_steps)

    def with_capacity(self, capacity: Capacity) -> "ConvLayer":
        return replace(self, **capacity)

    def init_weight(self, rng: np.random.Generator) -> np.ndarray:
        return uniform_init(rng, self.weight_shape, self.fan_in, self.init_k)

    def unflatten_neurons(self, values):
        _check_leading_axis(values, self.n_neurons, "n_neurons")
        return values.reshape(self.oc, self.h_out, self.w_out, *values.shape[1:])

    def broadcast_channels(self, values):
        _check_leading_axis(values, self.oc, "oc")
        return values.repeat(self.h_out * self.w_out, axis=0)

    def scan_steps(self, structure=None) -> int:
        return base_scan_steps(self.max_queue_len, self.chunk_size) + self.max_extra_steps

    # ScanLayer accessors of the dense Backend.scan plug-in (salt_core/backend.py:36-61)
    def neuron_delta_t(self, structure) -> np.ndarray:
        """(n_neurons, L): each position's Δt row, repeated for every output channel
        (layers/conv.py:167-169, tile_channels of connectivity/conv.py:221-225)."""
        return np.tile(np.asarray(structure.delta_t), (self.oc, 1))

    def neuron_n_real(self, structure) -> np.ndarray:
        """(n_neurons,): real taps per neuron (layers/conv.py:171-173)."""
        return np.tile(np.asarray(structure.n_real_events), self.oc)

    def gather_weight_codes(self, structure, q) -> np.ndarray:
        """(n_neurons, L) int32: q[oc, tap_c, tap_ky, tap_kx] on real-tap columns, 0 elsewhere
        (layers/conv.py:163-165 -> connectivity/conv.py:175-179, :210-219)."""
        q = np.asarray(q).reshape(self.weight_shape)
        tc, ky, kx = (np.asarray(getattr(structure, f)) for f in ("tap_c", "tap_ky", "tap_kx"))
        n_sp, L = tc.shape
        real = np.arange(L)[None, :] < np.asarray(structure.n_real_events)[:, None]
        codes = q[:, tc, ky, kx]                       # (oc, n_sp, L)
        return np.where(real[None], codes, 0).astype(np.int32).reshape(self.oc * n_sp, L)

    def with_chunk_size(self, chunk_size: int) -> "ConvLayer":
        return replace(self, chunk_size=chunk_size,
                       max_extra_steps=safe_extra_steps(self.max_queue_len, chunk_size))

    def forward(self, params, in_stream, *, backend=None, trace: bool = False) -> LayerOutput:
        """layers/conv.py:124-149 on the B200 backend."""
        from .backend import default_backend
        return (backend or default_backend()).forward_layer(self, params, in_stream, trace=trace)


@dataclass(frozen=True)
class FCLayer:
    """salt_core/layers/fc.py:23-137."""
    name: str
    n_in: int
    n_out: int
    init_k: float
    tau: float = 16.0
    v_th: float = 1.0
    alpha: float = 2.0
    chunk_size: int = 1
    max_out_spikes: int = 8192
    max_extra_steps: int = 0

    @property
    def n_neurons(self) -> int:
        return self.n_out

    @property
    def input_shape(self) -> tuple[int, ...]:
        return (self.n_in,)

    @property
    def output_shape(self) -> tuple[int, ...]:
        return (self.n_out,)

    @property
    def fan_in(self) -> int:
        return self.n_in

    @property
    def weight_shape(self) -> tuple[int, ...]:
        return (self.n_out, self.n_in)

    @property
    def capacity(self) -> Capacity:
        return Capacity(max_out_spikes=self.max_out_spikes, max_extra_steps=self.max_extra_steps)

    def with_capacity(self, capacity: Capacity) -> "FCLayer":
        return replace(self, **capacity)

    def init_weight(self, rng: np.random.Generator) -> np.ndarray:
        return uniform_init(rng, self.weight_shape, self.fan_in, self.init_k)

    def unflatten_neurons(self, values):
        _check_leading_axis(values, self.n_out, "n_out")
        return values.reshape(self.n_out, 1, 1, *values.shape[1:])

    def broadcast_channels(self, values):
        _check_leading_axis(values, self.n_out, "n_out")
        return values

    def scan_steps(self, stream_len: int) -> int:
        return base_scan_steps(stream_len, self.chunk_size) + self.max_extra_steps

    # ScanLayer accessors of the dense Backend.scan plug-in (salt_core/backend.py:36-61)
    def neuron_delta_t(self, structure) -> np.ndarray:
        """(n_out, E): the stream's Δt, the same row for every neuron (layers/fc.py:117-120)."""
        dt = np.asarray(structure.delta_t)
        return np.broadcast_to(dt[None, :], (self.n_out, dt.shape[0]))

    def neuron_n_real(self, structure) -> np.ndarray:
        """(n_out,) (layers/fc.py:122-124)."""
        return np.full(self.n_out, int(structure.n_real_events), np.int32)

    def gather_weight_codes(self, structure, q) -> np.ndarray:
        """(n_out, E) int32: q[:, source] on real events, 0 on pads (layers/fc.py:113-115 ->
        connectivity/fc.py:54-61; sources resolved as XLA's gather does)."""
        q = np.asarray(q).reshape(self.weight_shape)
        src = _jax_take(self.n_in, structure.source_idx)
        real = np.arange(src.shape[0]) < int(structure.n_real_events)
        return np.where(real[None, :], q[:, src], 0).astype(np.int32)

    def with_chunk_size(self, chunk_size: int) -> "FCLayer":
        return replace(self, chunk_size=chunk_size)

    def forward(self, params, in_stream, *, backend=None, trace: bool = False) -> LayerOutput:
        """layers/fc.py:84-101 on the B200 backend."""
        from .backend import default_backend
        return (backend or default_backend()).forward_layer(self, params, in_stream, trace=trace)


@dataclass(frozen=True)
class ConvSpec:
    """layers/conv.py:189-211"""
    oc: int
    k: int
    s: int
    p: int
    name: str | None = None
    options: Mapping[str, Any] = field(default_factory=dict)
    name_prefix: ClassVar[str] = "conv"

    def build(self, input_shape: tuple[int, ...], name: str) -> ConvLayer:
        if len(input_shape) != 3:
            raise ValueError(f"{name}: conv needs a spatial input (C, H, W), got {input_shape}")
        ic, h_in, w_in = input_shape
        return ConvLayer(name=name, ic=ic, h_in=h_in, w_in=w_in, oc=self.oc, k=self.k, s=self.s,
                         p=self.p, **self.options)


def conv(oc: int, k: int, s: int, p: int, *, name: str | None = None, **options) -> ConvSpec:
    """layers/conv.py:214-216"""
    return ConvSpec(oc=oc, k=k, s=s, p=p, name=name, options=options)


@dataclass(frozen=True)
class FCSpec:
    """layers/fc.py:139-153"""
    n_out: int
    name: str | None = None
    options: Mapping[str, Any] = field(default_factory=dict)
    name_prefix: ClassVar[str] = "fc"

    def build(self, input_shape: tuple[int, ...], name: str) -> FCLayer:
        return FCLayer(name=name, n_in=math.prod(input_shape), n_out=self.n_out, **self.options)


def fc(n_out: int, *, name: str | None = None, **options) -> FCSpec:
    """layers/fc.py:156-158"""
    return FCSpec(n_out=n_out, name=name, options=options)


def is_conv(layer) -> bool:
    return isinstance(layer, ConvLayer)
