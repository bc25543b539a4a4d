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
    """salt_core/layers/conv.py:107-186.  Output geometry (h_in + 2p - k) // s + 1."""
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

    def with_chunk_size(self, chunk_size: int) -> "ConvLayer":
        return replace(self, chunk_size=chunk_size,
                       max_extra_steps=safe_extra_steps(self.max_queue_len, chunk_size))

    def forward(self, params, in_stream, *, backend=None, trace: bool = False) -> LayerOutput:
        """layers/conv.py:209-234 on the B200 backend."""
        from .backend import default_backend
        return (backend or default_backend()).forward_layer(self, params, in_stream, trace=trace)


@dataclass(frozen=True)
class FCLayer:
    """salt_core/layers/fc.py:323-437."""
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

    def with_chunk_size(self, chunk_size: int) -> "FCLayer":
        return replace(self, chunk_size=chunk_size)

    def forward(self, params, in_stream, *, backend=None, trace: bool = False) -> LayerOutput:
        """layers/fc.py:385-402 on the B200 backend."""
        from .backend import default_backend
        return (backend or default_backend()).forward_layer(self, params, in_stream, trace=trace)


@dataclass(frozen=True)
class ConvSpec:
    """layers/conv.py:274-296"""
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
    """layers/conv.py:299-301"""
    return ConvSpec(oc=oc, k=k, s=s, p=p, name=name, options=options)


@dataclass(frozen=True)
class FCSpec:
    """layers/fc.py:440-454"""
    n_out: int
    name: str | None = None
    options: Mapping[str, Any] = field(default_factory=dict)
    name_prefix: ClassVar[str] = "fc"

    def build(self, input_shape: tuple[int, ...], name: str) -> FCLayer:
        return FCLayer(name=name, n_in=math.prod(input_shape), n_out=self.n_out, **self.options)


def fc(n_out: int, *, name: str | None = None, **options) -> FCSpec:
    """layers/fc.py:457-459"""
    return FCSpec(n_out=n_out, name=name, options=options)


def is_conv(layer) -> bool:
    return isinstance(layer, ConvLayer)
