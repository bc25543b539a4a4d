"""Quantised-layer parameters and the offline integer constants of the SALT integer path.

Mirrors ``salt_core/quant/params.py`` (QuantizedLayerParams), ``salt_core/quant/fixed_point.py``
(RoundMode, OverflowMode, bit-width limits) and ``salt_core/quant/codes.py`` (weight codes,
decay table, integer threshold).  These builders run once on the host, in numpy float32 like the
reference's JAX float32; the per-event integer arithmetic runs only in the CUDA kernels.
"""
from __future__ import annotations

import enum
import math
from typing import NamedTuple

import numpy as np

MAX_SHIFT_BITS = 15      # salt_core/quant/fixed_point.py:15
MAX_REGISTER_BITS = 30   # salt_core/quant/fixed_point.py:17


class RoundMode(str, enum.Enum):
    """salt_core/quant/fixed_point.py:20-23"""
    ROUND = "round"
    TRUNCATE = "truncate"


class OverflowMode(str, enum.Enum):
    """salt_core/quant/fixed_point.py:26-29"""
    WRAP = "wrap"
    SATURATE = "saturate"


class QuantizedLayerParams(NamedTuple):
    """salt_core/quant/params.py:9-21 — one layer's integer parameters."""
    q: np.ndarray                 # integer weight codes, shape = layer.weight_shape
    decay_table_int: np.ndarray   # build_decay_table_int(f_a, layer.tau)
    v_th_int: np.ndarray | None   # scalar or (n_neurons,); None = the layer never fires
    scale: np.ndarray             # scalar or (n_neurons,), only used by readout
    f_a: int
    f_V: int
    i_V: int
    overflow_mode: OverflowMode | str = OverflowMode.WRAP


def check_bit_widths(f_a: int, f_V: int, i_V: int) -> None:
    """The limits of fixed_point.wide_mul_shift (:57-60) and fit_to_bits (:79-82)."""
    if f_a > MAX_SHIFT_BITS:
        raise ValueError(f"shift_bits={f_a} exceeds {MAX_SHIFT_BITS}")
    if i_V + f_V > MAX_REGISTER_BITS:
        raise ValueError(f"total_bits={i_V + f_V} exceeds {MAX_REGISTER_BITS}")
    if f_a < 0 or f_V < 0 or i_V + f_V < 1:
        raise ValueError("bit widths must be non-negative and i_V + f_V >= 1")


def check_weight_codes(q) -> None:
    """salt_core/quant/backend.py:14-20 — q must have an integer dtype."""
    dtype = np.asarray(q).dtype
    if not np.issubdtype(dtype, np.integer):
        raise ValueError(f"q must be integer weight codes, got dtype {dtype}")


def max_weight_code(bits: int) -> int:
    """codes.py:12-14"""
    return 2 ** (bits - 1) - 1


def round_half_away_from_zero(x):
    """codes.py:17-23 (float32 like the reference)."""
    x = np.asarray(x)
    half = x.dtype.type(0.5) if x.dtype.kind == "f" else 0.5
    return np.sign(x) * np.floor(np.abs(x) + half)


def quantize_to_int(x, bits: int, *, axis: int | None = None, threshold=None):
    """codes.py:30-56 — symmetric linear quantisation -> (q int32, scale)."""
    if bits < 2:
        raise ValueError(f"bits must be >= 2, got {bits!r}")
    x = np.asarray(x, dtype=np.float32)
    if threshold is None:
        if axis is None:
            threshold = np.max(np.abs(x))
        else:
            reduce_axes = tuple(i for i in range(x.ndim) if i != axis)
            threshold = np.max(np.abs(x), axis=reduce_axes, keepdims=True)
    threshold = np.asarray(threshold, dtype=x.dtype)
    threshold = np.where(threshold > 0, threshold, np.ones_like(threshold))
    scale = threshold / np.float32(max_weight_code(bits))
    q = round_half_away_from_zero(np.clip(x, -threshold, threshold) / scale).astype(np.int32)
    return q, scale


def delta_t_max(f_a: int, tau: float) -> int:
    """codes.py:63-71 — depth of the decay table."""
    eps = 2.0 ** -(f_a + 1)
    log_base = math.log(1.0 - 1.0 / tau)
    return max(int(math.floor(math.log(eps) / log_base)), 0)


def build_decay_table_int(f_a: int, tau: float) -> np.ndarray:
    """codes.py:74-84 — table[i] = min(round((1-1/tau)^(i+1) * 2^f_a), 2^f_a - 1), int32.

    Computed in float32 like the reference.  The parity contract of this library is defined for a
    given table (the table is an input of the forward pass); a float32 ``pow`` that differs from
    XLA's in the last place could move a code only when a * 2^f_a lies within one ulp of a
    rounding tie.
    """
    n = delta_t_max(f_a, tau)
    delta_t = np.arange(1, n + 1, dtype=np.float32)
    a_exact = np.float32(1.0 - 1.0 / tau) ** delta_t
    code = round_half_away_from_zero(a_exact * np.float32(2 ** f_a))
    return np.minimum(code, 2 ** f_a - 1).astype(np.int32)


def apply_decay_table_int(delta_t, table_int):
    """codes.py:87-105 on the host (used by the dense Backend.scan plug-in only)."""
    delta_t = np.asarray(delta_t)
    if not np.all(delta_t == np.floor(delta_t)):
        raise ValueError("delta_t must hold integer milliseconds")
    if np.any((delta_t < 0) | (delta_t >= 2.0 ** 31)):
        raise ValueError("delta_t must lie in [0, 2^31)")
    d = delta_t.astype(np.int32)
    table = np.asarray(table_int, dtype=np.int32)
    n = table.shape[0]
    if n == 0:
        gathered = np.zeros_like(d)
    else:
        gathered = table[np.clip(d - 1, 0, n - 1)]
    return np.where(d > n, 0, gathered).astype(np.int32), d == 0


def v_th_to_int(v_th, s_c, f_V: int, i_V: int) -> np.ndarray:
    """codes.py:119-136 — physical threshold -> integer register threshold."""
    v = np.asarray(v_th, dtype=np.float32) / np.asarray(s_c, dtype=np.float32)
    code = round_half_away_from_zero(v * np.float32(2 ** f_V))
    half = 2 ** (i_V + f_V - 1)
    bad = (code < -half) | (code > half - 1)
    if np.any(bad):
        raise ValueError(f"integer threshold outside the i_V={i_V}, f_V={f_V} register range "
                         f"[{-half}, {half - 1}]; use v_th_int=None for a non-firing layer")
    return code.astype(np.int32)


def iv_from_measurement(M: float, T_c: float, b: int) -> int:
    """codes.py:143-154"""
    if M <= 0:
        raise ValueError(f"M must be > 0, got {M!r}")
    return math.floor(math.log2(M * max_weight_code(b) / T_c)) + 2


def weight_bits(q) -> int:
    """8 / 16 / 32: narrowest signed width holding every weight code."""
    q = np.asarray(q)
    if q.size == 0:
        return 8
    lo, hi = int(q.min()), int(q.max())
    if lo >= -128 and hi <= 127:
        return 8
    if lo >= -32768 and hi <= 32767:
        return 16
    return 32
