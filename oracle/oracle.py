"""CPU oracle for the SALT integer forward and float FC scan — TEST INFRASTRUCTURE ONLY.

ctypes wrapper around ``oracle/libsalt_oracle.so`` (a literal C restatement of the reference's
JAX integer path, see ``salt_oracle.c``).  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import this module; the product path never does.

Parity status: pinned against the reference's own known-answer tests
(``tests/golden/known_answers.json``, transcribed from ``salt_core/tests/test_*.py``).  The
reference itself cannot run in this image (it needs JAX), so no reference-generated outputs
exist; independent restatements (a dense per-neuron conv scan, a float64 event-by-event float
scan) cross-check the oracle in ``tests/``.

The functions take duck-typed layer/params objects whose attribute names follow the reference
(``ConvLayer`` fields ic, h_in, w_in, oc, k, s, p, max_queue_len, max_out_spikes,
max_extra_steps; ``FCLayer`` fields n_in, n_out, max_out_spikes, max_extra_steps;
``QuantizedLayerParams`` fields q, decay_table_int, v_th_int, f_a, f_V, i_V, overflow_mode).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import NamedTuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libsalt_oracle.so")
PAD_TIME = np.float32(1e12)

_i32p = ctypes.POINTER(ctypes.c_int32)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)


class _QP(ctypes.Structure):
    _fields_ = [("q", _i32p), ("lut", _i32p), ("lut_len", ctypes.c_int32), ("vth", _i32p),
                ("f_a", ctypes.c_int32), ("f_V", ctypes.c_int32), ("i_V", ctypes.c_int32),
                ("round_mode", ctypes.c_int32), ("overflow_mode", ctypes.c_int32)]


class _ConvGeom(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("ic", "h_in", "w_in", "oc", "k", "s", "p", "max_queue_len", "max_out_spikes",
                 "max_extra_steps")]


class _FCGeom(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("n_in", "n_out", "max_out_spikes",
                                                "max_extra_steps")]


class _LayerOut(ctypes.Structure):
    _fields_ = [("v_final", _i32p), ("vmin", _i32p), ("vmax", _i32p), ("spike_mask", _u8p),
                ("overflowed", _u8p), ("out_times", _f32p), ("out_src", _i32p),
                ("n_real_out", ctypes.c_int32), ("spike_count", ctypes.c_int32),
                ("needed_queue", ctypes.c_int32), ("any_overflow", ctypes.c_int32),
                ("vmin_all", ctypes.c_int32), ("vmax_all", ctypes.c_int32),
                ("fits", ctypes.c_int32), ("v_steps", _i32p), ("event_ms", _f32p)]


class _LayerSpec(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("conv", _ConvGeom), ("fc", _FCGeom), ("qp", _QP)]


_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc); returns the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.so_round_shift.restype = ctypes.c_int32
        _lib.so_wide_mul_shift.restype = ctypes.c_int32
        _lib.so_fit_to_bits.restype = ctypes.c_int32
        _lib.so_process_event.restype = ctypes.c_int32
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def _mode_round(m) -> int:
    m = getattr(m, "value", m)
    if m not in ("round", "truncate"):
        raise ValueError(f"bad round_mode {m!r}")
    return 0 if m == "round" else 1


def _mode_overflow(m) -> int:
    m = getattr(m, "value", m)
    if m not in ("wrap", "saturate"):
        raise ValueError(f"bad overflow_mode {m!r}")
    return 0 if m == "wrap" else 1


# ---------------------------------------------------------------- fixed point (scalars)

def round_shift(x: int, shift_bits: int, round_mode="round") -> int:
    """salt_core/quant/fixed_point.py:32-44"""
    return int(lib().so_round_shift(ctypes.c_int32(x), shift_bits, _mode_round(round_mode)))


def wide_mul_shift(a: int, v: int, shift_bits: int, round_mode="round") -> int:
    """salt_core/quant/fixed_point.py:47-65"""
    return int(lib().so_wide_mul_shift(ctypes.c_int32(a), ctypes.c_int32(v), shift_bits,
                                       _mode_round(round_mode)))


def fit_to_bits(x: int, total_bits: int, overflow_mode="wrap") -> tuple[int, bool]:
    """salt_core/quant/fixed_point.py:68-90"""
    ovf = ctypes.c_int32(0)
    r = lib().so_fit_to_bits(ctypes.c_int32(x), total_bits, _mode_overflow(overflow_mode),
                             ctypes.byref(ovf))
    return int(r), bool(ovf.value)


class EventResult(NamedTuple):
    v_final: int
    is_spiked: bool
    overflowed: bool
    v_unfitted: int


def process_event(v0_int, a_int, is_identity, q_int, v_th_int, *, f_a, f_V, i_V,
                  round_mode="round", overflow_mode="wrap") -> EventResult:
    """salt_core/quant/scan.py:22-52"""
    spk, ovf, u = ctypes.c_int32(0), ctypes.c_int32(0), ctypes.c_int32(0)
    v = lib().so_process_event(ctypes.c_int32(int(v0_int)), ctypes.c_int32(int(a_int)),
                               int(bool(is_identity)), ctypes.c_int32(int(q_int)),
                               int(v_th_int is not None),
                               ctypes.c_int32(0 if v_th_int is None else int(v_th_int)),
                               f_a, f_V, i_V, _mode_round(round_mode),
                               _mode_overflow(overflow_mode), ctypes.byref(spk),
                               ctypes.byref(ovf), ctypes.byref(u))
    return EventResult(int(v), bool(spk.value), bool(ovf.value), int(u.value))


def apply_decay_table_int(delta_t, table_int):
    """salt_core/quant/codes.py:87-105 -> (a_int, is_identity)."""
    dt = np.ascontiguousarray(np.asarray(delta_t, dtype=np.float32))
    lut = np.ascontiguousarray(np.asarray(table_int, dtype=np.int32))
    a = np.empty(dt.shape, np.int32)
    ident = np.empty(dt.shape, np.uint8)
    lib().so_apply_decay_table(_p(dt, _f32p), ctypes.c_int64(dt.size), _p(lut, _i32p),
                               lut.size, _p(a, _i32p), _p(ident, _u8p))
    return a, ident.astype(bool)


class LayerScan(NamedTuple):
    spike_mask: np.ndarray
    overflowed: np.ndarray
    v_final: np.ndarray
    v_unfitted_min: np.ndarray
    v_unfitted_max: np.ndarray


def run_layer(a_int, is_identity, q_int, v_th_int, *, f_a, f_V, i_V, round_mode="round",
              overflow_mode="wrap") -> LayerScan:
    """salt_core/quant/scan.py:65-80 (+ :97-132) on (n, L) inputs."""
    a = np.ascontiguousarray(a_int, dtype=np.int32)
    n, L = a.shape
    ident = np.ascontiguousarray(is_identity, dtype=np.uint8)
    q = np.ascontiguousarray(q_int, dtype=np.int32)
    vth = None if v_th_int is None else np.ascontiguousarray(
        np.broadcast_to(np.asarray(v_th_int, dtype=np.int32), (n,)))
    mask = np.empty((n, L), np.uint8)
    ovf = np.empty((n, L), np.uint8)
    vf, lo, hi = (np.empty(n, np.int32) for _ in range(3))
    lib().so_run_layer(_p(a, _i32p), _p(ident, _u8p), _p(q, _i32p),
                       None if vth is None else _p(vth, _i32p), n, L, f_a, f_V, i_V,
                       _mode_round(round_mode), _mode_overflow(overflow_mode), _p(mask, _u8p),
                       _p(ovf, _u8p), _p(vf, _i32p), _p(lo, _i32p), _p(hi, _i32p))
    return LayerScan(mask.astype(bool), ovf.astype(bool), vf, lo, hi)


# ---------------------------------------------------------------- layers

def _qp(params, round_mode, keep):
    q = np.ascontiguousarray(np.asarray(params.q), dtype=np.int32)
    if not np.issubdtype(np.asarray(params.q).dtype, np.integer):
        raise ValueError("q must be integer weight codes")
    lut = np.ascontiguousarray(np.asarray(params.decay_table_int), dtype=np.int32)
    keep += [q, lut]
    qp = _QP()
    qp.q = _p(q, _i32p)
    qp.lut = _p(lut, _i32p)
    qp.lut_len = lut.size
    qp.f_a, qp.f_V, qp.i_V = int(params.f_a), int(params.f_V), int(params.i_V)
    qp.round_mode = _mode_round(round_mode)
    qp.overflow_mode = _mode_overflow(getattr(params, "overflow_mode", "wrap"))
    return qp, q


def _vth(params, n, keep):
    if params.v_th_int is None:
        return None
    v = np.ascontiguousarray(np.broadcast_to(np.asarray(params.v_th_int, dtype=np.int32), (n,)))
    keep.append(v)
    return _p(v, _i32p)


def conv_out_hw(layer) -> tuple[int, int]:
    return ((layer.h_in + 2 * layer.p - layer.k) // layer.s + 1,
            (layer.w_in + 2 * layer.p - layer.k) // layer.s + 1)


def _conv_geom(layer):
    g = _ConvGeom()
    for f in ("ic", "h_in", "w_in", "oc", "k", "s", "p", "max_queue_len", "max_out_spikes",
              "max_extra_steps"):
        setattr(g, f, int(getattr(layer, f)))
    return g


def _fc_geom(layer):
    g = _FCGeom()
    for f in ("n_in", "n_out", "max_out_spikes", "max_extra_steps"):
        setattr(g, f, int(getattr(layer, f)))
    return g


class LayerResult(NamedTuple):
    """One layer for one sample, with the reference's field names where they exist."""
    v_final: np.ndarray          # (n,) int32
    v_unfitted_min: np.ndarray   # (n,)
    v_unfitted_max: np.ndarray   # (n,)
    spike_mask: np.ndarray       # (n, L) bool
    overflowed: np.ndarray       # (n, L) bool
    event_times: np.ndarray      # (max_out,) float32 output stream
    event_source_idx: np.ndarray  # (max_out,) int32
    n_real_events: int           # spikes, not clipped
    spike_count: int             # LayerDiag.spike_count (== n_real_events)
    needed_queue: int            # conv only
    any_overflow: bool
    vmin_all: int
    vmax_all: int
    fits: bool
    v_steps: np.ndarray | None = None   # (n, L) register after each column (trace=True)
    event_ms: np.ndarray | None = None  # (n, L) time of each column's event, NaN when idle


def _run(layer, params, times, src, n_in, round_mode, kind, trace=False):
    keep = []
    t = np.ascontiguousarray(np.asarray(times, dtype=np.float32))
    s = np.ascontiguousarray(np.asarray(src), dtype=np.int32)
    E = t.shape[0]
    if kind == "conv":
        h_out, w_out = conv_out_hw(layer)
        n = layer.oc * h_out * w_out
        L = layer.max_queue_len
    else:
        n = layer.n_out
        L = E
    M = layer.max_out_spikes
    qp, _ = _qp(params, round_mode, keep)
    qp.vth = _vth(params, n, keep)
    vf, lo, hi = (np.empty(n, np.int32) for _ in range(3))
    mask = np.empty((n, L), np.uint8)
    ovf = np.empty((n, L), np.uint8)
    ot = np.empty(max(M, 1), np.float32)
    osrc = np.empty(max(M, 1), np.int32)
    o = _LayerOut()
    o.v_final, o.vmin, o.vmax = _p(vf, _i32p), _p(lo, _i32p), _p(hi, _i32p)
    o.spike_mask, o.overflowed = _p(mask, _u8p), _p(ovf, _u8p)
    o.out_times, o.out_src = _p(ot, _f32p), _p(osrc, _i32p)
    vs = np.empty((n, L), np.int32) if trace else None
    ems = np.empty((n, L), np.float32) if trace else None
    if trace:
        o.v_steps, o.event_ms = _p(vs, _i32p), _p(ems, _f32p)
    if kind == "conv":
        g = _conv_geom(layer)
        rc = lib().so_conv_forward(ctypes.byref(g), ctypes.byref(qp), _p(t, _f32p), _p(s, _i32p),
                                   E, int(n_in), ctypes.byref(o))
    else:
        g = _fc_geom(layer)
        rc = lib().so_fc_forward(ctypes.byref(g), ctypes.byref(qp), _p(t, _f32p), _p(s, _i32p),
                                 E, int(n_in), ctypes.byref(o))
    if rc:
        raise ValueError(f"oracle layer failed rc={rc}")
    return LayerResult(vf, lo, hi, mask.astype(bool), ovf.astype(bool), ot[:M], osrc[:M],
                       int(o.n_real_out), int(o.spike_count), int(o.needed_queue),
                       bool(o.any_overflow),
                       int(o.vmin_all), int(o.vmax_all), bool(o.fits), vs, ems)


def conv_forward(layer, params, times, src, n_in, round_mode="round", trace=False
                 ) -> LayerResult:
    """salt_core/layers/conv.py:124-149 with salt_core/quant/backend.py:31-53."""
    return _run(layer, params, times, src, n_in, round_mode, "conv", trace)


def fc_forward(layer, params, times, src, n_in, round_mode="round", trace=False) -> LayerResult:
    """salt_core/layers/fc.py:84-101 with salt_core/quant/backend.py:31-53."""
    return _run(layer, params, times, src, n_in, round_mode, "fc", trace)


def is_conv(layer) -> bool:
    return hasattr(layer, "max_queue_len") and hasattr(layer, "oc")


def network_forward(layers, params, times, src, n_real, round_mode="round") -> list[LayerResult]:
    """salt_core/network.py:93-122 run_network for ONE sample; returns every layer's result."""
    out = []
    t, s, nin = np.asarray(times, np.float32), np.asarray(src, np.int32), int(n_real)
    for layer, p in zip(layers, params):
        r = (conv_forward if is_conv(layer) else fc_forward)(layer, p, t, s, nin, round_mode)
        out.append(r)
        t, s, nin = r.event_times, r.event_source_idx, r.n_real_events
    return out


def compress_candidates(n_flat, j_flat, n_out_spatial, max_queue_len, n_events):
    """salt_core/connectivity/conv.py:57-99 -> (local_to_global_j, n_real_per_neuron)."""
    nf = np.ascontiguousarray(n_flat, dtype=np.int32)
    jf = np.ascontiguousarray(j_flat, dtype=np.int32)
    l2g = np.empty((n_out_spatial, max_queue_len), np.int32)
    nr = np.empty(n_out_spatial, np.int32)
    rc = lib().so_compress_candidates(_p(nf, _i32p), _p(jf, _i32p), ctypes.c_int64(nf.size),
                                      n_out_spatial, max_queue_len, n_events, _p(l2g, _i32p),
                                      _p(nr, _i32p))
    if rc:
        raise ValueError(f"compress failed rc={rc}")
    return l2g, nr


def delta_t_three_regimes(t_gathered, n_real_per_neuron, global_last_time):
    """salt_core/connectivity/conv.py:102-125"""
    tg = np.ascontiguousarray(t_gathered, dtype=np.float32)
    nr = np.ascontiguousarray(n_real_per_neuron, dtype=np.int32)
    n, L = tg.shape
    dt = np.empty((n, L), np.float32)
    lib().so_delta_t_regimes(_p(tg, _f32p), _p(nr, _i32p), ctypes.c_float(global_last_time), n, L,
                             _p(dt, _f32p))
    return dt


def extract_output_events(spike_mask, spike_event_idx, event_times, max_total_spikes,
                          local_to_global_j=None):
    """salt_core/stream.py:67-100 (fc when local_to_global_j is None, else conv with the
    tiled (rows, L) table) -> (times, source_idx, n_real_events)."""
    m = np.ascontiguousarray(spike_mask, dtype=np.uint8)
    n, steps = m.shape
    ei = None if spike_event_idx is None else np.ascontiguousarray(spike_event_idx, np.int32)
    t = np.ascontiguousarray(event_times, dtype=np.float32)
    l2g = None if local_to_global_j is None else np.ascontiguousarray(local_to_global_j, np.int32)
    M = int(max_total_spikes)
    ot = np.empty(max(M, 1), np.float32)
    osrc = np.empty(max(M, 1), np.int32)
    nr = ctypes.c_int32(0)
    lib().so_extract_output_events(
        _p(m, _u8p), None if ei is None else _p(ei, _i32p), n, steps,
        None if l2g is None else _p(l2g, _i32p), 1 if l2g is None else l2g.shape[0],
        1 if l2g is None else l2g.shape[1], _p(t, _f32p), t.shape[0], M, _p(ot, _f32p),
        _p(osrc, _i32p), ctypes.byref(nr))
    return ot[:M], osrc[:M], int(nr.value)


def conv_structure(layer, times, src, n_in):
    """salt_core/connectivity/conv.py:128-172 -> dict of the ConvQueueStructure arrays."""
    t = np.ascontiguousarray(np.asarray(times, dtype=np.float32))
    s = np.ascontiguousarray(np.asarray(src), dtype=np.int32)
    h_out, w_out = conv_out_hw(layer)
    n_sp, L = h_out * w_out, layer.max_queue_len
    l2g = np.empty((n_sp, L), np.int32)
    nr = np.empty(n_sp, np.int32)
    dt = np.empty((n_sp, L), np.float32)
    tc, tky, tkx = (np.empty((n_sp, L), np.int32) for _ in range(3))
    g = _conv_geom(layer)
    rc = lib().so_conv_structure(ctypes.byref(g), _p(t, _f32p), _p(s, _i32p), t.shape[0],
                                 int(n_in), _p(l2g, _i32p), _p(nr, _i32p), _p(dt, _f32p),
                                 _p(tc, _i32p), _p(tky, _i32p), _p(tkx, _i32p))
    if rc:
        raise ValueError(f"oracle structure failed rc={rc}")
    return dict(local_to_global_j=l2g, n_real_events=nr, delta_t=dt, tap_c=tc, tap_ky=tky,
                tap_kx=tkx)


def network_batch(layers, params, times, src, n_real, round_mode="round", threads=None):
    """Threaded batch forward (CPU baseline): returns (v_final_last (B, n_out), spike_counts
    (B, n_layers), fits (B,))."""
    keep = []
    t = np.ascontiguousarray(np.asarray(times, dtype=np.float32))
    s = np.ascontiguousarray(np.asarray(src), dtype=np.int32)
    nr = np.ascontiguousarray(np.asarray(n_real), dtype=np.int32)
    B, E = t.shape
    specs = (_LayerSpec * len(layers))()
    for i, (layer, p) in enumerate(zip(layers, params)):
        qp, _ = _qp(p, round_mode, keep)
        if is_conv(layer):
            specs[i].kind = 0
            specs[i].conv = _conv_geom(layer)
            h, w = conv_out_hw(layer)
            n = layer.oc * h * w
        else:
            specs[i].kind = 1
            specs[i].fc = _fc_geom(layer)
            n = layer.n_out
        qp.vth = _vth(p, n, keep)
        specs[i].qp = qp
    last = layers[-1]
    n_last = last.n_out if not is_conv(last) else last.oc * np.prod(conv_out_hw(last))
    vf = np.empty((B, int(n_last)), np.int32)
    sc = np.empty((B, len(layers)), np.int32)
    fits = np.empty(B, np.int32)
    threads = threads or os.cpu_count() or 1
    rc = lib().so_network_batch(specs, len(layers), _p(t, _f32p), _p(s, _i32p), _p(nr, _i32p),
                                B, E, int(threads), _p(vf, _i32p), _p(sc, _i32p),
                                _p(fits, _i32p))
    if rc:
        raise ValueError(f"oracle batch failed rc={rc}")
    return vf, sc, fits.astype(bool)


# ---------------------------------------------------------------- float chunked scan

class _FloatGeom(ctypes.Structure):
    _fields_ = [("n_in", ctypes.c_int32), ("n_out", ctypes.c_int32),
                ("chunk_size", ctypes.c_int32), ("max_out_spikes", ctypes.c_int32),
                ("max_extra_steps", ctypes.c_int32), ("v_th", ctypes.c_float)]


class _FloatOut(ctypes.Structure):
    _fields_ = [("v_final", _f32p), ("spike_mask", _u8p), ("spike_event_idx", _i32p),
                ("out_times", _f32p), ("out_src", _i32p), ("out_gain", _f32p),
                ("n_real_out", ctypes.c_int32), ("extra_steps_needed", ctypes.c_int32),
                ("fits", ctypes.c_int32), ("v_steps", _f32p), ("event_ms", _f32p)]


class FloatResult(NamedTuple):
    """FCLayer.forward with FloatBackend (layers/fc.py:84-106): FloatLayerResult's forward
    values (float/scan.py:15-22; s_spike and s_value equal spike_mask there), the output
    EventStream (stream.py:16-21) and the layer's needs (LayerDiag.needed)."""
    v_final: np.ndarray           # (n_out,) float32
    spike_mask: np.ndarray | None  # (n_out, max_steps) bool
    spike_event_idx: np.ndarray | None
    event_times: np.ndarray       # (max_out_spikes,) float32
    event_source_idx: np.ndarray  # (max_out_spikes,) int32
    event_gain: np.ndarray        # (max_out_spikes,) float32
    n_real_events: int            # spikes in the layer, not clipped to max_out_spikes
    spike_count: int
    extra_steps_needed: int
    fits: bool
    v_steps: np.ndarray | None = None   # (n_out, max_steps) with trace=True
    event_ms: np.ndarray | None = None


def decay_base(tau) -> np.ndarray:
    """float32(1 - 1/tau) per neuron: the base XLA raises to the Δt power (affine.py:27-31,
    where a Python-float base meets a float32 exponent array)."""
    return np.asarray(1.0 - 1.0 / np.asarray(tau, dtype=np.float64), dtype=np.float32)


def float_fc_forward(layer, w, times, src, n_real, gain=None, tau=None, *, dense=True,
                     threads=1, trace=False) -> FloatResult:
    """One float FC layer over one stream.  layer has the FCLayer fields n_in, n_out, tau,
    v_th, chunk_size, max_out_spikes, max_extra_steps; w is (n_out, n_in) float32; tau, when
    given, overrides layer.tau per neuron (n_out,).  dense=True also returns the
    (n_out, max_steps) spike_mask / spike_event_idx arrays."""
    n_out, n_in = int(layer.n_out), int(layer.n_in)
    t = np.ascontiguousarray(np.asarray(times, dtype=np.float32))
    s = np.ascontiguousarray(np.asarray(src), dtype=np.int32)
    L = int(t.shape[0])
    wf = np.ascontiguousarray(np.asarray(w, dtype=np.float32).reshape(n_out, n_in))
    base = decay_base(np.broadcast_to(layer.tau if tau is None else tau, (n_out,)))
    g = None if gain is None else np.ascontiguousarray(np.asarray(gain, dtype=np.float32))
    C = int(layer.chunk_size)
    steps = -(-L // C) + int(layer.max_extra_steps)
    M = int(layer.max_out_spikes)
    geom = _FloatGeom(n_in, n_out, C, M, int(layer.max_extra_steps), float(layer.v_th))
    vf = np.empty(n_out, np.float32)
    mask = np.empty((n_out, steps), np.uint8) if dense else None
    eidx = np.empty((n_out, steps), np.int32) if dense else None
    ot = np.empty(max(M, 1), np.float32)
    os_ = np.empty(max(M, 1), np.int32)
    og = np.empty(max(M, 1), np.float32)
    vs = np.empty((n_out, steps), np.float32) if trace else None
    ms = np.empty((n_out, steps), np.float32) if trace else None
    out = _FloatOut(_p(vf, _f32p), _p(mask, _u8p) if dense else None,
                    _p(eidx, _i32p) if dense else None, _p(ot, _f32p), _p(os_, _i32p),
                    _p(og, _f32p), 0, 0, 0, _p(vs, _f32p) if trace else None,
                    _p(ms, _f32p) if trace else None)
    rc = lib().so_float_fc_forward(ctypes.byref(geom), _p(wf, _f32p), _p(base, _f32p),
                                   _p(t, _f32p), _p(s, _i32p),
                                   _p(g, _f32p) if g is not None else None, L, int(n_real),
                                   int(threads), ctypes.byref(out))
    if rc:
        raise ValueError(f"oracle float layer failed rc={rc}")
    return FloatResult(vf, mask.astype(bool) if dense else None, eidx, ot[:M], os_[:M], og[:M],
                       int(out.n_real_out), int(out.n_real_out), int(out.extra_steps_needed),
                       bool(out.fits), vs, ms)


def float_seq64(layer, w, times, src, n_real, gain=None, tau=None, near=1e-6):
    """Float64 yardstick of a float FC layer's sequential semantics (so_float_seq64): returns
    (v_final (n_out,) float64, first_near (n_out,) int32: the first event whose value came within
    near * |v_th| of the threshold, len(times) when none did)."""
    n_out, n_in = int(layer.n_out), int(layer.n_in)
    t = np.ascontiguousarray(np.asarray(times, dtype=np.float32))
    s = np.ascontiguousarray(np.asarray(src), dtype=np.int32)
    wf = np.ascontiguousarray(np.asarray(w, dtype=np.float32).reshape(n_out, n_in))
    base = decay_base(np.broadcast_to(layer.tau if tau is None else tau, (n_out,)))
    g = None if gain is None else np.ascontiguousarray(np.asarray(gain, dtype=np.float32))
    vf = np.empty(n_out, np.float64)
    fn = np.empty(n_out, np.int32)
    rc = lib().so_float_seq64(n_in, n_out, _p(wf, _f32p), _p(base, _f32p), _p(t, _f32p),
                              _p(s, _i32p), _p(g, _f32p) if g is not None else None,
                              int(t.shape[0]), int(n_real), int(layer.chunk_size),
                              int(layer.max_extra_steps), ctypes.c_double(float(layer.v_th)),
                              ctypes.c_double(float(near)),
                              vf.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), _p(fn, _i32p))
    if rc:
        raise ValueError(f"oracle float64 yardstick failed rc={rc}")
    return vf, fn


def affine_scan(a, b):
    """lax.associative_scan(combine, AffineMap(a, b)) of float/affine.py:20-24, in float32."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    b = np.ascontiguousarray(np.asarray(b, dtype=np.float32))
    oa, ob = np.empty_like(a), np.empty_like(b)
    rc = lib().so_affine_scan(_p(a, _f32p), _p(b, _f32p), ctypes.c_int64(a.shape[0]),
                              _p(oa, _f32p), _p(ob, _f32p))
    if rc:
        raise ValueError(f"oracle affine scan failed rc={rc}")
    return oa, ob


class _FloatConvGeom(ctypes.Structure):
    _fields_ = [("conv", _ConvGeom), ("chunk_size", ctypes.c_int32), ("v_th", ctypes.c_float)]


class _FloatConvOut(ctypes.Structure):
    _fields_ = [("v_final", _f32p), ("spike_mask", _u8p), ("spike_event_idx", _i32p),
                ("v_steps", _f32p), ("event_ms", _f32p), ("out_times", _f32p),
                ("out_src", _i32p), ("out_gain", _f32p), ("n_real_out", ctypes.c_int32),
                ("needed_queue", ctypes.c_int32), ("extra_steps_needed", ctypes.c_int32),
                ("fits", ctypes.c_int32)]


class FloatConvResult(NamedTuple):
    """ConvLayer.forward with FloatBackend (layers/conv.py:124-149) for one sample: the forward
    values, output EventStream, needs, and (trace=True) LayerForwardTrace's per-step arrays
    (trace.py:13-22; pointer resolved to ms as resolve_ms_conv does)."""
    v_final: np.ndarray            # (n_neurons,) float32
    spike_mask: np.ndarray | None  # (n_neurons, max_steps) bool
    spike_event_idx: np.ndarray | None
    v_steps: np.ndarray | None     # (n_neurons, max_steps) float32
    event_ms: np.ndarray | None
    event_times: np.ndarray
    event_source_idx: np.ndarray
    event_gain: np.ndarray
    n_real_events: int
    needed_queue: int
    extra_steps_needed: int
    fits: bool


def float_conv_forward(layer, w, times, src, n_real, gain=None, *, trace=False
                       ) -> FloatConvResult:
    """One float conv layer over one stream.  layer has the ConvLayer fields (geometry, tau,
    v_th, chunk_size, max_queue_len, max_out_spikes, max_extra_steps); w is (oc, ic, k, k)."""
    t = np.ascontiguousarray(np.asarray(times, dtype=np.float32))
    s = np.ascontiguousarray(np.asarray(src), dtype=np.int32)
    E = int(t.shape[0])
    wf = np.ascontiguousarray(np.asarray(w, dtype=np.float32).reshape(layer.weight_shape))
    g = None if gain is None else np.ascontiguousarray(np.asarray(gain, dtype=np.float32))
    L, C = int(layer.max_queue_len), int(layer.chunk_size)
    steps = -(-L // C) + int(layer.max_extra_steps)
    n = int(layer.n_neurons)
    M = int(layer.max_out_spikes)
    geom = _FloatConvGeom(_conv_geom(layer), C, float(layer.v_th))
    vf = np.empty(n, np.float32)
    mask = np.empty((n, steps), np.uint8)
    eidx = np.empty((n, steps), np.int32)
    vs = np.empty((n, steps), np.float32) if trace else None
    ms = np.empty((n, steps), np.float32) if trace else None
    ot = np.empty(max(M, 1), np.float32)
    os_ = np.empty(max(M, 1), np.int32)
    og = np.empty(max(M, 1), np.float32)
    out = _FloatConvOut(_p(vf, _f32p), _p(mask, _u8p), _p(eidx, _i32p),
                        _p(vs, _f32p) if trace else None, _p(ms, _f32p) if trace else None,
                        _p(ot, _f32p), _p(os_, _i32p), _p(og, _f32p), 0, 0, 0, 0)
    base = float(decay_base(layer.tau))
    rc = lib().so_float_conv_forward(ctypes.byref(geom), _p(wf, _f32p), ctypes.c_float(base),
                                     _p(t, _f32p), _p(s, _i32p),
                                     _p(g, _f32p) if g is not None else None, E, int(n_real),
                                     ctypes.byref(out))
    if rc:
        raise ValueError(f"oracle float conv layer failed rc={rc}")
    return FloatConvResult(vf, mask.astype(bool), eidx, vs, ms, ot[:M], os_[:M], og[:M],
                           int(out.n_real_out), int(out.needed_queue),
                           int(out.extra_steps_needed), bool(out.fits))
