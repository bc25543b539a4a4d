"""ctypes binding of libsalt_b200.so (include/salt_b200.h).

The library must have been built (``build.py``); importing the product path without it raises:
there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsalt_b200.so")

SALT_OK, SALT_BAD_ARG, SALT_CUDA_ERROR, SALT_NO_DEVICE, SALT_WORKSPACE_TOO_SMALL = 0, 1, 2, 3, 4
_i32 = ctypes.c_int32
_vp = ctypes.c_void_p


class QuantDesc(ctypes.Structure):
    _fields_ = [(n, _i32) for n in ("f_a", "f_V", "i_V", "round_mode", "overflow_mode", "lut_len",
                                    "has_vth", "q_bits", "needs_tail")]


class ConvDesc(ctypes.Structure):
    _fields_ = [(n, _i32) for n in ("ic", "h_in", "w_in", "oc", "k", "s", "p", "max_queue_len",
                                    "max_out_spikes", "max_extra_steps")]


class FCDesc(ctypes.Structure):
    _fields_ = [(n, _i32) for n in ("n_in", "n_out", "max_out_spikes", "max_extra_steps")]


class StreamIn(ctypes.Structure):
    _fields_ = [("times", _vp), ("src", _vp), ("n_real", _vp), ("capacity", _i32),
                ("virtual_pads", _i32)]


class StreamOut(ctypes.Structure):
    _fields_ = [("times", _vp), ("src", _vp), ("n_real", _vp)]


class LayerStats(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("spike_count", "needed_queue", "overflowed", "vmin", "vmax",
                                   "fits")]


class FloatFCDesc(ctypes.Structure):
    _fields_ = [("n_in", _i32), ("n_out", _i32), ("chunk_size", _i32), ("max_out_spikes", _i32),
                ("max_extra_steps", _i32), ("v_th", ctypes.c_float)]


class FloatConvDesc(ctypes.Structure):
    _fields_ = [("ic", _i32), ("h_in", _i32), ("w_in", _i32), ("oc", _i32), ("k", _i32),
                ("s", _i32), ("p", _i32), ("max_queue_len", _i32), ("max_out_spikes", _i32),
                ("max_extra_steps", _i32), ("chunk_size", _i32), ("v_th", ctypes.c_float)]


class FloatConvStats(ctypes.Structure):
    _fields_ = [("spike_count", _vp), ("needed_queue", _vp), ("needed_extra_steps", _vp),
                ("fits", _vp)]


class FloatTrace(ctypes.Structure):
    _fields_ = [("v_steps", _vp), ("event_ms", _vp), ("spike_mask", _vp), ("v_max", _vp),
                ("v_min", _vp)]


class FloatLayerStats(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("spike_count", "needed_extra_steps", "fits")]


class NeuronTrace(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("first_overflow", "v_before", "v_after", "spiked", "time_ms",
                                   "v_min", "v_max", "v_final", "spike_count")]


class LayerSpec(ctypes.Structure):
    _fields_ = [("kind", _i32), ("conv", ConvDesc), ("fc", FCDesc), ("quant", QuantDesc),
                ("q_host", _vp), ("lut_host", _vp), ("vth_host", _vp)]


# every function of include/salt_b200.h: name -> (restype, argtypes)
_SIGS = {
    "salt_conv_layer_workspace_size": (_i32, [_vp, _vp, _i32, _i32, _vp]),
    "salt_conv_layer_forward": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp,
                                       ctypes.c_size_t, _vp]),
    "salt_conv_layer_forward_noalloc": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp,
                                               _vp, _vp]),
    "salt_fc_layer_workspace_size": (_i32, [_vp, _vp, _i32, _i32, _vp]),
    "salt_fc_layer_forward": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp,
                                     ctypes.c_size_t, _vp]),
    "salt_quant_scan_dense": (_i32, [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                     _vp, _vp]),
    "salt_quant_scan_dense_trace": (_i32, [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                           _vp, _vp, _vp, _vp]),
    "salt_network_create": (_i32, [_vp, _i32, _vp]),
    "salt_network_destroy": (_i32, [_vp]),
    "salt_network_workspace_size": (_i32, [_vp, _i32, _i32, _vp]),
    "salt_network_forward_part": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp,
                                         _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "salt_network_forward": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                    ctypes.c_size_t, _vp]),
    "salt_network_last_launch_count": (_i32, [_vp]),
    "salt_network_set_profiling": (_i32, [_vp, _i32]),
    "salt_network_profile_read": (_i32, [_vp, _vp, _vp, _vp, _i32]),
    "salt_conv_layer_trace": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp,
                                     _vp]),
    "salt_fc_layer_trace": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "salt_stream_h2d_real": (_i32, [_vp, _vp, ctypes.c_int64, _vp, _i32, _i32, _vp, _vp, _vp]),
    "salt_float_fc_layer_workspace_size": (_i32, [_vp, _i32, _i32, _i32, _vp]),
    "salt_float_conv_layer_workspace_size": (_i32, [_vp, _i32, _i32, _vp]),
    "salt_float_conv_layer_forward": (_i32, [_vp, _vp, ctypes.c_float, _i32, _vp, _vp, _vp, _vp,
                                             _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "salt_float_fc_layer_trace": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp]),
    "salt_float_fc_set_profiling": (_i32, [_i32]),
    "salt_float_fc_profile_read": (_i32, [_vp, _vp, _vp, _i32]),
    "salt_float_fc_layer_forward": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp,
                                           ctypes.c_size_t, _vp]),
    "salt_malloc": (_i32, [ctypes.c_size_t, _vp, _vp]),
    "salt_free": (_i32, [_vp, _vp]),
    "salt_host_alloc": (_i32, [ctypes.c_size_t, _vp]),
    "salt_host_free": (_i32, [_vp]),
    "salt_memcpy_async": (_i32, [_vp, _vp, ctypes.c_size_t, _vp]),
    "salt_memset_async": (_i32, [_vp, _i32, ctypes.c_size_t, _vp]),
    "salt_device_count": (_i32, [_vp]),
    "salt_set_device": (_i32, [_i32]),
    "salt_get_device": (_i32, [_vp]),
    "salt_device_synchronize": (_i32, []),
    "salt_stream_create": (_i32, [_vp]),
    "salt_stream_create_high_priority": (_i32, [_vp]),
    "salt_stream_destroy": (_i32, [_vp]),
    "salt_stream_synchronize": (_i32, [_vp]),
    "salt_stream_wait_event": (_i32, [_vp, _vp]),
    "salt_event_create": (_i32, [_i32, _vp]),
    "salt_event_destroy": (_i32, [_vp]),
    "salt_event_record": (_i32, [_vp, _vp]),
    "salt_event_synchronize": (_i32, [_vp]),
    "salt_event_query": (_i32, [_vp, _vp]),
    "salt_event_elapsed_ms": (_i32, [_vp, _vp, _vp]),
    "salt_graph_begin_capture": (_i32, [_vp]),
    "salt_graph_end_capture": (_i32, [_vp, _vp]),
    "salt_graph_launch": (_i32, [_vp, _vp]),
    "salt_graph_destroy": (_i32, [_vp]),
    "salt_last_error": (ctypes.c_char_p, []),
    "salt_version": (ctypes.c_char_p, []),
    "salt_launch_counter": (ctypes.c_int64, [_i32]),
}

_lib = None


class SaltError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"salt_b200 status {status}: {message}")
        self.status = status


class ArgumentError(SaltError, ValueError):
    """SALT_BAD_ARG: the reference raises ValueError for the same inputs."""


def lib():
    """The loaded library; raises when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with build.py (there is no "
                               "CPU fallback for the salt_b200 kernels)")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def check(status: int) -> None:
    if status == SALT_OK:
        return
    msg = lib().salt_last_error().decode(errors="replace")
    if status == SALT_BAD_ARG:
        raise ArgumentError(status, msg)
    raise SaltError(status, msg)


def exported_symbols() -> list[str]:
    return list(_SIGS)


def byref(x):
    return ctypes.cast(ctypes.pointer(x), _vp)
