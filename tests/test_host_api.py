"""Host-side logic that needs no GPU: the C ABI library loads and exports every entry point of
include/salt_b200.h with struct layouts that match the ctypes binding; the reference-mirroring
Python API (geometry, capacity, input checks, offline integer codes); argument errors the
library reports before touching a device."""
import ctypes
import math
import os
import re
import subprocess

import numpy as np
import pytest

import salt_b200 as S
from salt_b200 import _lib
from salt_b200.capacity import GrowthPolicy, safe_extra_steps
from salt_b200.quant import QuantizedLayerParams, apply_decay_table_int, v_th_to_int

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "salt_b200.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(salt_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_function():
    lib = _lib.lib()
    missing = [f for f in header_functions() if not hasattr(lib, f)]
    assert not missing, missing
    assert set(header_functions()) == set(_lib.exported_symbols())
    assert b"sm_100a" in lib.salt_version()


def test_struct_layouts_match_the_header(tmp_path):
    structs = {"salt_quant_desc": _lib.QuantDesc, "salt_conv_desc": _lib.ConvDesc,
               "salt_fc_desc": _lib.FCDesc, "salt_stream_in": _lib.StreamIn,
               "salt_stream_out": _lib.StreamOut, "salt_layer_stats": _lib.LayerStats,
               "salt_layer_spec": _lib.LayerSpec, "salt_float_fc_desc": _lib.FloatFCDesc,
               "salt_float_layer_stats": _lib.FloatLayerStats,
               "salt_neuron_trace": _lib.NeuronTrace,
               "salt_float_conv_desc": _lib.FloatConvDesc,
               "salt_float_conv_stats": _lib.FloatConvStats,
               "salt_float_trace": _lib.FloatTrace}
    src = tmp_path / "sizes.c"
    src.write_text('#include <stdio.h>\n#include "salt_b200.h"\nint main(void){\n' + "".join(
        f'printf("{n} %zu\\n", sizeof({n}));\n' for n in structs) + "return 0;}\n")
    exe = tmp_path / "sizes"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    for line in out.split("\n"):
        if line:
            name, size = line.split()
            assert ctypes.sizeof(structs[name]) == int(size), name


def test_bad_arguments_are_reported_before_any_device_work():
    lib = _lib.lib()
    d = _lib.ConvDesc(2, 34, 34, 16, 3, 2, 0, 64, 100, 0)
    q = _lib.QuantDesc(10, 0, 24, 0, 0, 148, 1, 8, 0)
    n = ctypes.c_size_t(0)
    assert lib.salt_conv_layer_workspace_size(_lib.byref(d), _lib.byref(q), 4, 1000,
                                              _lib.byref(n)) == _lib.SALT_OK
    assert n.value > 0
    bad = _lib.QuantDesc(16, 0, 24, 0, 0, 148, 1, 8, 0)      # f_a > MAX_SHIFT_BITS
    assert lib.salt_conv_layer_workspace_size(_lib.byref(d), _lib.byref(bad), 4, 1000,
                                              _lib.byref(n)) == _lib.SALT_BAD_ARG
    assert b"f_a" in lib.salt_last_error()
    bad = _lib.QuantDesc(10, 8, 24, 0, 0, 148, 1, 8, 0)       # i_V + f_V > MAX_REGISTER_BITS
    assert lib.salt_conv_layer_workspace_size(_lib.byref(d), _lib.byref(bad), 4, 1000,
                                              _lib.byref(n)) == _lib.SALT_BAD_ARG
    degenerate = _lib.ConvDesc(2, 2, 2, 16, 3, 2, 0, 64, 100, 0)
    assert lib.salt_conv_layer_workspace_size(_lib.byref(degenerate), _lib.byref(q), 4, 1000,
                                              _lib.byref(n)) == _lib.SALT_BAD_ARG
    f = _lib.FCDesc(0, 10, 1, 0)
    assert lib.salt_fc_layer_workspace_size(_lib.byref(f), _lib.byref(q), 4, 1000,
                                            _lib.byref(n)) == _lib.SALT_BAD_ARG
    # the tile partition holds per-tile masks in one block's shared memory: a 226x226 output
    # plane (15 x 57 = 855 tiles of 16 x 4) fits, a 3999x3999 one is refused before any launch
    big_ok = _lib.ConvDesc(1, 453, 453, 16, 3, 2, 0, 64, 100, 0)
    assert lib.salt_conv_layer_workspace_size(_lib.byref(big_ok), _lib.byref(q), 1, 1000,
                                              _lib.byref(n)) == _lib.SALT_OK
    too_big = _lib.ConvDesc(1, 8000, 8000, 16, 3, 2, 0, 64, 100, 0)
    assert lib.salt_conv_layer_workspace_size(_lib.byref(too_big), _lib.byref(q), 1, 1000,
                                              _lib.byref(n)) == _lib.SALT_BAD_ARG
    assert b"tile" in lib.salt_last_error()


def test_float_conv_arguments_are_checked_on_the_host():
    lib = _lib.lib()
    n = ctypes.c_size_t(0)
    d = _lib.FloatConvDesc(2, 34, 34, 16, 3, 2, 0, 64, 100, 0, 1, 1.0)
    assert lib.salt_float_conv_layer_workspace_size(_lib.byref(d), 4, 1000,
                                                    _lib.byref(n)) == _lib.SALT_OK
    assert n.value > 0
    for bad in (_lib.FloatConvDesc(2, 34, 34, 16, 3, 2, 0, 64, 100, 0, 1, 0.0),    # v_th <= 0
                _lib.FloatConvDesc(2, 34, 34, 16, 3, 2, 0, 64, 100, 0, 0, 1.0),    # chunk 0
                _lib.FloatConvDesc(2, 34, 34, 16, 3, 2, 0, 0, 100, 0, 1, 1.0),     # no queue
                _lib.FloatConvDesc(2, 2, 2, 16, 3, 2, 0, 64, 100, 0, 1, 1.0)):     # degenerate
        assert lib.salt_float_conv_layer_workspace_size(_lib.byref(bad), 4, 1000,
                                                        _lib.byref(n)) == _lib.SALT_BAD_ARG


def test_workspace_is_independent_of_the_queue_capacity():
    lib = _lib.lib()
    q = _lib.QuantDesc(10, 0, 24, 0, 0, 148, 1, 8, 0)
    sizes = []
    for L in (16, 4096, 1 << 30):
        d = _lib.ConvDesc(2, 34, 34, 16, 3, 2, 0, L, 1000, 0)
        n = ctypes.c_size_t(0)
        assert lib.salt_conv_layer_workspace_size(_lib.byref(d), _lib.byref(q), 64, 20000,
                                                  _lib.byref(n)) == 0
        sizes.append(n.value)
    assert len(set(sizes)) == 1


def test_conv_geometry_and_specs():
    net = S.Network.build((2, 34, 34), [S.conv(16, k=3, s=2, p=0, init_k=5.0),
                                        S.conv(32, k=3, s=2, p=1, init_k=5.0),
                                        S.fc(10, init_k=5.0, v_th=1e9)])
    c1, c2, f = net.layers
    assert (c1.h_out, c1.w_out, c1.n_neurons) == (16, 16, 4096)
    assert (c2.h_out, c2.w_out, c2.n_neurons) == (8, 8, 2048)
    assert f.n_in == 2048 and [l.name for l in net.layers] == ["conv1", "conv2", "fc1"]
    assert c1.max_extra_steps == safe_extra_steps(c1.max_queue_len, c1.chunk_size)
    # the reference's production padding gives 34 -> 17 -> 9 and an FC input of 32*9*9
    net2 = S.Network.build((2, 34, 34), [S.conv(16, k=3, s=2, p=1, init_k=5.0),
                                         S.conv(32, k=3, s=2, p=1, init_k=5.0),
                                         S.fc(10, init_k=5.0)])
    assert net2.layers[2].n_in == 32 * 9 * 9
    with pytest.raises(ValueError):
        S.ConvLayer(name="x", ic=1, h_in=2, w_in=2, oc=1, k=5, s=1, p=0, init_k=1.0)
    with pytest.raises(ValueError):
        S.Network((2, 34, 34), [S.FCLayer(name="f", n_in=10, n_out=2, init_k=1.0)])
    v = np.arange(c1.n_neurons)
    assert c1.unflatten_neurons(v).shape == (16, 16, 16)
    assert c1.broadcast_channels(np.arange(16)).shape == (4096,)


def test_input_events_checked_rejects_what_the_reference_rejects():
    t = np.array([[0.0, 1.0, 2.0, 1e12]], np.float32)
    s = np.zeros((1, 4), np.int32)
    S.InputEvents.checked(t, s, np.array([3]))           # the pad may be anything
    with pytest.raises(ValueError):
        S.InputEvents.checked(np.array([[0.0, 1.5]]), s[:, :2], np.array([2]))
    with pytest.raises(ValueError):
        S.InputEvents.checked(np.array([[3.0, 1.0]]), s[:, :2], np.array([2]))
    with pytest.raises(ValueError):
        S.InputEvents.checked(np.array([[-1.0, 1.0]]), s[:, :2], np.array([2]))
    with pytest.raises(ValueError):
        S.InputEvents.checked(np.array([[0.0, 2.0 ** 31]]), s[:, :2], np.array([2]))


def test_capacity_fits_and_growth_policy():
    cap = S.Capacity(max_queue_len=10, max_out_spikes=5, max_extra_steps=0)
    diag = S.LayerDiag(np.array([3, 9]), np.zeros(2),
                       {"max_queue_len": np.array([10, 11]), "max_out_spikes": np.array([5, 5]),
                        "max_extra_steps": np.array([0, 0])})
    assert list(cap.fits(diag)) == [True, False]
    grown = GrowthPolicy().grown(cap, {"max_queue_len": 11, "max_out_spikes": 5,
                                       "max_extra_steps": 0}, chunk_size=1)
    assert grown["max_queue_len"] == math.ceil(11 * 1.5)
    with pytest.raises(KeyError):
        cap.replace(nope=1)


def test_offline_codes():
    for f_a, tau in [(8, 16.0), (4, 4.0), (12, 16.0), (10, 20.0)]:
        d = S.delta_t_max(f_a, tau)
        eps, base = 2.0 ** -(f_a + 1), 1.0 - 1.0 / tau
        assert base ** d >= eps > base ** (d + 1)
        t = S.build_decay_table_int(f_a, tau)
        assert np.all(np.diff(t) <= 0) and t.min() >= 0 and t.max() <= 2 ** f_a - 1
    assert S.delta_t_max(10, 20.0) == 148 and S.delta_t_max(6, 20.0) == 94
    a, ident = apply_decay_table_int([0.0, 1.0, 2.0, 3.0, 60.0], S.build_decay_table_int(4, 4.0))
    assert list(ident) == [True, False, False, False, False] and list(a[1:]) == [12, 9, 7, 0]
    with pytest.raises(ValueError):
        apply_decay_table_int([1.5], S.build_decay_table_int(4, 4.0))
    assert int(v_th_to_int(1.0, 0.5, 2, 8)) == 8
    with pytest.raises(ValueError):
        v_th_to_int(1000.0, 1.0, 0, 4)
    q, scale = S.quantize_to_int(np.array([0.5, -1.0, 0.25]), 8)
    assert list(q) == [64, -127, 32]
    assert list(S.round_half_away_from_zero(np.array([2.5, -2.5, 0.4]))) == [3.0, -3.0, 0.0]


def test_backend_rejects_float_weight_codes_and_wide_registers():
    layer = S.FCLayer(name="f", n_in=2, n_out=2, init_k=5.0)
    from salt_b200.backend import quant_desc
    base = QuantizedLayerParams(q=np.ones((2, 2), np.int32), decay_table_int=np.array([12], np.int32),
                                v_th_int=np.array([8, 8]), scale=1.0, f_a=4, f_V=0, i_V=16)
    quant_desc(base, "round", 2)
    with pytest.raises(ValueError):
        quant_desc(base._replace(q=np.ones((2, 2)) * 0.5), "round", 2)
    with pytest.raises(ValueError):
        quant_desc(base._replace(f_a=16), "round", 2)
    with pytest.raises(ValueError):
        quant_desc(base._replace(i_V=31), "round", 2)
    with pytest.raises(ValueError):
        quant_desc(base, "ceil", 2)
    d, _ = quant_desc(base._replace(v_th_int=np.array([0, 8])), "round", 2)
    assert d.needs_tail == 1
    d, _ = quant_desc(base._replace(q=np.full((2, 2), 300)), "round", 2)
    assert d.q_bits == 16
    del layer


def test_workloads_are_deterministic_and_shaped_like_the_configs():
    from salt_b200 import workloads as W
    a, b = W.config2(seed=3), W.config2(seed=3)
    np.testing.assert_array_equal(a.times, b.times)
    np.testing.assert_array_equal(a.src, b.src)
    assert a.batch == 64 and abs(a.n_real.mean() - 5000) < 100
    assert a.src.max() < 2 * 34 * 34
    c1 = W.config1()
    assert c1.events == 5000 and int(c1.params[0].v_th_int[0]) == 256
    c3 = W.config3(seed=1, batch=32)
    assert c3.n_real.min() >= 2000 and c3.n_real.max() <= 20000
    real = np.arange(c3.times.shape[1])[None, :] < c3.n_real[:, None]
    assert np.all(np.diff(np.where(real, c3.times, np.inf), axis=1)[real[:, 1:]] >= 0)
    t, s = W.burst_events(np.random.default_rng(0), 5000, 2 * 128 * 128)
    assert np.all(np.diff(t) >= 0) and np.all(t == np.floor(t))


_NO_TORCH_IMPORTS = """
import sys
sys.path.insert(0, {root!r})
import salt_b200
from salt_b200 import (backend, plan, device, float_backend, sharding, comm, quant_run, io,
                       calibrate, workloads, trace)
assert 'torch' not in sys.modules, 'the package imported torch'
print('ok')
"""


def test_package_never_imports_torch():
    """The product path is numpy + the C ABI: importing every module of the package leaves torch
    unimported (device memory, streams, events, graphs and NCCL go through libsalt_b200 and
    libnccl)."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _NO_TORCH_IMPORTS.format(root=root)],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stderr[-2000:]


def test_nccl_unique_id_survives_the_round_trip():
    """The 128-byte NCCL unique id (with its zero bytes) reaches ncclCommInitRank unchanged."""
    from salt_b200.comm import _UniqueId
    raw = bytes(range(128))[::-1]
    assert _UniqueId.from_bytes(raw).to_bytes() == raw
    with pytest.raises(ValueError):
        _UniqueId.from_bytes(b"short")
