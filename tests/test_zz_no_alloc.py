"""salt_conv_layer_forward_noalloc (the conv layer forward whose scratch is the library's fixed
device array) against salt_conv_layer_forward with a caller workspace, through the C ABI.

Calls follow one another on one stream with different layers and inputs, so each call starts
from the scratch contents the previous one left behind.  The file runs last so that the
first call's one-time setup also happens after every other test has used the library."""
import ctypes
import os
import re

import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from salt_b200 import _lib
from salt_b200.backend import conv_desc, quant_desc
from _cases import make_events, make_params

_HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                       "salt_b200.h")
_m = re.search(r"#define SALT_NOALLOC_SCRATCH_BYTES \(\(size_t\)(\d+) << (\d+)\)",
               open(_HEADER).read())
NOALLOC_SCRATCH_BYTES = int(_m.group(1)) << int(_m.group(2))


def _layer(geom, L=96, M=2000):
    ic, h, w, oc, k, s, p = geom
    return S.ConvLayer(name="c", ic=ic, h_in=h, w_in=w, oc=oc, k=k, s=s, p=p, init_k=1.0,
                       tau=20.0, max_queue_len=L, max_out_spikes=M)


def _run(layer, params, times, src, nr, noalloc):
    """One conv layer forward through the C ABI; returns host copies of every output."""
    from salt_b200 import device as D

    lib = _lib.lib()
    B, E = times.shape
    qd, vth = quant_desc(params, "round", layer.n_neurons)
    d = conv_desc(layer)
    q = D.to_device(np.asarray(params.q).reshape(layer.weight_shape), np.int32)
    lut = D.to_device(params.decay_table_int, np.int32)
    vt = D.to_device(vth, np.int32)
    t_d, s_d, n_d = D.to_device(times, np.float32), D.to_device(src, np.int32), D.to_device(nr, np.int32)
    M = layer.max_out_spikes
    out_t = D.DeviceArray.full((B, M), -1.0, np.float32)
    out_s = D.DeviceArray.full((B, M), -1, np.int32)
    out_n = D.DeviceArray.full((B,), -1, np.int32)
    v_final = D.DeviceArray.full((B, layer.n_neurons), -7, np.int32)
    stats = D.DeviceArray.full((6, B), -7, np.int32)
    p = D.ptr
    sin = _lib.StreamIn(p(t_d), p(s_d), p(n_d), E, 1)
    sout = _lib.StreamOut(p(out_t), p(out_s), p(out_n))
    st = _lib.LayerStats(*[p(stats[i]) for i in range(6)])
    stream = D.stream_handle()
    args = (_lib.byref(d), _lib.byref(qd), p(q), p(lut), p(vt), B, _lib.byref(sin),
            _lib.byref(sout), p(v_final), _lib.byref(st))
    if noalloc:
        _lib.check(lib.salt_conv_layer_forward_noalloc(*args, stream))
    else:
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.salt_conv_layer_workspace_size(_lib.byref(d), _lib.byref(qd), B, E,
                                                      _lib.byref(nbytes)))
        assert nbytes.value <= NOALLOC_SCRATCH_BYTES
        ws = D.workspace(nbytes.value)
        _lib.check(lib.salt_conv_layer_forward(*args, p(ws), nbytes.value, stream))
    D.current_stream().synchronize()
    n = out_n.numpy()
    k = np.minimum(n, M)
    ot, os_ = out_t.numpy(), out_s.numpy()
    return dict(n_real=n, v_final=v_final.numpy(), stats=stats.numpy(),
                times=[ot[b, :k[b]] for b in range(B)], src=[os_[b, :k[b]] for b in range(B)])


CALLS = [  # (geometry (ic, h, w, oc, k, s, p), batch, stream capacity, seed)
    ((2, 34, 34, 8, 3, 1, 1), 6, 900, 1),     # 1156 positions: the tiled path
    ((2, 34, 34, 16, 3, 2, 0), 12, 1500, 2),  # one tile per sample, more spike words
    ((2, 34, 34, 8, 3, 1, 1), 6, 900, 3),     # back to the first layout over new inputs
]


@pytest.mark.gpu
def test_noalloc_matches_the_workspace_entry_on_consecutive_calls():
    for geom, B, E, seed in CALLS:
        rng = np.random.default_rng(seed)
        layer = _layer(geom)
        params = make_params(layer, rng, vth=(60, 200))
        times, src, nr = make_events(rng, B, E, geom[0] * geom[1] * geom[2])
        got = _run(layer, params, times, src, nr, noalloc=True)
        ref = _run(layer, params, times, src, nr, noalloc=False)
        assert int(ref["n_real"].sum()) > 0
        # integer work: equality is the tolerance
        np.testing.assert_array_equal(got["n_real"], ref["n_real"])
        np.testing.assert_array_equal(got["v_final"], ref["v_final"])
        np.testing.assert_array_equal(got["stats"], ref["stats"])
        for b in range(B):
            np.testing.assert_array_equal(got["times"][b], ref["times"][b])
            np.testing.assert_array_equal(got["src"][b], ref["src"][b])
        # and pinned to the CPU oracle directly (the stream is read with virtual pads: entries
        # past n_real are time 1e12, source 0)
        for b in range(B):
            t, s = times[b].copy(), src[b].copy()
            t[nr[b]:], s[nr[b]:] = np.float32(1e12), 0
            o = O.conv_forward(layer, params, t, s, int(nr[b]))
            np.testing.assert_array_equal(got["v_final"][b], o.v_final)
            assert int(got["n_real"][b]) == o.n_real_events
            np.testing.assert_array_equal(got["times"][b], o.event_times[:len(got["times"][b])])
            np.testing.assert_array_equal(got["src"][b], o.event_source_idx[:len(got["src"][b])])


def test_noalloc_rejects_layers_beyond_the_fixed_scratch():
    """Checked on the host before anything is enqueued, so no device is needed."""
    lib = _lib.lib()
    layer = _layer((2, 34, 34, 16, 3, 2, 0))
    d = conv_desc(layer)
    qd, _ = quant_desc(make_params(layer, np.random.default_rng(0)), "round", layer.n_neurons)
    B, E = 256, 20000
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.salt_conv_layer_workspace_size(_lib.byref(d), _lib.byref(qd), B, E,
                                                  _lib.byref(nbytes)))
    assert nbytes.value > NOALLOC_SCRATCH_BYTES
    sin = _lib.StreamIn(None, None, None, E, 1)
    sout = _lib.StreamOut(None, None, None)
    rc = lib.salt_conv_layer_forward_noalloc(_lib.byref(d), _lib.byref(qd), None, None, None, B,
                                             _lib.byref(sin), _lib.byref(sout), None, None, None)
    assert rc == _lib.SALT_WORKSPACE_TOO_SMALL
    msg = lib.salt_last_error().decode()
    assert str(NOALLOC_SCRATCH_BYTES) in msg and str(nbytes.value) in msg
