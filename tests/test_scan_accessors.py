"""The layers' ScanLayer accessors (neuron_delta_t, gather_weight_codes, neuron_n_real — what the
dense Backend.scan plug-in reads from a layer, salt_core/backend.py:36-61) on CPU: fed with a
queue structure and scanned by the oracle's dense run_layer, they reproduce the oracle's whole
layer (queue building, integer scan) for conv and FC layers."""
import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from salt_b200.quant import apply_decay_table_int
from _cases import make_events, make_params


def _dense(layer, structure, params):
    dt = layer.neuron_delta_t(structure).astype(np.float32)
    a, ident = apply_decay_table_int(dt, params.decay_table_int)
    q = layer.gather_weight_codes(structure, params.q)
    return O.run_layer(a, ident, q, params.v_th_int, f_a=params.f_a, f_V=params.f_V,
                       i_V=params.i_V, overflow_mode=params.overflow_mode)


@pytest.mark.parametrize("L", [40, 4])
def test_conv_accessors(L):
    rng = np.random.default_rng(L)
    layer = S.ConvLayer(name="c", ic=2, h_in=9, w_in=9, oc=6, k=3, s=2, p=1, init_k=1.0,
                        tau=20.0, max_queue_len=L, max_out_spikes=500)
    params = make_params(layer, rng, vth=(60, 200), f_a=8, f_V=1, i_V=10)
    times, src, nr = make_events(rng, 3, 120, 2 * 81)
    for b in range(3):
        st = S.ConvQueueStructure(n_input_events=int(nr[b]),
                                  **O.conv_structure(layer, times[b], src[b], int(nr[b])))
        got = _dense(layer, st, params)
        ref = O.conv_forward(layer, params, times[b], src[b], int(nr[b]))
        np.testing.assert_array_equal(got.v_final, ref.v_final)
        np.testing.assert_array_equal(got.spike_mask, ref.spike_mask)
        np.testing.assert_array_equal(got.v_unfitted_max, ref.v_unfitted_max)
        n_real = layer.neuron_n_real(st)
        assert n_real.shape == (layer.n_neurons,)
        np.testing.assert_array_equal(n_real[:st.n_real_events.size], st.n_real_events)


def test_fc_accessors():
    rng = np.random.default_rng(5)
    layer = S.FCLayer(name="f", n_in=30, n_out=12, init_k=1.0, tau=20.0, max_out_spikes=400)
    params = make_params(layer, rng, vth=(100, 250))
    times, src, nr = make_events(rng, 3, 100, 30)
    src[1, ::7] -= 35     # negative sources: XLA wraps them once, then clamps
    for b in range(3):
        t = times[b]
        gap = np.diff(t, prepend=np.float32(0.0)).astype(np.float32)
        real = np.arange(t.shape[0]) < nr[b]
        st = S.FCQueueStructure(np.where(real, gap, np.float32(0)), src[b], int(nr[b]))
        got = _dense(layer, st, params)
        ref = O.fc_forward(layer, params, t, src[b], int(nr[b]))
        np.testing.assert_array_equal(got.v_final, ref.v_final)
        np.testing.assert_array_equal(got.spike_mask, ref.spike_mask)
        assert np.all(layer.neuron_n_real(st) == nr[b])
