"""The dense Backend.scan plug-in (QuantB200Backend.scan, the drop-in for QuantBackend.scan of
salt_core/quant/backend.py:31-53 behind the protocol of salt_core/backend.py:64-74) called the
way the reference's layers call it (layers/conv.py:132, layers/fc.py:88): with the layer, its
materialised queue structure (built here by the oracle's restatement of
connectivity/conv.py:128-172 and connectivity/fc.py:20-33) and the layer's parameters.  Every
ScanOutput field is compared with the oracle's dense scan of the same queue."""
import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from _cases import make_events, make_params

pytestmark = pytest.mark.gpu


def _conv_structure(layer, times, src, n_in):
    st = O.conv_structure(layer, times, src, n_in)
    return S.ConvQueueStructure(n_input_events=int(n_in), **st)


def _fc_structure(times, src, n_in):
    t = np.asarray(times, np.float32)
    gap = np.diff(t, prepend=np.float32(0.0)).astype(np.float32)
    real = np.arange(t.shape[0]) < int(n_in)
    return S.FCQueueStructure(np.where(real, gap, np.float32(0.0)), np.asarray(src, np.int32),
                              int(n_in))


def _check(out, ref, L):
    r = out.result
    np.testing.assert_array_equal(r.spike_mask, ref.spike_mask)
    np.testing.assert_array_equal(r.v_final, ref.v_final)
    np.testing.assert_array_equal(r.overflowed, ref.overflowed)
    np.testing.assert_array_equal(r.v_unfitted_min, ref.v_unfitted_min)
    np.testing.assert_array_equal(r.v_unfitted_max, ref.v_unfitted_max)
    np.testing.assert_array_equal(r.spike_event_idx,
                                  np.broadcast_to(np.arange(L), r.spike_mask.shape))
    assert out.spike_gain.dtype == np.float32 and np.all(out.spike_gain == 1.0)
    assert out.spike_gain.shape == r.spike_mask.shape
    assert int(out.extra_steps_needed) == 0 and np.ndim(out.extra_steps_needed) == 0


@pytest.mark.parametrize("trace", [False, True])
@pytest.mark.parametrize("geom,L", [((2, 12, 12, 16, 3, 2, 1), 48), ((1, 6, 6, 4, 3, 1, 1), 3)])
def test_conv_scan_plugin(geom, L, trace):
    """A queue long enough for every tap, and one that truncates (needed > L)."""
    ic, h, w, oc, k, s, p = geom
    rng = np.random.default_rng(300 + L)
    layer = S.ConvLayer(name="c", ic=ic, h_in=h, w_in=w, oc=oc, k=k, s=s, p=p, init_k=1.0,
                        tau=20.0, max_queue_len=L, max_out_spikes=500)
    params = make_params(layer, rng, vth=(60, 200), f_a=8, f_V=1, i_V=10, overflow="saturate")
    times, src, nr = make_events(rng, 2, 200, ic * h * w)
    backend = S.QuantB200Backend("round")
    for b in range(2):
        structure = _conv_structure(layer, times[b], src[b], int(nr[b]))
        out = backend.scan(layer, structure, params, None, trace=trace)
        ref = O.conv_forward(layer, params, times[b], src[b], int(nr[b]), trace=trace)
        _check(out, ref, L)
        if trace:
            np.testing.assert_array_equal(out.v_steps, ref.v_steps)
            np.testing.assert_array_equal(out.v_steps[:, -1], ref.v_final)
            np.testing.assert_array_equal(out.pointer_steps, out.result.spike_event_idx)
        else:
            assert out.v_steps is None and out.pointer_steps is None


@pytest.mark.parametrize("trace", [False, True])
@pytest.mark.parametrize("fires", [True, False])
def test_fc_scan_plugin(fires, trace):
    rng = np.random.default_rng(310 + fires)
    layer = S.FCLayer(name="f", n_in=90, n_out=24, init_k=1.0, tau=20.0, max_out_spikes=600)
    params = make_params(layer, rng, vth=(100, 250), fires=fires, f_a=10, i_V=9)
    times, src, nr = make_events(rng, 2, 150, 90)
    src[0, 5] = -3        # a negative source wraps once, as XLA's gather does
    backend = S.QuantB200Backend("truncate")
    for b in range(2):
        out = backend.scan(layer, _fc_structure(times[b], src[b], nr[b]), params, None,
                           trace=trace)
        ref = O.fc_forward(layer, params, times[b], src[b], int(nr[b]), "truncate", trace=trace)
        _check(out, ref, times.shape[1])
        if trace:
            np.testing.assert_array_equal(out.v_steps, ref.v_steps)


def test_scan_rejects_float_codes():
    layer = S.FCLayer(name="f", n_in=4, n_out=2, init_k=1.0, tau=20.0)
    params = make_params(layer, np.random.default_rng(1))
    params = params._replace(q=params.q.astype(np.float32))
    with pytest.raises(ValueError):
        S.QuantB200Backend().scan(layer, _fc_structure(np.zeros(3), np.zeros(3), 3), params,
                                  None, trace=False)
