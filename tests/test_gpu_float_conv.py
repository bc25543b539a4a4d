"""GPU parity of the float conv layer (ConvLayer.forward with FloatBackend), the float per-step
traces and the calibration forward, against the CPU oracle.

The oracle composes each chunk in lax.associative_scan's order and calls the C library's powf;
the kernel streams the chunk as a left fold and calls CUDA's powf.  So potentials are compared
within a float32 tolerance, and spike sets, queue needs and output streams exactly, on seeded
cases whose potentials do not graze the threshold."""
import dataclasses

import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from salt_b200.calibrate import calibrate_v_abs_max, v_abs_max_per_channel, v_range_per_channel
from _cases import make_events, stream_of

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-5, 2e-5


def _w(layer, rng, scale=0.6):
    return rng.normal(0.0, scale, layer.weight_shape).astype(np.float32)


def _gains(rng, B, E):
    return rng.uniform(0.5, 1.5, (B, E)).astype(np.float32)


def _check_conv(layer, w, times, src, nr, gain=None, trace=False):
    st = stream_of(times, src, nr)
    if gain is not None:
        st = st._replace(event_gain=gain)
    out = S.FloatB200Backend().forward_layer(layer, w, st, trace=trace)
    for b in range(times.shape[0]):
        ref = O.float_conv_forward(layer, w, times[b], src[b], int(nr[b]),
                                   None if gain is None else gain[b], trace=trace)
        np.testing.assert_allclose(out.result.v_final[b], ref.v_final, rtol=RTOL, atol=ATOL,
                                   err_msg=f"v_final b={b}")
        assert int(out.result.spike_count[b]) == ref.n_real_events, f"spikes b={b}"
        n = min(ref.n_real_events, layer.max_out_spikes)
        np.testing.assert_array_equal(out.stream.event_source_idx[b][:n], ref.event_source_idx[:n])
        np.testing.assert_array_equal(out.stream.event_times[b][:n], ref.event_times[:n])
        assert int(out.diag.needed["max_queue_len"][b]) == ref.needed_queue
        assert int(out.diag.needed["max_extra_steps"][b]) == ref.extra_steps_needed
        if trace:
            np.testing.assert_array_equal(out.trace.spike_mask[b], ref.spike_mask)
            np.testing.assert_allclose(out.trace.v_steps[b], ref.v_steps, rtol=RTOL, atol=ATOL)
            np.testing.assert_array_equal(np.isnan(out.trace.event_ms[b]), np.isnan(ref.event_ms))
            np.testing.assert_array_equal(np.nan_to_num(out.trace.event_ms[b]),
                                          np.nan_to_num(ref.event_ms))
    return out


def _layer(ic=2, h=10, w=10, oc=8, k=3, s=2, p=1, L=48, M=400, C=1, extra=None, v_th=1.0,
           tau=8.0):
    return S.ConvLayer(name="c", ic=ic, h_in=h, w_in=w, oc=oc, k=k, s=s, p=p, init_k=1.0, tau=tau,
                       v_th=v_th, chunk_size=C, max_queue_len=L, max_out_spikes=M,
                       max_extra_steps=extra)


def test_reference_known_answers_on_the_gpu():
    """test_conv_queue.py:232-288 and :613-634 through the B200 layer."""
    wk = np.array([[ky * 3 + kx + 1 for kx in range(3)] for ky in range(3)], np.float32)[None, None]
    one = _layer(ic=1, h=5, w=5, oc=1, L=1, C=1, extra=0, v_th=1e9, tau=4.0)
    out = S.FloatB200Backend().forward_layer(one, wk, stream_of(
        np.array([1.0], np.float32), np.array([6], np.int32), 1))
    exp = np.zeros(9, np.float32)
    exp[[0, 1, 3, 4]] = [9.0, 7.0, 3.0, 1.0]
    np.testing.assert_allclose(out.result.v_final, exp, atol=1e-6)
    three = _layer(ic=1, h=5, w=5, oc=1, L=3, C=3, extra=2, v_th=1e9, tau=4.0)
    out = S.FloatB200Backend().forward_layer(three, wk, stream_of(
        np.array([1.0, 2.0, 5.0], np.float32), np.array([6, 0, 12], np.int32), 3))
    assert abs(float(out.result.v_final[1]) - 2.21484375) < 1e-6
    full = S.ConvLayer(name="conv", ic=1, h_in=4, w_in=4, oc=1, k=3, s=2, p=1, init_k=1.0,
                       tau=4.0, v_th=1e9, max_queue_len=3, max_out_spikes=16)
    out = S.FloatB200Backend().forward_layer(full, np.full((1, 1, 3, 3), 0.1, np.float32),
                                             stream_of(np.array([1.0, 2.0, 3.0, 5.0], np.float32),
                                                       np.array([0, 3, 0, 15], np.int32), 4))
    assert abs(float(out.result.v_final[0]) - 0.087890625) < 1e-6
    short = dataclasses.replace(full, max_queue_len=2, max_extra_steps=0)
    out = S.FloatB200Backend().forward_layer(short, np.full((1, 1, 3, 3), 0.1, np.float32),
                                             stream_of(np.array([1.0, 2.0, 3.0, 5.0], np.float32),
                                                       np.array([0, 3, 0, 15], np.int32), 4))
    assert int(out.diag.needed["max_queue_len"]) == 3


GEOMS = [  # (ic, h, w, oc, k, s, p)
    (2, 10, 10, 8, 3, 2, 1),
    (2, 12, 12, 16, 3, 2, 0),
    (3, 9, 7, 5, 3, 1, 1),
    (1, 6, 6, 40, 2, 2, 0),     # two channel groups
    (2, 8, 8, 4, 5, 1, 2),
]


@pytest.mark.parametrize("geom", GEOMS)
@pytest.mark.parametrize("C", [1, 4])
def test_float_conv_matches_oracle(geom, C):
    ic, h, w, oc, k, s, p = geom
    rng = np.random.default_rng(hash((geom, C)) % 2 ** 32)
    layer = _layer(ic, h, w, oc, k, s, p, L=40, M=500, C=C)
    times, src, nr = make_events(rng, 4, 160, ic * h * w, t_max=60)
    _check_conv(layer, _w(layer, rng), times, src, nr)


def test_float_conv_gains_truncation_and_short_queues():
    rng = np.random.default_rng(21)
    layer = _layer(L=6, M=25, C=2, extra=1)      # queues and steps run out, outputs truncated
    times, src, nr = make_events(rng, 5, 200, 200, t_max=80, pad_time="big")
    nr[1], nr[2] = 0, 260                        # empty sample, n_real beyond the stream
    out = _check_conv(layer, _w(layer, rng, 1.0), times, src, nr, gain=_gains(rng, 5, 200))
    assert not out.diag.needed["max_queue_len"].max() <= 6


@pytest.mark.parametrize("C", [1, 3])
def test_float_conv_traces_match_oracle(C):
    rng = np.random.default_rng(31 + C)
    layer = _layer(ic=2, h=8, w=8, oc=6, L=24, M=300, C=C)
    times, src, nr = make_events(rng, 3, 90, 128, t_max=50)
    _check_conv(layer, _w(layer, rng), times, src, nr, trace=True)


def test_float_fc_traces_match_oracle():
    rng = np.random.default_rng(41)
    layer = S.FCLayer(name="f", n_in=50, n_out=20, init_k=1.0, tau=10.0, v_th=1.0, chunk_size=1,
                      max_out_spikes=400)
    w = rng.normal(0, 0.5, (20, 50)).astype(np.float32)
    times, src, nr = make_events(rng, 3, 120, 50, t_max=60)
    out = S.FloatB200Backend().forward_layer(layer, w, stream_of(times, src, nr), trace=True)
    for b in range(3):
        ref = O.float_fc_forward(layer, w, times[b], src[b], int(nr[b]), trace=True)
        np.testing.assert_array_equal(out.trace.spike_mask[b], ref.spike_mask)
        np.testing.assert_allclose(out.trace.v_steps[b], ref.v_steps, rtol=RTOL, atol=ATOL)
        np.testing.assert_array_equal(np.isnan(out.trace.event_ms[b]), np.isnan(ref.event_ms))
        np.testing.assert_array_equal(np.nan_to_num(out.trace.event_ms[b]),
                                      np.nan_to_num(ref.event_ms))


def _float_net():
    return S.Network.build((2, 10, 10), [
        S.conv(8, k=3, s=2, p=1, init_k=1.0, tau=8.0, v_th=1.0, chunk_size=1, max_queue_len=64,
               max_out_spikes=600),
        S.conv(12, k=3, s=2, p=1, init_k=1.0, tau=8.0, v_th=1.0, chunk_size=1, max_queue_len=64,
               max_out_spikes=400),
        S.fc(5, init_k=1.0, tau=8.0, v_th=1e9, chunk_size=1, max_out_spikes=1)])


def test_float_network_chain_and_ranges_match_oracle():
    rng = np.random.default_rng(51)
    net = _float_net()
    ws = [_w(l, rng, 0.8) if isinstance(l, S.ConvLayer) else rng.normal(0, 0.3, (l.n_out, l.n_in)).astype(
        np.float32) for l in net.layers]
    times, src, nr = make_events(rng, 3, 150, 200, t_max=60)
    be = S.FloatB200Backend()
    out = be.run_network(net.layers, ws, stream_of(times, src, nr), trace=True, v_range=True,
                         keep_streams=True)
    for b in range(3):
        t, s_, n = times[b], src[b], int(nr[b])
        for i, layer in enumerate(net.layers):
            if isinstance(layer, S.ConvLayer):
                ref = O.float_conv_forward(layer, ws[i], t, s_, n, trace=True)
            else:
                ref = O.float_fc_forward(layer, ws[i], t, s_, n, trace=True)
            np.testing.assert_allclose(out.results[i].v_final[b], ref.v_final, rtol=RTOL,
                                       atol=ATOL)
            assert int(out.results[i].spike_count[b]) == ref.n_real_events
            (vmax, vmin), = v_range_per_channel([layer], [ref.v_steps])
            np.testing.assert_allclose(out.v_ranges[i][0][b], vmax, rtol=RTOL, atol=ATOL)
            np.testing.assert_allclose(out.v_ranges[i][1][b], vmin, rtol=RTOL, atol=ATOL)
            np.testing.assert_allclose(out.traces[i].v_steps[b], ref.v_steps, rtol=RTOL,
                                       atol=ATOL)
            st = out.streams[i]
            t, s_, n = (st.event_times[b], st.event_source_idx[b], int(st.n_real_events[b]))


def test_calibration_matches_the_oracle_reduction():
    """example/quant_run.py:30-44 on the GPU vs the oracle's traces through the reference's
    host reduction (v_range_per_channel, merge, |.|max)."""
    rng = np.random.default_rng(61)
    net = _float_net()
    ws = [_w(l, rng, 0.8) if isinstance(l, S.ConvLayer) else rng.normal(0, 0.3, (l.n_out, l.n_in)).astype(
        np.float32) for l in net.layers]
    times, src, nr = make_events(rng, 7, 150, 200, t_max=60)
    raw = S.InputEvents(times, src, nr)
    got = calibrate_v_abs_max(net, ws, raw, batch_size=3)
    per_sample = []
    for b in range(7):
        t, s_, n = times[b], src[b], int(nr[b])
        steps = []
        for i, layer in enumerate(net.layers):
            if isinstance(layer, S.ConvLayer):
                ref = O.float_conv_forward(layer, ws[i], t, s_, n, trace=True)
            else:
                ref = O.float_fc_forward(layer, ws[i], t, s_, n, trace=True)
            steps.append(ref.v_steps)
            t, s_, n = ref.event_times, ref.event_source_idx, ref.n_real_events
        per_sample.append(v_range_per_channel(net.layers, steps))
    from salt_b200.calibrate import merge_v_ranges
    want = v_abs_max_per_channel(merge_v_ranges(per_sample))
    for g, w_ in zip(got, want):
        np.testing.assert_allclose(g, w_, rtol=RTOL, atol=ATOL)


def test_float_conv_rejects_bad_thresholds_and_chunks():
    layer = _layer(v_th=0.0)
    with pytest.raises(ValueError):
        S.FloatB200Backend().forward_layer(layer, np.zeros(layer.weight_shape, np.float32),
                                           stream_of(np.zeros((1, 4), np.float32),
                                                     np.zeros((1, 4), np.int32), np.array([4])))
