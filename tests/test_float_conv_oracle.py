"""The float conv oracle (ConvLayer.forward with FloatBackend) against the reference's known
answers: salt_core/tests/test_conv_queue.py (single event :232-248, degenerate and genuine
catch-up :250-288, pad events :290-313, zero-event neuron :316-331, a fire in mid-queue
:480-526, a queue full of real events :613-634), plus calibration's range helpers against
test_quant_calibrate.py."""
import dataclasses

import numpy as np
import pytest

import oracle as O
import salt_b200 as S

TOL = 1e-6


def _weight():
    """W[0, 0, ky, kx] = ky*3 + kx + 1 (test_conv_queue.py:38-42)."""
    return np.array([[ky * 3 + kx + 1 for kx in range(3)] for ky in range(3)],
                    np.float32)[None, None]


def _layer(L, steps, v_th=1e9, oc=1):
    """k3 s2 p1 onto a 3x3 plane, tau 4; the reference tests run chunk_size = max_steps."""
    C = steps
    return S.ConvLayer(name="c", ic=1, h_in=5, w_in=5, oc=oc, k=3, s=2, p=1, init_k=1.0, tau=4.0,
                       v_th=v_th, chunk_size=C, max_queue_len=L, max_out_spikes=64,
                       max_extra_steps=steps - (-(-L // C)))


def _src(x, y, c=None):
    c = np.zeros(len(x), np.int64) if c is None else np.asarray(c)
    return (c * 25 + np.asarray(y) * 5 + np.asarray(x)).astype(np.int32)


def test_single_event():
    out = O.float_conv_forward(_layer(1, 1), _weight(), [1.0], _src([1], [1]), 1)
    expected = np.zeros(9, np.float32)
    expected[[0, 1, 3, 4]] = [9.0, 7.0, 3.0, 1.0]
    np.testing.assert_allclose(out.v_final, expected, atol=TOL)
    assert out.v_final[2] == 0.0 and not np.isnan(out.v_final).any()


def test_two_events_degenerate_catchup():
    out = O.float_conv_forward(_layer(3, 3), _weight(), [1.0, 2.0], _src([1, 0], [1, 0]), 2)
    expected = np.zeros(9, np.float32)
    expected[[0, 1, 3, 4]] = [11.75, 5.25, 2.25, 0.75]
    np.testing.assert_allclose(out.v_final, expected, atol=TOL)


def test_genuine_catchup_decays():
    out = O.float_conv_forward(_layer(3, 3), _weight(), [1.0, 2.0, 5.0],
                               _src([1, 0, 2], [1, 0, 2]), 3)
    assert abs(float(out.v_final[1]) - 2.21484375) < TOL


def test_pad_event_is_not_a_tap():
    pads = O.float_conv_forward(_layer(3, 3), _weight(), [1.0, 2.0, 1e12],
                                _src([1, 0, 0], [1, 0, 0]), 2)
    plain = O.float_conv_forward(_layer(3, 3), _weight(), [1.0, 2.0], _src([1, 0], [1, 0]), 2)
    np.testing.assert_array_equal(pads.v_final, plain.v_final)


def test_fire_in_mid_queue_maps_the_column_to_the_global_event():
    t = [1.0, 1.5, 2.0, 2.5, 5.0]
    src = _src([1, 2, 1, 2, 0], [1, 2, 1, 2, 0])
    out = O.float_conv_forward(_layer(5, 5, v_th=15.0), _weight(), t, src, 5, trace=True)
    assert out.spike_mask[0, 0] and out.spike_event_idx[0, 0] == 1
    # the spike of position 0 comes from global event j = 2 (t = 2.0)
    k = int(np.nonzero(out.event_source_idx[:out.n_real_events] == 0)[0][0])
    assert out.event_times[k] == 2.0
    assert out.event_gain[k] == 1.0
    # the output stream is sorted by global event index, then neuron
    real = out.event_times[:out.n_real_events]
    assert np.all(np.diff(real) >= 0)


def _full_queue(L):
    layer = S.ConvLayer(name="conv", ic=1, h_in=4, w_in=4, oc=1, k=3, s=2, p=1, init_k=1.0,
                        tau=4.0, v_th=1e9, max_queue_len=L, max_out_spikes=16)
    return O.float_conv_forward(layer, np.full((1, 1, 3, 3), 0.1, np.float32),
                                [1.0, 2.0, 3.0, 5.0], np.array([0, 3, 0, 15], np.int32), 4)


def test_full_queue_needs_the_catchup_column():
    out = _full_queue(2)
    assert out.needed_queue == 3 and not out.fits


def test_queue_with_room_decays_to_the_global_last_time():
    out = _full_queue(3)
    assert out.fits
    assert abs(float(out.v_final[0]) - 0.087890625) < TOL


def test_trace_rows_end_at_v_final_and_mark_idle_steps():
    rng = np.random.default_rng(3)
    layer = S.ConvLayer(name="c", ic=2, h_in=8, w_in=8, oc=4, k=3, s=2, p=1, init_k=1.0,
                        tau=6.0, v_th=0.8, chunk_size=1, max_queue_len=24, max_out_spikes=200)
    E = 60
    t = np.sort(rng.integers(0, 40, E)).astype(np.float32)
    src = rng.integers(0, 2 * 64, E).astype(np.int32)
    w = rng.normal(0, 0.5, layer.weight_shape).astype(np.float32)
    out = O.float_conv_forward(layer, w, t, src, E, trace=True)
    np.testing.assert_array_equal(out.v_steps[:, -1], out.v_final)
    # steps whose pointer is at or past the neuron's real taps carry NaN times
    finite = np.isfinite(out.event_ms)
    assert np.all(np.isin(out.event_ms[finite], t))
    # chunk_size 1: one column per step, spikes reset to 0
    assert np.all(out.v_steps[out.spike_mask] == 0.0)


def test_calibration_ranges_match_hand_computation():
    """test_quant_calibrate.py:13-65: per-channel (max, min) over steps and positions."""
    from salt_b200.calibrate import merge_v_ranges, v_abs_max_per_channel, v_range_per_channel
    conv = S.ConvLayer(name="conv", ic=1, h_in=1, w_in=2, oc=2, k=1, s=1, p=0, init_k=5.0,
                       chunk_size=1, max_queue_len=3)
    fc = S.FCLayer(name="out", n_in=4, n_out=3, init_k=5.0)
    conv_steps = np.array([[0.1, 0.4, 0.2], [-0.3, 0.0, 0.0], [0.5, 0.9, -0.1],
                           [0.2, 0.2, 0.2]], np.float32)
    fc_steps = np.array([[1.0, 2.0, 3.0], [-4.0, -1.0, 0.0], [0.0, 0.0, 0.0]], np.float32)
    (cmax, cmin), (fmax, fmin) = v_range_per_channel([conv, fc], [conv_steps, fc_steps])
    np.testing.assert_allclose(cmax, [0.4, 0.9])
    np.testing.assert_allclose(cmin, [-0.3, -0.1])
    np.testing.assert_allclose(fmax, [3.0, 0.0, 0.0])
    np.testing.assert_allclose(fmin, [1.0, -4.0, 0.0])
    with pytest.raises(ValueError):
        v_range_per_channel([dataclasses.replace(conv, chunk_size=2), fc],
                            [conv_steps, fc_steps])
    [(vmax, vmin)] = merge_v_ranges([[(np.array([1.0, 2.0]), np.array([-1.0, 0.5]))],
                                     [(np.array([3.0, 1.0]), np.array([0.0, -2.0]))]])
    np.testing.assert_array_equal(vmax, [3.0, 2.0])
    np.testing.assert_array_equal(vmin, [-1.0, -2.0])
    with pytest.raises(ValueError):
        merge_v_ranges([])
    [m] = v_abs_max_per_channel([(np.array([3.0, 1.0]), np.array([-1.0, -2.0]))])
    np.testing.assert_array_equal(m, [3.0, 2.0])
