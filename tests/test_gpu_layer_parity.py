"""GPU parity: the fused B200 layer pipeline vs the CPU oracle (literal restatement of the
reference), bit for bit, on seeded random layers.  Covers the geometries, capacity truncation
(queue and output), the rare tail path (v_th_int <= 0), saturate / truncate modes, empty and
over-full input streams and multi-tile output planes."""
import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from _cases import make_events, make_params, materialised, stream_of

pytestmark = pytest.mark.gpu


def _check_layer(layer, params, times, src, nr, round_mode="round", backend=None):
    backend = backend or S.QuantB200Backend(round_mode)
    out = backend.forward_layer(layer, params, stream_of(times, src, nr))
    M = layer.max_out_spikes
    for b in range(times.shape[0]):
        ref = (O.conv_forward if isinstance(layer, S.ConvLayer) else O.fc_forward)(
            layer, params, times[b], src[b], int(nr[b]), round_mode)
        np.testing.assert_array_equal(out.result.v_final[b], ref.v_final, err_msg=f"v_final b={b}")
        assert int(out.stream.n_real_events[b]) == ref.n_real_events, f"n_real b={b}"
        np.testing.assert_array_equal(out.stream.event_source_idx[b], ref.event_source_idx,
                                      err_msg=f"src b={b}")
        np.testing.assert_array_equal(out.stream.event_times[b], ref.event_times,
                                      err_msg=f"times b={b}")
        assert int(out.result.spike_count[b]) == ref.n_real_events
        assert bool(out.result.overflowed[b]) == ref.any_overflow, f"overflow b={b}"
        assert int(out.result.v_unfitted_min[b]) == ref.vmin_all, f"vmin b={b}"
        assert int(out.result.v_unfitted_max[b]) == ref.vmax_all, f"vmax b={b}"
        if isinstance(layer, S.ConvLayer):
            assert int(out.diag.needed["max_queue_len"][b]) == ref.needed_queue
        fits = bool(layer.capacity.fits(S.LayerDiag(
            out.diag.spike_count[b], out.diag.firing_rate[b],
            {k: v[b] for k, v in out.diag.needed.items()})))
        assert fits == ref.fits
    return out


CONV_GEOMS = [  # (ic, h, w, oc, k, s, p)
    (2, 12, 12, 16, 3, 2, 0),
    (2, 12, 12, 16, 3, 2, 1),
    (3, 9, 11, 8, 3, 1, 1),
    (1, 7, 7, 1, 1, 1, 0),
    (4, 10, 10, 32, 5, 2, 2),
    (2, 8, 8, 48, 3, 2, 1),
    (1, 6, 5, 64, 2, 2, 0),
    (2, 9, 9, 5, 4, 3, 1),
    (3, 9, 7, 5, 5, 1, 2),   # 5 candidate positions per axis
    (2, 8, 8, 4, 4, 1, 1),   # 4 per axis
]


@pytest.mark.parametrize("geom", CONV_GEOMS)
def test_conv_layer_matches_oracle(geom):
    ic, h, w, oc, k, s, p = geom
    rng = np.random.default_rng(hash(geom) % 2 ** 32)
    layer = S.ConvLayer(name="c", ic=ic, h_in=h, w_in=w, oc=oc, k=k, s=s, p=p, init_k=1.0,
                        tau=20.0, max_queue_len=64, max_out_spikes=400)
    params = make_params(layer, rng, vth=(60, 200))
    times, src, nr = make_events(rng, 5, 150, ic * h * w)
    _check_layer(layer, params, times, src, nr)


@pytest.mark.parametrize("L", [1, 3, 8])
def test_conv_queue_truncation(L):
    rng = np.random.default_rng(10 + L)
    layer = S.ConvLayer(name="c", ic=1, h_in=6, w_in=6, oc=4, k=3, s=1, p=1, init_k=1.0,
                        tau=8.0, max_queue_len=L, max_out_spikes=200)
    params = make_params(layer, rng, vth=(20, 60), f_a=6)
    times, src, nr = make_events(rng, 4, 80, 36, t_max=40)
    out = _check_layer(layer, params, times, src, nr)
    assert not np.all(out.diag.needed["max_queue_len"] <= L)


@pytest.mark.parametrize("M", [1, 2, 7, 30])
def test_conv_output_truncation(M):
    rng = np.random.default_rng(20 + M)
    layer = S.ConvLayer(name="c", ic=2, h_in=6, w_in=6, oc=8, k=3, s=2, p=1, init_k=1.0,
                        tau=8.0, max_queue_len=64, max_out_spikes=M)
    params = make_params(layer, rng, vth=(5, 30), f_a=6)
    times, src, nr = make_events(rng, 4, 90, 72, t_max=50)
    out = _check_layer(layer, params, times, src, nr)
    assert np.any(out.stream.n_real_events > M)


@pytest.mark.parametrize("M", [3, 60])
def test_conv_output_truncation_two_channel_groups_several_tiles(M):
    """40 channels (two 32-lane channel groups) over a 14x14 plane (several tiles): the channel
    cut of the truncated samples counts each group's spike words at channel g * 32 + bit."""
    rng = np.random.default_rng(25 + M)
    layer = S.ConvLayer(name="c", ic=2, h_in=14, w_in=14, oc=40, k=3, s=1, p=1, init_k=1.0,
                        tau=8.0, max_queue_len=64, max_out_spikes=M)
    params = make_params(layer, rng, vth=(5, 30), f_a=6)
    times, src, nr = make_events(rng, 3, 120, 2 * 14 * 14, t_max=60)
    out = _check_layer(layer, params, times, src, nr)
    assert np.any(out.stream.n_real_events > M)


def test_conv_many_tiles():
    """A 64x200 output plane with rows of 13000 events (no fewer than its 12800 positions, so
    64-position tiles): 208 tiles of 16x4 positions, whose partition needs more than the default
    48 KB of shared memory per block."""
    rng = np.random.default_rng(27)
    layer = S.ConvLayer(name="c", ic=1, h_in=64, w_in=200, oc=4, k=3, s=1, p=1, init_k=1.0,
                        tau=8.0, max_queue_len=64, max_out_spikes=20000)
    params = make_params(layer, rng, vth=(5, 30), f_a=6)
    times, src, nr = make_events(rng, 2, 13000, 64 * 200, t_max=2000)
    _check_layer(layer, params, times, src, nr)


@pytest.mark.parametrize("ic,h,w", [(8, 64, 64), (2, 1, 400)])
def test_conv_sparse_input_takes_large_tiles(ic, h, w):
    """Input rows shorter than the output plane: the layer is planned with tiles of up to 256
    positions (32x32 plane: four 16x16 tiles; 1x200 plane: one tile 200 positions wide)."""
    rng = np.random.default_rng(28 + h)
    layer = S.ConvLayer(name="c", ic=ic, h_in=h, w_in=w, oc=24, k=3, s=2, p=1, init_k=1.0,
                        tau=8.0, max_queue_len=16, max_out_spikes=400)
    params = make_params(layer, rng, vth=(3, 20), f_a=6)
    times, src, nr = make_events(rng, 6, 40, ic * h * w, t_max=100)
    _check_layer(layer, params, times, src, nr)


@pytest.mark.parametrize("vth", [(-20, 0), (-5, 5)])
def test_conv_tail_columns_fire_when_threshold_not_positive(vth):
    rng = np.random.default_rng(30)
    for M in (500, 9):
        layer = S.ConvLayer(name="c", ic=1, h_in=5, w_in=5, oc=3, k=3, s=2, p=1, init_k=1.0,
                            tau=8.0, max_queue_len=12, max_out_spikes=M)
        params = make_params(layer, rng, vth=vth, f_a=6, per_neuron_vth=True)
        times, src, nr = make_events(rng, 3, 20, 25, t_max=30)
        _check_layer(layer, params, times, src, nr)


@pytest.mark.parametrize("overflow,round_mode", [("saturate", "round"), ("wrap", "truncate"),
                                                 ("saturate", "truncate")])
def test_conv_narrow_register_modes(overflow, round_mode):
    rng = np.random.default_rng(40)
    layer = S.ConvLayer(name="c", ic=2, h_in=8, w_in=8, oc=16, k=3, s=2, p=1, init_k=1.0,
                        tau=20.0, max_queue_len=64, max_out_spikes=300)
    params = make_params(layer, rng, vth=(100, 250), f_a=8, f_V=2, i_V=8, overflow=overflow)
    times, src, nr = make_events(rng, 4, 200, 128)
    out = _check_layer(layer, params, times, src, nr, round_mode=round_mode)
    assert np.any(out.result.overflowed)


@pytest.mark.parametrize("overflow,round_mode,fires", [
    ("saturate", "round", True), ("wrap", "truncate", True), ("saturate", "truncate", False),
    ("wrap", "round", False)])
def test_fc_narrow_register_modes(overflow, round_mode, fires):
    rng = np.random.default_rng(41)
    layer = S.FCLayer(name="f", n_in=96, n_out=40, init_k=1.0, tau=20.0, max_out_spikes=500)
    params = make_params(layer, rng, vth=(100, 250), f_a=8, f_V=2, i_V=8, overflow=overflow,
                         fires=fires)
    times, src, nr = make_events(rng, 4, 200, 96)
    out = _check_layer(layer, params, times, src, nr, round_mode=round_mode)
    assert np.any(out.result.overflowed)


def test_conv_empty_and_overfull_inputs():
    rng = np.random.default_rng(50)
    layer = S.ConvLayer(name="c", ic=2, h_in=6, w_in=6, oc=4, k=3, s=2, p=0, init_k=1.0,
                        tau=20.0, max_queue_len=32, max_out_spikes=50)
    params = make_params(layer, rng, vth=(40, 90))
    nr = np.array([0, 40, 1000, 7], np.int32)   # n_real may exceed the stream length
    times, src, _ = make_events(rng, 4, 40, 72, n_real=np.minimum(nr, 40), pad_time="big")
    _check_layer(layer, params, times, src, nr)


def test_conv_multi_tile_plane():
    rng = np.random.default_rng(60)
    layer = S.ConvLayer(name="c", ic=2, h_in=70, w_in=66, oc=32, k=3, s=2, p=1, init_k=1.0,
                        tau=20.0, max_queue_len=48, max_out_spikes=3000)
    params = make_params(layer, rng, vth=(60, 160))
    times, src, nr = make_events(rng, 3, 3000, 2 * 70 * 66)
    _check_layer(layer, params, times, src, nr)


def test_conv_out_of_range_sources_clamp_like_jax():
    rng = np.random.default_rng(70)
    layer = S.ConvLayer(name="c", ic=2, h_in=5, w_in=5, oc=4, k=3, s=1, p=1, init_k=1.0,
                        tau=20.0, max_queue_len=32, max_out_spikes=100)
    params = make_params(layer, rng, vth=(30, 60))
    times, src, nr = make_events(rng, 2, 30, 50)
    src[0, ::3] += 50           # channel index beyond ic
    src[1, ::4] -= 60           # negative flat index
    _check_layer(layer, params, times, src, nr)


@pytest.mark.parametrize("n_out,fires", [(128, True), (10, False), (45, True), (33, False)])
def test_fc_layer_matches_oracle(n_out, fires):
    rng = np.random.default_rng(80 + n_out)
    layer = S.FCLayer(name="f", n_in=200, n_out=n_out, init_k=1.0, tau=20.0, max_out_spikes=500)
    params = make_params(layer, rng, vth=(100, 300), fires=fires)
    times, src, nr = make_events(rng, 4, 300, 200)
    _check_layer(layer, params, times, src, nr)


@pytest.mark.parametrize("n_out,fires,batch", [(3, True, 7), (8, True, 5), (16, True, 9),
                                               (12, False, 3), (16, False, 1), (9, True, 11)])
def test_fc_packed_narrow_layers(n_out, fires, batch):
    """Layers of at most 16 neurons run several samples per warp: odd batch sizes leave a warp
    partly empty, and ragged n_real gives the packed samples different lengths."""
    rng = np.random.default_rng(130 + n_out + batch)
    layer = S.FCLayer(name="f", n_in=64, n_out=n_out, init_k=1.0, tau=20.0, max_out_spikes=400)
    params = make_params(layer, rng, vth=(60, 200), fires=fires)
    nr = rng.integers(0, 250, size=batch).astype(np.int32)
    nr[0] = 250
    times, src, _ = make_events(rng, batch, 250, 64, n_real=nr)
    _check_layer(layer, params, times, src, nr)


@pytest.mark.parametrize("n_in,n_out,q_max", [(2312, 128, 127), (4000, 40, 3000)])
def test_fc_wide_inputs(n_in, n_out, q_max):
    """Weight tables past the shared-memory stage (int16 codes over 4000 inputs, read from global
    memory) and configuration 1's 2312x128 layer (int8 codes staged per neuron group)."""
    rng = np.random.default_rng(140 + n_out)
    layer = S.FCLayer(name="f", n_in=n_in, n_out=n_out, init_k=1.0, tau=20.0, max_out_spikes=900)
    params = make_params(layer, rng, vth=(300, 900), q_max=q_max)
    times, src, nr = make_events(rng, 3, 400, n_in)
    _check_layer(layer, params, times, src, nr)


@pytest.mark.parametrize("M", [1, 5, 40])
def test_fc_output_truncation(M):
    rng = np.random.default_rng(90 + M)
    layer = S.FCLayer(name="f", n_in=50, n_out=40, init_k=1.0, tau=20.0, max_out_spikes=M)
    params = make_params(layer, rng, vth=(20, 60), f_a=8)
    times, src, nr = make_events(rng, 3, 120, 50)
    out = _check_layer(layer, params, times, src, nr)
    assert np.any(out.stream.n_real_events > M)


def test_fc_tail_pads_fire_with_nonpositive_threshold():
    rng = np.random.default_rng(100)
    for M in (400, 13):
        layer = S.FCLayer(name="f", n_in=30, n_out=6, init_k=1.0, tau=10.0, max_out_spikes=M)
        params = make_params(layer, rng, vth=(-10, 2), f_a=6, per_neuron_vth=True)
        times, src, nr = make_events(rng, 3, 40, 30, pad_time="big")
        _check_layer(layer, params, times, src, nr)


def test_dense_scan_matches_oracle_run_layer():
    rng = np.random.default_rng(110)
    n, L = 300, 70
    a = rng.integers(0, 1024, size=(n, L)).astype(np.int32)
    ident = rng.random((n, L)) < 0.3
    q = rng.integers(-127, 128, size=(n, L)).astype(np.int32)
    vth = rng.integers(50, 200, size=n).astype(np.int32)
    for overflow in ("wrap", "saturate"):
        got = S.QuantB200Backend().scan_dense(a, ident, q, vth, f_a=10, f_V=1, i_V=9,
                                             overflow_mode=overflow)
        ref = O.run_layer(a, ident, q, vth, f_a=10, f_V=1, i_V=9, overflow_mode=overflow)
        np.testing.assert_array_equal(got.v_final, ref.v_final)
        np.testing.assert_array_equal(got.spike_mask, ref.spike_mask)
        np.testing.assert_array_equal(got.overflowed, ref.overflowed)
        np.testing.assert_array_equal(got.v_unfitted_min, ref.v_unfitted_min)
        np.testing.assert_array_equal(got.v_unfitted_max, ref.v_unfitted_max)


def _small_net(rng):
    net = S.Network.build((2, 8, 8), [
        S.conv(4, k=3, s=1, p=1, init_k=5.0, max_queue_len=40, max_out_spikes=512, tau=16.0),
        S.conv(4, k=3, s=2, p=1, init_k=5.0, max_queue_len=128, max_out_spikes=256, tau=16.0),
        S.fc(10, init_k=5.0, v_th=1e9, max_out_spikes=8, tau=16.0)])
    params = [make_params(l, rng, vth=(40, 90), f_a=8, f_V=2, i_V=16, tau=16.0,
                          fires=i < 2) for i, l in enumerate(net.layers)]
    return net, params


def test_network_chain_matches_oracle_layer_by_layer():
    rng = np.random.default_rng(120)
    net, params = _small_net(rng)
    times, src, nr = make_events(rng, 6, 40, 128, t_max=30)
    raw = S.InputEvents.checked(times, src, nr)
    out = net.apply_batched(params, raw, keep_streams=True)
    for b in range(6):
        refs = O.network_forward(net.layers, params, times[b], src[b], nr[b])
        for li, ref in enumerate(refs):
            np.testing.assert_array_equal(out.results[li].v_final[b], ref.v_final)
            assert int(out.results[li].spike_count[b]) == ref.spike_count
            np.testing.assert_array_equal(out.streams[li].event_source_idx[b],
                                          ref.event_source_idx)
            np.testing.assert_array_equal(out.streams[li].event_times[b], ref.event_times)
        assert bool(out.fits[b]) == all(r.fits for r in refs)


def test_network_plan_matches_layerwise_run():
    rng = np.random.default_rng(130)
    net, params = _small_net(rng)
    times, src, nr = make_events(rng, 9, 40, 128, t_max=30)
    raw = S.InputEvents.checked(times, src, nr)
    ref = net.apply_batched(params, raw)
    plan = S.QuantB200Backend().compile(net.layers, params, batch=9, in_capacity=40)
    logits, spikes, fits = plan(raw)
    np.testing.assert_array_equal(logits, ref.last.v_final)
    np.testing.assert_array_equal(spikes, np.stack([r.spike_count for r in ref.results], 1))
    np.testing.assert_array_equal(fits, ref.fits)
    assert plan.last_launch_count() > 0
