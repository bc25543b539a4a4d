"""Per-column traces (trace=True) and overflow forensics on the GPU against the oracle:
run_layer_traced's v_steps, the spike mask, event_ms (quant/scan.py:83-94, trace.py:25-55), and
the first-overflow records that example/quant_run.py's overflow analysis reports."""
import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from salt_b200.quant_run import (headroom_bits, min_extra_bits, overflow_events,
                                 quant_forward_split)
from _cases import make_events, make_params, stream_of

pytestmark = pytest.mark.gpu

LAYERS = {
    "conv": lambda: S.ConvLayer(name="c", ic=2, h_in=8, w_in=8, oc=16, k=3, s=2, p=1, init_k=1.0,
                                tau=20.0, max_queue_len=24, max_out_spikes=500),
    "conv_k5": lambda: S.ConvLayer(name="c", ic=3, h_in=9, w_in=7, oc=5, k=5, s=1, p=2,
                                   init_k=1.0, tau=20.0, max_queue_len=40, max_out_spikes=900),
    "fc": lambda: S.FCLayer(name="f", n_in=96, n_out=20, init_k=1.0, tau=20.0, max_out_spikes=900),
}


def _same_nan(a, b):
    np.testing.assert_array_equal(np.isnan(a), np.isnan(b))
    np.testing.assert_array_equal(np.nan_to_num(a, nan=-1.0), np.nan_to_num(b, nan=-1.0))


@pytest.mark.parametrize("kind", list(LAYERS))
@pytest.mark.parametrize("mode", ["plain", "narrow_saturate", "tails"])
def test_layer_trace_matches_oracle(kind, mode):
    rng = np.random.default_rng(hash((kind, mode)) % 2 ** 32)
    layer = LAYERS[kind]()
    n_addr = layer.ic * layer.h_in * layer.w_in if kind != "fc" else layer.n_in
    kw = dict(vth=(60, 200))
    if mode == "narrow_saturate":
        kw.update(f_a=8, f_V=2, i_V=8, overflow="saturate", vth=(100, 250))
    if mode == "tails":
        kw.update(vth=(-20, 40))
    params = make_params(layer, rng, **kw)
    nr = np.array([0, 60, 200, 10 ** 6])
    times, src, _ = make_events(rng, 4, 200, n_addr, n_real=np.minimum(nr, 200))
    out = S.QuantB200Backend().forward_layer(layer, params, stream_of(times, src, nr), trace=True)
    fwd = O.conv_forward if kind != "fc" else O.fc_forward
    for b in range(4):
        ref = fwd(layer, params, times[b], src[b], int(nr[b]), trace=True)
        np.testing.assert_array_equal(out.trace.v_steps[b], ref.v_steps, err_msg=f"b={b}")
        np.testing.assert_array_equal(out.trace.spike_mask[b], ref.spike_mask)
        _same_nan(out.trace.event_ms[b], ref.event_ms)
        np.testing.assert_array_equal(out.trace.v_steps[b][:, -1], out.result.v_final[b])


def test_network_trace_equals_layer_traces():
    rng = np.random.default_rng(3)
    net = S.Network.build((2, 8, 8), [
        S.conv(4, k=3, s=1, p=1, init_k=5.0, max_queue_len=40, max_out_spikes=512),
        S.conv(4, k=3, s=2, p=1, init_k=5.0, max_queue_len=128, max_out_spikes=256),
        S.fc(6, init_k=5.0, v_th=1e9, max_out_spikes=1)])
    params = [make_params(l, rng, vth=(40, 90), f_a=8, fires=i < 2)
              for i, l in enumerate(net.layers)]
    times, src, nr = make_events(rng, 3, 60, 128, t_max=30)
    out = net.apply_batched(params, S.InputEvents.checked(times, src, nr), trace=True,
                            keep_streams=True)
    for b in range(3):
        refs = O.network_forward(net.layers, params, times[b], src[b], nr[b])
        t, s, n = times[b], src[b], int(nr[b])
        for li, layer in enumerate(net.layers):
            fwd = O.conv_forward if O.is_conv(layer) else O.fc_forward
            ref = fwd(layer, params[li], t, s, n, trace=True)
            np.testing.assert_array_equal(out.traces[li].v_steps[b], ref.v_steps)
            t, s, n = refs[li].event_times, refs[li].event_source_idx, refs[li].n_real_events


def test_overflow_forensics_match_the_oracle_traces():
    rng = np.random.default_rng(5)
    net = S.Network.build((2, 8, 8), [
        S.conv(8, k=3, s=2, p=1, init_k=5.0, max_queue_len=64, max_out_spikes=400),
        S.fc(4, init_k=5.0, v_th=1e9, max_out_spikes=1)])
    params = [make_params(l, rng, vth=(150, 300), f_a=8, f_V=2, i_V=8, fires=i == 0)
              for i, l in enumerate(net.layers)]
    times, src, nr = make_events(rng, 5, 150, 128, t_max=60)
    raw = S.InputEvents.checked(times, src, nr)
    out = quant_forward_split(net, params, "round", raw, batch_size=5)
    assert out.overflowed.any()
    hb = headroom_bits(params, out)
    assert any(h is not None and h < 0 for h in hb)
    events = overflow_events(net, params, "round", raw, out)
    assert 0 < len(events) <= 50
    for ev in events[:20]:
        b = ev["sample"]
        li = [l.name for l in net.layers].index(ev["layer"])
        layer = net.layers[li]
        if li == 0:
            t, s, n = times[b], src[b], int(nr[b])
        else:
            r0 = O.conv_forward(net.layers[0], params[0], times[b], src[b], int(nr[b]))
            t, s, n = r0.event_times, r0.event_source_idx, r0.n_real_events
        fwd = O.conv_forward if O.is_conv(layer) else O.fc_forward
        ref = fwd(layer, params[li], t, s, n, trace=True)
        shape = layer.unflatten_neurons(np.zeros(layer.n_neurons)).shape
        neuron = int(np.ravel_multi_index((ev["channel"], ev["y"], ev["x"]), shape))
        col = int(np.argmax(ref.overflowed[neuron]))
        assert ref.overflowed[neuron, col]
        assert ev["v_before"] == (int(ref.v_steps[neuron, col - 1]) if col else 0)
        assert ev["v_after"] == int(ref.v_steps[neuron, col])
        assert ev["spiked"] == bool(ref.spike_mask[neuron, col])
        assert ev["true_min"] == int(ref.v_unfitted_min[neuron])
        assert ev["true_max"] == int(ref.v_unfitted_max[neuron])
        ms = float(ref.event_ms[neuron, col])
        assert (np.isnan(ms) and np.isnan(ev["time_ms"])) or ms == ev["time_ms"]
    extra, rounds = min_extra_bits(net, params, "round", raw, 5, None, out)
    assert rounds == sum(extra) and extra[0] >= 1
    widened = [p._replace(i_V=p.i_V + e) for p, e in zip(params, extra)]
    assert not quant_forward_split(net, widened, "round", raw, 5).overflowed.any()
