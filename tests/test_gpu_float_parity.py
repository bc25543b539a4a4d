"""GPU parity of the float FC layer (salt_float_fc_layer_forward) against the float oracle (the
chunk-by-chunk restatement of salt_core/float) and the reference's own known answers.

Tolerance (the north star's): v_final within 1e-5 relative (1e-6 absolute near 0), and identical
spike sets except where a value lies within +-1e-6 * v_th of the threshold.  The kernel runs
each chunk's events in order with fused multiply-adds where the reference composes the chunk's
maps in associative-scan order, so float32 rounding may flip a fire decision only there: a
neuron's spikes may differ from the oracle's only at or after an event whose exact (float64)
value came within the band (oracle.float_seq64), and such a neuron's later values are not
compared; every other neuron's v_final is.  There is no cap on their number: the band alone
decides.  needed max_extra_steps may differ by one where sum(b+)/v_th sits on an integer (the
reference sums in float32 in XLA's order)."""
import json
import os

import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from test_oracle_known_answers import check_float_result, float_layer_from_case

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "known_answers.json")))


@pytest.mark.parametrize("c", [c for c in CASES if c["kind"] == "float_fc_layer"],
                         ids=lambda c: c["source"])
def test_float_known_answers_on_gpu(c):
    layer = float_layer_from_case(c)
    stream = S.EventStream(np.array(c["times"], np.float32), np.array(c["src"], np.int32),
                           np.ones(len(c["times"]), np.float32), np.int32(c["n_real"]))
    out = S.FloatB200Backend().forward_layer(layer, np.array(c["w"], np.float32), stream)
    fits = bool(layer.capacity.fits(out.diag))
    check_float_result(c, out.result.v_final, int(out.result.spike_count),
                       int(out.stream.n_real_events), out.stream.event_times,
                       out.stream.event_source_idx,
                       int(out.diag.needed["max_extra_steps"]), fits)


def _batch(seed, B, n_in, n_out, E, chunk, extra, t_max, w_sd, M=None, tau=20.0, gain=False,
           n_real=None, per_neuron_tau=False, silent=0):
    rng = np.random.default_rng(seed)
    layer = S.FCLayer(name="f", n_in=n_in, n_out=n_out, init_k=1.0, tau=tau, v_th=1.0,
                      chunk_size=chunk, max_out_spikes=M or 4 * E, max_extra_steps=extra)
    w = rng.normal(0.0, w_sd, (n_out, n_in)).astype(np.float32)
    w[:silent] = -np.abs(w[:silent])  # inhibited neurons: never fire
    t = np.sort(rng.integers(0, t_max, (B, E)), axis=1).astype(np.float32)
    s = rng.integers(0, n_in, (B, E)).astype(np.int32)
    nr = (rng.integers(E // 2, E + 1, B) if n_real is None else np.asarray(n_real)).astype(np.int32)
    g = rng.uniform(0.5, 1.5, (B, E)).astype(np.float32) if gain else np.ones((B, E), np.float32)
    taus = rng.uniform(5.0, 50.0, n_out) if per_neuron_tau else None
    return layer, w, t, s, nr, g, taus


BAND = 1e-6          # spike decisions may differ only within +-BAND * v_th of the threshold
RTOL, ATOL = 1e-5, 1e-6


def _ref_spike_times(ref, o, t):
    if ref.spike_mask is not None:
        return [float(t[j]) for j in ref.spike_event_idx[o][ref.spike_mask[o]]]
    k = min(ref.n_real_events, ref.event_times.shape[0])
    return sorted(float(x) for x in ref.event_times[:k][ref.event_source_idx[:k] == o])


def _check_against_oracle(layer, w, t, s, nr, g, taus, out, dense=True, threads=1):
    gain_used = not np.all(g == 1.0)
    for b in range(t.shape[0]):
        gb = g[b] if gain_used else None
        ref = O.float_fc_forward(layer, w, t[b], s[b], int(nr[b]), gain=gb, tau=taus,
                                 dense=dense, threads=threads)
        _, first_near = O.float_seq64(layer, w, t[b], s[b], int(nr[b]), gain=gb, tau=taus,
                                      near=BAND)
        E = len(t[b])
        vf = np.asarray(out.result.v_final[b])
        S_gpu = int(out.result.spike_count[b])
        k = min(S_gpu, layer.max_out_spikes)
        times = out.stream.event_times[b][:k]
        src = out.stream.event_source_idx[b][:k]
        complete = S_gpu <= layer.max_out_spikes  # the stream holds every spike
        if not dense:
            assert ref.n_real_events <= layer.max_out_spikes, "oracle stream must be complete"
        diverged = 0
        for o in range(layer.n_out):
            ref_t = _ref_spike_times(ref, o, t[b])
            if complete:
                got_t = sorted(float(x) for x in times[src == o])
                if got_t != ref_t:
                    i = next(i for i in range(min(len(got_t), len(ref_t)) + 1)
                             if i == min(len(got_t), len(ref_t)) or got_t[i] != ref_t[i])
                    t_diff = min(got_t[i] if i < len(got_t) else np.inf,
                                 ref_t[i] if i < len(ref_t) else np.inf)
                    assert first_near[o] < E and t[b][first_near[o]] <= t_diff, \
                        f"b={b} neuron {o}: spikes differ at t={t_diff} with no value within " \
                        f"{BAND} of v_th before it"
                    diverged += 1
                    continue
            elif first_near[o] < E:
                continue   # truncated stream: a flipped decision here cannot be told apart
            np.testing.assert_allclose(vf[o], ref.v_final[o], rtol=RTOL, atol=ATOL,
                                       err_msg=f"v_final b={b} neuron {o}")
        if diverged == 0 and (complete or np.all(first_near == E)):
            assert S_gpu == ref.n_real_events, f"spike count b={b}"
            np.testing.assert_array_equal(src, ref.event_source_idx[:k], err_msg=f"src b={b}")
            np.testing.assert_array_equal(times, ref.event_times[:k], err_msg=f"times b={b}")
        assert abs(int(out.diag.needed["max_extra_steps"][b]) - ref.extra_steps_needed) <= 1
    return diverged


PARITY = [
    # (id, kwargs)
    ("chunk1", dict(seed=11, B=3, n_in=48, n_out=40, E=600, chunk=1, extra=0, t_max=200,
                    w_sd=0.3)),
    ("chunk64_safe", dict(seed=12, B=3, n_in=48, n_out=64, E=1500, chunk=64, extra=1500,
                          t_max=300, w_sd=0.3)),
    ("chunk16_cut", dict(seed=13, B=2, n_in=32, n_out=33, E=800, chunk=16, extra=4, t_max=150,
                         w_sd=0.4)),
    ("gain", dict(seed=14, B=2, n_in=32, n_out=70, E=900, chunk=8, extra=900, t_max=120,
                  w_sd=0.3, gain=True)),
    ("tau_per_neuron", dict(seed=15, B=2, n_in=64, n_out=96, E=1200, chunk=32, extra=1200,
                            t_max=400, w_sd=0.25, per_neuron_tau=True)),
    ("truncated_out", dict(seed=16, B=2, n_in=16, n_out=40, E=700, chunk=4, extra=700,
                           t_max=100, w_sd=0.5, M=50)),
    ("empty_and_overfull", dict(seed=17, B=3, n_in=16, n_out=20, E=400, chunk=8, extra=400,
                                t_max=90, w_sd=0.4, n_real=[0, 400, 10 ** 6])),
    ("many_segments", dict(seed=18, B=1, n_in=64, n_out=32, E=30000, chunk=256, extra=30000,
                           t_max=6000, w_sd=0.12)),
    ("big_gaps_powf", dict(seed=19, B=2, n_in=16, n_out=24, E=500, chunk=8, extra=500,
                           t_max=20000, w_sd=0.6)),
    # segments longer than the first-fire tracking window, with neurons that never fire
    ("silent_neurons", dict(seed=20, B=1, n_in=16, n_out=40, E=40000, chunk=128, extra=40000,
                            t_max=8000, w_sd=0.15, silent=12)),
]


@pytest.mark.parametrize("kw", [k for _, k in PARITY], ids=[i for i, _ in PARITY])
def test_float_layer_matches_oracle(kw):
    layer, w, t, s, nr, g, taus = _batch(**kw)
    stream = S.EventStream(t, s, g, nr)
    out = S.FloatB200Backend().forward_layer(layer, w, stream, tau=taus)
    _check_against_oracle(layer, w, t, s, nr, g, taus, out)


def test_float_chain_matches_layer_by_layer():
    """network.py:93-122: a firing hidden FC layer feeding a non-firing readout, run as one
    device chain, equals the two layers run one after the other."""
    rng = np.random.default_rng(21)
    hidden = S.FCLayer(name="h", n_in=64, n_out=48, init_k=1.0, tau=16.0, v_th=1.0, chunk_size=16,
                       max_out_spikes=3000, max_extra_steps=2000)
    readout = S.FCLayer(name="o", n_in=48, n_out=10, init_k=1.0, tau=16.0, v_th=1e9,
                        chunk_size=64, max_out_spikes=1, max_extra_steps=0)
    w1 = rng.normal(0, 0.3, (48, 64)).astype(np.float32)
    w2 = rng.normal(0, 0.3, (10, 48)).astype(np.float32)
    t = np.sort(rng.integers(0, 300, (2, 2000)), axis=1).astype(np.float32)
    s = rng.integers(0, 64, (2, 2000)).astype(np.int32)
    nr = np.array([2000, 1500], np.int32)
    stream = S.EventStream(t, s, np.ones_like(t), nr)
    be = S.FloatB200Backend()
    net = be.run_network([hidden, readout], [w1, w2], stream, keep_streams=True)
    h = be.forward_layer(hidden, w1, stream)
    o = be.forward_layer(readout, w2, h.stream)
    np.testing.assert_array_equal(net.results[0].v_final, h.result.v_final)
    np.testing.assert_array_equal(net.last.v_final, o.result.v_final)
    assert np.all(net.results[0].spike_count > 0)
    np.testing.assert_array_equal(net.fits, h.diag.spike_count <= 3000)
    for b in range(2):  # and the readout against the oracle on the hidden layer's stream
        hs = h.stream
        ref = O.float_fc_forward(readout, w2, hs.event_times[b], hs.event_source_idx[b],
                                 int(hs.n_real_events[b]), dense=False)
        np.testing.assert_allclose(o.result.v_final[b], ref.v_final, rtol=1e-5, atol=1e-5)


def test_float_rejects_non_positive_threshold():
    layer = S.FCLayer(name="f", n_in=2, n_out=2, init_k=1.0, v_th=0.0)
    stream = S.EventStream(np.zeros(3, np.float32), np.zeros(3, np.int32),
                           np.ones(3, np.float32), np.int32(3))
    with pytest.raises(ValueError):
        S.FloatB200Backend().forward_layer(layer, np.ones((2, 2), np.float32), stream)


def test_config5_neuron_subset_full_stream():
    """Configuration 5's layer (4096 -> 4096, per-neuron tau, chunk 4096, one stream of 10^6
    events) on a 64-neuron subset over the full stream: neurons are independent, so the first 64
    neurons of the full layer see exactly what they see here."""
    from dataclasses import replace
    from salt_b200 import workloads as W
    wl = W.config5(seed=0)
    k = 64
    layer = replace(wl.layer, n_out=k, max_out_spikes=200_000)
    out = S.FloatB200Backend().forward_layer(layer, wl.w[:k], S.EventStream(
        wl.times, wl.src, np.ones_like(wl.times), wl.n_real), tau=wl.tau[:k])
    assert int(out.result.spike_count[0]) > 1000
    _check_against_oracle(layer, wl.w[:k], wl.times, wl.src, wl.n_real, np.ones_like(wl.times),
                          wl.tau[:k], out, dense=False, threads=8)
