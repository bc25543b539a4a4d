"""The CPU oracle against the reference's own known-answer tests (tests/golden/known_answers.json,
transcribed from salt_core/tests/*.py and the integer-inference spec).  This pins the oracle
before it is used to check the GPU kernels."""
import json
import os

import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from salt_b200.quant import QuantizedLayerParams

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "known_answers.json")))


def _ids(kind):
    return [c for c in CASES if c["kind"] == kind]


def layer_from_case(c):
    if c["kind"] == "conv_layer":
        return S.ConvLayer(name="c", ic=c["ic"], h_in=c["h_in"], w_in=c["w_in"], oc=c["oc"],
                           k=c["k"], s=c["s"], p=c["p"], init_k=5.0, tau=c["tau"],
                           max_queue_len=c["max_queue_len"], max_out_spikes=c["max_out_spikes"])
    return S.FCLayer(name="f", n_in=c["n_in"], n_out=c["n_out"], init_k=5.0, tau=c["tau"],
                     max_out_spikes=c["max_out_spikes"])


def params_from_case(c, layer):
    q = np.ones(layer.weight_shape, np.int32) if c["q"] == "ones" else np.array(c["q"], np.int32)
    vth = None if c["vth"] is None else np.broadcast_to(
        np.array(c["vth"], np.int32), (layer.n_neurons,)).copy()
    return QuantizedLayerParams(q=q, decay_table_int=S.build_decay_table_int(c["f_a"], c["tau"]),
                                v_th_int=vth, scale=np.array(c.get("scale", 1.0), np.float32),
                                f_a=c["f_a"], f_V=c["f_V"], i_V=c["i_V"],
                                overflow_mode=c.get("overflow", "wrap"))


def check_layer_result(c, v_final, spike_count, n_real, times, src, needed_queue, fits):
    np.testing.assert_array_equal(v_final, c["v_final"]) if "v_final" in c else None
    if "spike_count" in c:
        assert spike_count == c["spike_count"]
    if "src_prefix" in c:
        k = len(c["src_prefix"])
        assert list(src[:k]) == c["src_prefix"]
        assert list(times[:k]) == c["times_prefix"]
    if "needed_queue" in c:
        assert needed_queue == c["needed_queue"]
    if "fits" in c:
        assert fits == c["fits"]


@pytest.mark.parametrize("c", _ids("round_shift"), ids=lambda c: c["source"])
def test_round_shift(c):
    assert [O.round_shift(x, c["shift"], c["mode"]) for x in c["x"]] == c["expected"]


@pytest.mark.parametrize("c", _ids("wide_mul_shift"), ids=lambda c: c["source"])
def test_wide_mul_shift(c):
    assert O.wide_mul_shift(c["a"], c["v"], c["shift"], c["mode"]) == c["expected"]


@pytest.mark.parametrize("c", _ids("fit_to_bits"), ids=lambda c: c["source"])
def test_fit_to_bits(c):
    got = [O.fit_to_bits(x, c["total"], c["mode"]) for x in c["x"]]
    assert [g[0] for g in got] == c["expected"]
    assert [g[1] for g in got] == c["overflowed"]


@pytest.mark.parametrize("c", _ids("process_event"), ids=lambda c: c["source"])
def test_process_event(c):
    r = O.process_event(c["v0"], c["a"], c["ident"], c["q"], c["vth"], f_a=c["f_a"], f_V=c["f_V"],
                        i_V=c["i_V"], round_mode=c["round"], overflow_mode=c["overflow"])
    for key, field in (("v_final", "v_final"), ("spiked", "is_spiked"),
                       ("overflowed", "overflowed"), ("v_unfitted", "v_unfitted")):
        if key in c:
            assert getattr(r, field) == c[key], key


@pytest.mark.parametrize("c", _ids("run_layer"), ids=lambda c: c["source"])
def test_run_layer(c):
    r = O.run_layer(np.array(c["a"]), np.array(c["ident"]), np.array(c["q"]), np.array(c["vth"]),
                    f_a=c["f_a"], f_V=c["f_V"], i_V=c["i_V"])
    np.testing.assert_array_equal(r.v_final, c["v_final"])
    for key in ("spike_mask", "overflowed", "v_unfitted_min", "v_unfitted_max"):
        if key in c:
            np.testing.assert_array_equal(getattr(r, key), np.array(c[key]))


@pytest.mark.parametrize("c", _ids("decay_table"), ids=lambda c: c["source"])
def test_decay_table(c):
    t = S.build_decay_table_int(c["f_a"], c["tau"])
    assert t.dtype == np.int32 and t.shape == (S.delta_t_max(c["f_a"], c["tau"]),)
    assert list(t[:len(c["prefix"])]) == c["prefix"]


@pytest.mark.parametrize("c", _ids("apply_decay"), ids=lambda c: c["source"])
def test_apply_decay(c):
    a, ident = O.apply_decay_table_int(c["delta_t"], S.build_decay_table_int(c["f_a"], c["tau"]))
    assert list(ident) == c["is_identity"]
    assert list(a[1:]) == c["a_tail"]


@pytest.mark.parametrize("c", _ids("compress"), ids=lambda c: c["source"])
def test_compress_candidates(c):
    l2g, nr = O.compress_candidates(c["n_flat"], c["j_flat"], c["n_out_spatial"],
                                    c["max_queue_len"], c["n_events"])
    for row, want in c["rows"].items():
        assert list(l2g[int(row)]) == want
    assert list(nr) == c["n_real"]


@pytest.mark.parametrize("c", _ids("delta_t_regimes"), ids=lambda c: c["source"])
def test_delta_t_regimes(c):
    dt = O.delta_t_three_regimes(c["t_gathered"], c["n_real"], c["global_last"])
    np.testing.assert_array_equal(dt, np.array(c["expected"], np.float32))


@pytest.mark.parametrize("c", _ids("extract_conv"), ids=lambda c: c["source"])
def test_extract_output_events_conv(c):
    t, s, n = O.extract_output_events(c["spike_mask"], c["spike_event_idx"], c["event_times"],
                                      c["max_total_spikes"], c["local_to_global_j"])
    assert n == c["n_real"]
    assert list(s[:n]) == c["src_prefix"]
    assert list(t[:n]) == c["times_prefix"]
    assert np.all(t[n:] > c["pad_times_above"])


@pytest.mark.parametrize("c", _ids("fc_layer") + _ids("conv_layer"), ids=lambda c: c["source"])
def test_layer(c):
    layer = layer_from_case(c)
    params = params_from_case(c, layer)
    fwd = O.conv_forward if c["kind"] == "conv_layer" else O.fc_forward
    r = fwd(layer, params, np.array(c["times"], np.float32), np.array(c["src"], np.int32),
            c["n_real"])
    check_layer_result(c, r.v_final, r.spike_count, r.n_real_events, r.event_times,
                       r.event_source_idx, r.needed_queue, r.fits)
    if "readout" in c:
        v = r.v_final.astype(np.float32) * np.float32(2.0 ** -c["f_V"]) * np.array(
            c["scale"], np.float32)
        np.testing.assert_allclose(v, c["readout"])


# ---------------------------------------------------------------- float chunked scan

def float_layer_from_case(c):
    return S.FCLayer(name="f", n_in=c["n_in"], n_out=c["n_out"], init_k=1.0, tau=c["tau"],
                     v_th=c["v_th"], chunk_size=c["chunk_size"],
                     max_out_spikes=c["max_out_spikes"], max_extra_steps=c["max_extra_steps"])


def check_float_result(c, v_final, spike_count, n_real_out, times, src, extra_needed, fits):
    """The expectations a float_fc_layer case states (the reference test's own assertions)."""
    if "v_final" in c:
        np.testing.assert_allclose(v_final, c["v_final"], rtol=0, atol=c["v_tol"])
    if "v_final_differs" in c:
        assert not np.allclose(v_final, c["v_final_differs"])
    if "spike_count" in c:
        assert spike_count == c["spike_count"]
    if "n_real_out" in c:
        assert n_real_out == c["n_real_out"]
    if "extra_steps_needed" in c:
        assert extra_needed == c["extra_steps_needed"]
    if "fits" in c:
        assert fits == c["fits"]
    if "src_prefix" in c:
        k = len(c["src_prefix"])
        assert list(src[:k]) == c["src_prefix"]
        assert list(times[:k]) == c["times_prefix"]
    if "spikes_per_neuron" in c:  # the spike times of every neuron, from the output stream
        k = min(n_real_out, len(times))
        for o, js in enumerate(c["spikes_per_neuron"]):
            got = sorted(float(t) for t, s in zip(times[:k], src[:k]) if s == o)
            assert got == sorted(c["times"][j] for j in js), f"neuron {o}"


@pytest.mark.parametrize("c", _ids("float_fc_layer"), ids=lambda c: c["source"])
def test_float_layer(c):
    layer = float_layer_from_case(c)
    r = O.float_fc_forward(layer, np.array(c["w"], np.float32), np.array(c["times"], np.float32),
                           np.array(c["src"], np.int32), c["n_real"])
    check_float_result(c, r.v_final, r.spike_count, r.n_real_events, r.event_times,
                       r.event_source_idx, r.extra_steps_needed, r.fits)
    if "spikes_per_neuron" in c:  # the reference asserts spike_event_idx per neuron directly
        for o, js in enumerate(c["spikes_per_neuron"]):
            assert list(r.spike_event_idx[o][r.spike_mask[o]]) == js


@pytest.mark.parametrize("c", _ids("affine_scan"), ids=lambda c: c["source"])
def test_affine_scan_matches_sequential_composition(c):
    a = np.float32(1.0 - 1.0 / c["tau"]) ** np.array(c["n_ms"], np.float32)
    A, B = O.affine_scan(a, np.array(c["w"], np.float32))
    v, seq = c["v0"], []
    for n, w in zip(c["n_ms"], c["w"]):
        v = v * (1.0 - 1.0 / c["tau"]) ** n + w
        seq.append(v)
    np.testing.assert_allclose(A * np.float32(c["v0"]) + B, seq, rtol=0, atol=c["tol"])
