"""The reference's network-description and model file formats (salt_core/io.py): round trips,
the exact array keys and JSON fields, a file laid out by hand from the documented format, and the
errors on malformed files."""
import json

import numpy as np
import pytest

import salt_b200 as S
from salt_b200 import io as sio
from salt_b200.quant_run import QuantSplitOutput, check_against_reference


def _net():
    return S.Network.build((2, 12, 12), [
        S.conv(8, k=3, s=2, p=1, init_k=5.0, tau=20.0, max_queue_len=40, max_out_spikes=300),
        S.fc(10, init_k=5.0, tau=20.0, v_th=1e9, max_out_spikes=1)])


def _params(net, rng):
    out = []
    for i, l in enumerate(net.layers):
        out.append(S.QuantizedLayerParams(
            q=rng.integers(-127, 128, l.weight_shape).astype(np.int32),
            decay_table_int=S.build_decay_table_int(10, 20.0),
            v_th_int=np.full(l.n_neurons, 200, np.int32) if i == 0 else None,
            scale=np.float32(0.5), f_a=10, f_V=0, i_V=24,
            overflow_mode="saturate" if i == 0 else "wrap"))
    return out


def test_network_description_round_trip_keeps_every_field():
    net = _net()
    d = sio.network_to_dict(net)
    assert d["format"] == 1 and d["input_shape"] == [2, 12, 12]
    assert d["layers"][0]["type"] == "conv" and d["layers"][1]["type"] == "fc"
    assert set(d["layers"][0]) == {"type", "name", "ic", "h_in", "w_in", "oc", "k", "s", "p",
                                   "init_k", "tau", "v_th", "alpha", "chunk_size",
                                   "max_queue_len", "max_out_spikes", "max_extra_steps"}
    back = sio.network_from_dict(json.loads(json.dumps(d)))
    assert back == net
    with pytest.raises(ValueError):
        sio.network_from_dict({**d, "format": 2})
    with pytest.raises(ValueError):
        sio.network_from_dict({**d, "layers": [{"type": "pool"}]})


def test_quantized_model_round_trip_and_keys(tmp_path):
    net = _net()
    params = _params(net, np.random.default_rng(0))
    path = tmp_path / "model.npz"
    sio.save_quantized(path, net, params, "truncate", {"batch_size": 16, "note": "x"})
    with np.load(path) as z:
        assert set(z.files) == {"__network__", "__quant__", "conv1/q", "conv1/decay_table_int",
                                "conv1/v_th_int", "conv1/scale", "fc1/q", "fc1/decay_table_int",
                                "fc1/scale"}
        quant = json.loads(str(z["__quant__"]))
    assert quant == {"format": 1, "round_mode": "truncate",
                     "layers": {"conv1": {"f_a": 10, "f_V": 0, "i_V": 24,
                                          "overflow_mode": "saturate"},
                                "fc1": {"f_a": 10, "f_V": 0, "i_V": 24, "overflow_mode": "wrap"}},
                     "metadata": {"batch_size": 16, "note": "x"}}
    m = sio.load_quantized(path)
    assert m.network == net and m.round_mode == S.RoundMode.TRUNCATE
    assert m.metadata == {"batch_size": 16, "note": "x"}
    for a, b in zip(m.params, params):
        np.testing.assert_array_equal(a.q, b.q)
        np.testing.assert_array_equal(a.decay_table_int, b.decay_table_int)
        assert (a.v_th_int is None) == (b.v_th_int is None)
        assert (a.f_a, a.f_V, a.i_V) == (b.f_a, b.f_V, b.i_V)
        assert S.OverflowMode(a.overflow_mode) == S.OverflowMode(b.overflow_mode)


def test_a_file_laid_out_from_the_documented_format_loads(tmp_path):
    """The layout io.py:129-155 documents, written directly with numpy."""
    desc = {"format": 1, "input_shape": [4], "layers": [
        {"type": "fc", "name": "out", "n_in": 4, "n_out": 3, "init_k": 5.0, "tau": 16.0,
         "v_th": 1e9, "alpha": 2.0, "chunk_size": 1, "max_out_spikes": 1, "max_extra_steps": 0}]}
    quant = {"format": 1, "round_mode": "round",
             "layers": {"out": {"f_a": 8, "f_V": 2, "i_V": 16, "overflow_mode": "wrap"}},
             "metadata": {}}
    path = tmp_path / "m.npz"
    np.savez(path, __network__=np.asarray(json.dumps(desc)), __quant__=np.asarray(json.dumps(quant)),
             **{"out/q": np.arange(12, dtype=np.int32).reshape(3, 4),
                "out/decay_table_int": np.array([240, 225], np.int32),
                "out/scale": np.asarray(0.25, np.float32)})
    m = sio.load_quantized(path)
    assert m.network.layers[0].n_out == 3 and m.params[0].v_th_int is None
    assert m.params[0].q.shape == (3, 4) and m.params[0].f_V == 2


def test_malformed_files_are_rejected(tmp_path):
    np.savez(tmp_path / "a.npz", x=np.zeros(1))
    with pytest.raises(ValueError):
        sio.load_quantized(tmp_path / "a.npz")
    net = _net()
    sio.save_weights(tmp_path / "w.npz", net, net.init(0))
    with pytest.raises(ValueError):   # weights only: no quantisation settings
        sio.load_quantized(tmp_path / "w.npz")
    back, w = sio.load_weights(tmp_path / "w.npz")
    assert back == net and w[0].shape == net.layers[0].weight_shape
    with pytest.raises(ValueError):
        sio.save_quantized(tmp_path / "b.npz", net, _params(net, np.random.default_rng(1))[:1],
                           "round", {})


def test_check_against_reference_reports_differing_samples():
    base = QuantSplitOutput(v_final_int=np.arange(12).reshape(4, 3), preds=np.array([2, 2, 2, 2]),
                            spike_count=np.ones((4, 2), np.int32),
                            truncated=np.zeros((4, 2), bool), overflowed=np.zeros((4, 2), bool),
                            v_unfitted_min=np.zeros((4, 2)), v_unfitted_max=np.zeros((4, 2)),
                            needed={})
    ref = {k: getattr(base, k).copy() for k in ("v_final_int", "preds", "spike_count",
                                                 "truncated", "overflowed")}
    assert all(len(v) == 0 for v in check_against_reference(base, ref).values())
    ref["v_final_int"][2, 1] += 1
    ref["overflowed"][3, 0] = True
    d = check_against_reference(base, ref)
    assert list(d["v_final_int"]) == [2] and list(d["overflowed"]) == [3]
    assert len(d["preds"]) == 0
