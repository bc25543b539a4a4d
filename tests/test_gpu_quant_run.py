"""The whole-split integer forward, capacity growth and the saved-reference check on the GPU
(example/quant_run.py:71-136, example/quantize.py:306-330), against the oracle."""
import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from salt_b200 import io as sio
from salt_b200.quant_run import (check_quantized, quant_forward_split, reference_arrays,
                                 run_until_fits)
from _cases import make_events, make_params

pytestmark = pytest.mark.gpu


def _model(rng, L=64, M=400):
    net = S.Network.build((2, 10, 10), [
        S.conv(8, k=3, s=2, p=1, init_k=5.0, tau=20.0, max_queue_len=L, max_out_spikes=M),
        S.conv(16, k=3, s=1, p=1, init_k=5.0, tau=20.0, max_queue_len=L, max_out_spikes=M),
        S.fc(5, init_k=5.0, tau=20.0, v_th=1e9, max_out_spikes=1)])
    params = [make_params(l, rng, vth=(50, 120), fires=i < 2) for i, l in enumerate(net.layers)]
    return net, params


def test_split_forward_matches_the_oracle_and_the_saved_reference(tmp_path):
    rng = np.random.default_rng(31)
    net, params = _model(rng)
    times, src, nr = make_events(rng, 11, 250, 200)
    raw = S.InputEvents.checked(times, src, nr)
    out = quant_forward_split(net, params, "round", raw, batch_size=4)
    vf, sc, fits = O.network_batch(net.layers, params, times, src, nr)
    np.testing.assert_array_equal(out.v_final_int, vf)
    np.testing.assert_array_equal(out.spike_count, sc)
    np.testing.assert_array_equal(~out.truncated.any(axis=1), fits)
    scores = vf.astype(np.float32) * np.float32(2.0 ** -params[-1].f_V) * np.float32(1.0)
    np.testing.assert_array_equal(out.preds, np.argmax(scores, axis=1))
    # save model + reference, then check: identical; a planted difference is found
    sio.save_quantized(tmp_path / "model.npz", net, params, "round", {"batch_size": 4})
    np.savez(tmp_path / "reference.npz", **reference_arrays(out))
    rc, diffs = check_quantized(tmp_path / "model.npz", tmp_path / "reference.npz", raw)
    assert rc == 0 and all(len(v) == 0 for v in diffs.values())
    ref = reference_arrays(out)
    ref["spike_count"] = ref["spike_count"].copy()
    ref["spike_count"][6, 1] += 1
    np.savez(tmp_path / "reference_bad.npz", **ref)
    rc, diffs = check_quantized(tmp_path / "model.npz", tmp_path / "reference_bad.npz", raw)
    assert rc == 1 and list(diffs["spike_count"]) == [6]


def test_run_until_fits_grows_tight_capacities_to_the_roomy_result():
    rng = np.random.default_rng(32)
    tight, params = _model(rng, L=4, M=8)
    roomy = tight.replace_layers([l.with_capacity(l.capacity.replace(
        **({"max_queue_len": 4096} if hasattr(l, "max_queue_len") else {}),
        max_out_spikes=8192 if l.n_neurons > 5 else 1)) for l in tight.layers])
    times, src, nr = make_events(rng, 6, 300, 200)
    raw = S.InputEvents.checked(times, src, nr)
    grown, out, n = run_until_fits(tight, params, "round", raw, batch_size=3)
    assert n >= 1 and not out.truncated.any()
    ref = quant_forward_split(roomy, params, "round", raw, batch_size=6)
    np.testing.assert_array_equal(out.v_final_int, ref.v_final_int)
    np.testing.assert_array_equal(out.spike_count, ref.spike_count)
    for l in grown.layers[:2]:
        assert l.max_queue_len > 4 and l.max_out_spikes > 8
