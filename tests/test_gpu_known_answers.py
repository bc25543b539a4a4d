"""The reference's known-answer cases through the B200 kernels (dense scan plug-in and the fused
layer pipeline) — the same vectors that pin the oracle."""
import json
import os

import numpy as np
import pytest

import salt_b200 as S
from test_oracle_known_answers import check_layer_result, layer_from_case, params_from_case

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "known_answers.json")))


@pytest.mark.parametrize("c", [c for c in CASES if c["kind"] == "run_layer"],
                         ids=lambda c: c["source"])
def test_run_layer_on_gpu(c):
    r = S.QuantB200Backend().scan_dense(np.array(c["a"]), np.array(c["ident"]), np.array(c["q"]),
                                        np.array(c["vth"]), f_a=c["f_a"], f_V=c["f_V"],
                                        i_V=c["i_V"])
    np.testing.assert_array_equal(r.v_final, c["v_final"])
    for key in ("spike_mask", "overflowed", "v_unfitted_min", "v_unfitted_max"):
        if key in c:
            np.testing.assert_array_equal(getattr(r, key), np.array(c[key]))


@pytest.mark.parametrize("c", [c for c in CASES if c["kind"] in ("fc_layer", "conv_layer")],
                         ids=lambda c: c["source"])
def test_layer_on_gpu(c):
    layer = layer_from_case(c)
    params = params_from_case(c, layer)
    stream = S.EventStream(np.array(c["times"], np.float32), np.array(c["src"], np.int32),
                           np.ones(len(c["times"]), np.float32), np.int32(c["n_real"]))
    out = layer.forward(params, stream, backend=S.QuantB200Backend())
    fits = bool(layer.capacity.fits(out.diag))
    needed = int(out.diag.needed.get("max_queue_len", 0))
    check_layer_result(c, out.result.v_final, int(out.result.spike_count),
                       int(out.stream.n_real_events), out.stream.event_times,
                       out.stream.event_source_idx, needed, fits)
    if "readout" in c:
        np.testing.assert_allclose(S.QuantB200Backend().readout(out.result, params).v_final,
                                   c["readout"])
