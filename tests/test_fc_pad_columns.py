"""Pad columns of an FC layer are identity steps whose unfitted value is the register
(salt_core/quant/scan.py:40-42 with connectivity/fc.py:26-29 masking pads to Δt = 0, q = 0):
after a last real event that wrapped, the pads put the wrapped register into the sample's
unfitted range.  The oracle shows it on the CPU; the GPU layer must agree."""
import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from _cases import stream_of


def _case(fires):
    layer = S.FCLayer(name="f", n_in=4, n_out=3, init_k=1.0, tau=20.0, max_out_spikes=16)
    q = np.full(layer.weight_shape, 120, np.int32)
    vth = np.full(layer.n_neurons, 127, np.int32) if fires else None
    params = S.QuantizedLayerParams(q=q, decay_table_int=S.build_decay_table_int(10, 20.0),
                                    v_th_int=vth, scale=np.float32(1.0), f_a=10, f_V=0, i_V=8,
                                    overflow_mode="wrap")
    # two events at one time: V = 120, then 240 wraps to -16 (8-bit register); row 1 has no pads
    times = np.array([[5, 5, 0, 0], [5, 5, 5, 5]], np.float32)
    src = np.zeros((2, 4), np.int32)
    nr = np.array([2, 4], np.int32)
    return layer, params, times, src, nr


@pytest.mark.parametrize("fires", [False, True])
def test_oracle_pad_columns_see_the_wrapped_register(fires):
    layer, params, times, src, nr = _case(fires)
    ref = O.fc_forward(layer, params, times[0], src[0], 2, "round")
    assert ref.any_overflow
    assert ref.vmin_all == -16 and ref.vmax_all == 240
    full = O.fc_forward(layer, params, times[1], src[1], 4, "round")
    # no pads: 120, 240 -> -16, 104, 224 -> -32; the extremes come from real events only
    assert full.vmax_all == 240 and full.vmin_all == 0


@pytest.mark.gpu
@pytest.mark.parametrize("fires", [False, True])
def test_gpu_pad_columns_see_the_wrapped_register(fires):
    layer, params, times, src, nr = _case(fires)
    out = S.QuantB200Backend("round").forward_layer(layer, params, stream_of(times, src, nr))
    for b in range(2):
        ref = O.fc_forward(layer, params, times[b], src[b], int(nr[b]), "round")
        assert int(out.result.v_unfitted_min[b]) == ref.vmin_all
        assert int(out.result.v_unfitted_max[b]) == ref.vmax_all
        np.testing.assert_array_equal(out.result.v_final[b], ref.v_final)
