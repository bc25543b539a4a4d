"""The float oracle (chunk-by-chunk associative-scan restatement of salt_core/float) against an
independent float64 sequential restatement: the chunked scan with its step limit equals the
event-by-event recurrence with chunk step accounting, up to float32 rounding (neurons whose
values came within rounding distance of v_th are set apart)."""
import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from _float_ref import sequential_float64


def _case(seed, n_in, n_out, E, chunk, extra, t_max, w_sd, n_real=None, tau=20.0, gain=False):
    rng = np.random.default_rng(seed)
    layer = S.FCLayer(name="f", n_in=n_in, n_out=n_out, init_k=1.0, tau=tau, v_th=1.0,
                      chunk_size=chunk, max_out_spikes=4 * E, max_extra_steps=extra)
    w = rng.normal(0.0, w_sd, (n_out, n_in)).astype(np.float32)
    t = np.sort(rng.integers(0, t_max, E)).astype(np.float32)
    s = rng.integers(0, n_in, E).astype(np.int32)
    g = rng.uniform(0.5, 1.5, E).astype(np.float32) if gain else None
    return layer, w, t, s, (E if n_real is None else n_real), g


CASES = [dict(seed=1, n_in=16, n_out=24, E=300, chunk=1, extra=0, t_max=100, w_sd=0.4),
         dict(seed=2, n_in=16, n_out=24, E=300, chunk=8, extra=300, t_max=100, w_sd=0.4),
         dict(seed=3, n_in=16, n_out=24, E=300, chunk=8, extra=3, t_max=100, w_sd=0.4),
         dict(seed=4, n_in=8, n_out=40, E=250, chunk=32, extra=0, t_max=60, w_sd=0.3, gain=True),
         dict(seed=5, n_in=8, n_out=16, E=250, chunk=5, extra=10, t_max=400, w_sd=0.5,
              n_real=180),
         dict(seed=6, n_in=8, n_out=16, E=250, chunk=16, extra=0, t_max=30, w_sd=0.2, tau=4.0)]


@pytest.mark.parametrize("kw", CASES, ids=lambda k: f"seed{k['seed']}")
def test_chunked_oracle_equals_sequential_float64(kw):
    layer, w, t, s, nr, g = _case(**kw)
    r = O.float_fc_forward(layer, w, t, s, nr, gain=g)
    v64, spikes, gap, _ = sequential_float64(layer, w, t, s, nr, gain=g)
    clean = gap > 1e-4
    assert clean.mean() > 0.8
    np.testing.assert_allclose(r.v_final[clean], v64[clean], rtol=1e-4, atol=1e-4)
    for o in np.nonzero(clean)[0]:
        got = list(r.spike_event_idx[o][r.spike_mask[o]])
        assert got == spikes[o], f"neuron {o}"
    if clean.all():
        assert r.n_real_events == sum(len(x) for x in spikes)
