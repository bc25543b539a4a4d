"""Properties of the CPU oracle that need no GPU: the split wide multiply equals exact big-integer
arithmetic (as salt_core/tests/test_fixed_point.py:101-118 checks), the C queue construction
equals an independent dense restatement (every neuron sees every event, as the reference's
salt_core/tests/_reference.py does), and the threaded batch driver agrees with the per-sample
path."""
import numpy as np
import pytest

import oracle as O
import salt_b200 as S
from _cases import make_events, make_params


def test_wide_mul_shift_equals_exact_integer_arithmetic():
    rng = np.random.default_rng(3)
    shift = 15
    for a, v in zip(rng.integers(0, 2 ** shift, 500), rng.integers(-(2 ** 29), 2 ** 29, 500)):
        exact = int(a) * int(v)
        assert O.wide_mul_shift(int(a), int(v), shift, "round") == (exact + (1 << 14)) >> shift
        assert O.wide_mul_shift(int(a), int(v), shift, "truncate") == exact >> shift


def _wrap32(x):
    return ((np.asarray(x, np.int64) + 2 ** 31) % 2 ** 32) - 2 ** 31


def test_split_decay_equals_one_wide_product_for_in_range_codes():
    """The kernels' one-multiply decay, low 32 bits of (a*V + half) >> f_a, against the
    reference's int32 split a*(V>>f_a) + ((a*(V & mask) + half) >> f_a) (fixed_point.py:47-65),
    for every f_a <= 15, decay codes in [0, 2^f_a] and register values over the whole int32
    range; out-of-range codes can make the split form's a*lo term wrap, which is why a layer with
    needs_tail keeps the split form."""
    rng = np.random.default_rng(11)
    edge_v = np.array([0, 1, -1, 2 ** 29 - 1, -(2 ** 29), 2 ** 31 - 1, -(2 ** 31)], np.int64)
    for f_a in range(16):
        for half in ({0, (1 << (f_a - 1))} if f_a else {0}):
            a = np.concatenate([rng.integers(0, 2 ** f_a + 1, 4000),
                                [0, 1, 2 ** f_a - 1, 2 ** f_a]]).astype(np.int64)
            v = np.concatenate([rng.integers(-(2 ** 31), 2 ** 31, a.size - edge_v.size), edge_v])
            lo = v & ((1 << f_a) - 1)
            split = _wrap32(_wrap32(a * (v >> f_a)) + (_wrap32(a * lo + half) >> f_a))
            wide = _wrap32((a * v + half) >> f_a)
            np.testing.assert_array_equal(split, wide)
    # a code beyond the range: the split form's inner term wraps and the two differ
    f_a, a, v = 15, 2 ** 20, 2 ** 15 - 1
    lo = v & ((1 << f_a) - 1)
    assert _wrap32(_wrap32(a * (v >> f_a)) + (_wrap32(a * lo) >> f_a)) != _wrap32((a * v) >> f_a)


def test_register_stays_in_range_when_steps_are_below_the_headroom():
    """The kernels leave the register fit out when every decay code lies in [0, 2^f_a] and a
    neuron sees fewer than 2^(i_V - q_bits) weighted steps: the unfitted value after n steps is
    within n * 2^(q_bits - 1) * 2^f_V, below half the register range.  Checked on the
    reference's integer update (split product, int32 wrap) with worst-case weights."""
    rng = np.random.default_rng(12)
    for f_a, f_V, i_V, q_bits in [(10, 0, 24, 8), (6, 2, 20, 8), (15, 0, 30, 16), (8, 3, 14, 4)]:
        half = 1 << (i_V + f_V - 1)
        n = (1 << (i_V - q_bits)) - 1
        qmax = 1 << (q_bits - 1)
        for trial in range(3):
            a = rng.integers(0, (1 << f_a) + 1, n).astype(np.int64)
            a[rng.random(n) < 0.3] = 1 << f_a                  # identity steps (dt = 0)
            sign = 1 if trial == 0 else (-1 if trial == 1 else None)
            q = (np.full(n, sign * qmax) if sign else
                 rng.choice([-qmax, qmax - 1], n)).astype(np.int64)
            v, peak = 0, 0
            rh = 1 << (f_a - 1) if f_a else 0
            for k in range(n):
                lo = v & ((1 << f_a) - 1)
                dec = int(_wrap32(_wrap32(a[k] * (v >> f_a)) + (_wrap32(a[k] * lo + rh) >> f_a)))
                u = int(_wrap32(dec + (int(q[k]) << f_V)))
                assert abs(u) <= (k + 1) * qmax * (1 << f_V)
                assert -half <= u < half
                peak = max(peak, abs(u))
                v = u                                             # no fit needed
            assert peak < half


def test_decay_step_never_grows_magnitude():
    """salt_core/tests/test_fixed_point.py:49-58"""
    rng = np.random.default_rng(0)
    for a, v in zip(rng.integers(0, 64, 2000), rng.integers(-100000, 100000, 2000)):
        for mode in ("round", "truncate"):
            assert abs(O.wide_mul_shift(int(a), int(v), 6, mode)) <= abs(int(v))


def _dense_conv_reference(layer, params, times, src, n_in):
    """Every output neuron scans every real input event; events outside its receptive field are
    skipped, the catch-up decay to the last input time is applied at the end (the reference's
    dense oracle, salt_core/tests/_reference.py:19-61, in integer form).  Returns v_final."""
    K, Sd, P = layer.k, layer.s, layer.p
    hw = layer.h_in * layer.w_in
    lut = params.decay_table_int
    v_final = np.zeros(layer.n_neurons, np.int64)
    n_eff = min(n_in, len(times))
    for oc in range(layer.oc):
        for oy in range(layer.h_out):
            for ox in range(layer.w_out):
                nid = (oc * layer.h_out + oy) * layer.w_out + ox
                v, prev, count = 0, 0.0, 0
                for j in range(n_eff):
                    c, rem = divmod(int(src[j]), hw)
                    y, x = divmod(rem, layer.w_in)
                    ky, kx = y + P - oy * Sd, x + P - ox * Sd
                    if not (0 <= ky < K and 0 <= kx < K):
                        continue
                    if count >= layer.max_queue_len:
                        count += 1
                        continue
                    dt = int(np.float32(times[j]) - np.float32(prev))
                    prev = np.float32(times[j])
                    a = 0 if dt > len(lut) else int(lut[min(max(dt - 1, 0), len(lut) - 1)])
                    r = O.process_event(v, a, dt == 0, int(params.q[oc, c, ky, kx]),
                                        int(params.v_th_int[nid]), f_a=params.f_a, f_V=params.f_V,
                                        i_V=params.i_V)
                    v = r.v_final
                    count += 1
                if count < layer.max_queue_len:
                    last = np.float32(times[n_eff - 1]) if n_eff else np.float32(0)
                    dt = int(last - np.float32(prev)) if count else 0
                    a = 0 if dt > len(lut) else int(lut[min(max(dt - 1, 0), len(lut) - 1)])
                    v = O.process_event(v, a, dt == 0, 0, int(params.v_th_int[nid]),
                                        f_a=params.f_a, f_V=params.f_V, i_V=params.i_V).v_final
                v_final[nid] = v
    return v_final


@pytest.mark.parametrize("geom", [(1, 6, 6, 2, 3, 2, 1), (2, 5, 7, 3, 3, 1, 1), (1, 7, 5, 2, 2, 2, 0)])
def test_oracle_conv_matches_dense_per_neuron_scan(geom):
    ic, h, w, oc, k, s, p = geom
    rng = np.random.default_rng(sum(geom))
    layer = S.ConvLayer(name="c", ic=ic, h_in=h, w_in=w, oc=oc, k=k, s=s, p=p, init_k=1.0,
                        tau=8.0, max_queue_len=12, max_out_spikes=500)
    params = make_params(layer, rng, vth=(30, 80), f_a=6)
    times, src, nr = make_events(rng, 3, 40, ic * h * w, t_max=60)
    for b in range(3):
        ref = _dense_conv_reference(layer, params, times[b], src[b], int(nr[b]))
        got = O.conv_forward(layer, params, times[b], src[b], int(nr[b]))
        np.testing.assert_array_equal(got.v_final, ref)


def test_threaded_batch_driver_matches_per_sample_forward():
    rng = np.random.default_rng(5)
    net = S.Network.build((2, 8, 8), [
        S.conv(4, k=3, s=1, p=1, init_k=5.0, max_queue_len=40, max_out_spikes=512),
        S.conv(4, k=3, s=2, p=1, init_k=5.0, max_queue_len=128, max_out_spikes=256),
        S.fc(10, init_k=5.0, v_th=1e9, max_out_spikes=1)])
    params = [make_params(l, rng, vth=(40, 90), f_a=8, fires=i < 2)
              for i, l in enumerate(net.layers)]
    times, src, nr = make_events(rng, 5, 40, 128, t_max=30)
    vf, sc, fits = O.network_batch(net.layers, params, times, src, nr, threads=3)
    for b in range(5):
        refs = O.network_forward(net.layers, params, times[b], src[b], nr[b])
        np.testing.assert_array_equal(vf[b], refs[-1].v_final)
        assert list(sc[b]) == [r.spike_count for r in refs]
        assert fits[b] == all(r.fits for r in refs)
