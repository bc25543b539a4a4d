"""Seeded random layer cases shared by the parity tests (test-only helpers)."""
from __future__ import annotations

import numpy as np

import salt_b200 as S


def make_params(layer, rng, *, q_max=127, vth=(128, 512), f_a=10, f_V=0, i_V=24, tau=20.0,
                overflow="wrap", fires=True, per_neuron_vth=False):
    q = rng.integers(-q_max, q_max + 1, size=layer.weight_shape).astype(np.int32)
    lut = S.build_decay_table_int(f_a, tau)
    if not fires:
        v = None
    elif per_neuron_vth:
        v = rng.integers(vth[0], vth[1] + 1, size=layer.n_neurons).astype(np.int32)
    else:
        chans = rng.integers(vth[0], vth[1] + 1, size=layer.output_shape[0]).astype(np.int32)
        v = layer.broadcast_channels(chans)
    return S.QuantizedLayerParams(q=q, decay_table_int=lut, v_th_int=v, scale=np.float32(1.0),
                                  f_a=f_a, f_V=f_V, i_V=i_V, overflow_mode=overflow)


def make_events(rng, B, E, n_addr, *, t_max=300, n_real=None, pad_time="last"):
    """(B, E) float32 integer-ms times sorted per sample, int32 sources, n_real per sample."""
    times = np.zeros((B, E), np.float32)
    src = np.zeros((B, E), np.int32)
    nr = np.zeros(B, np.int32)
    for b in range(B):
        n = int(rng.integers(0, E + 1)) if n_real is None else int(n_real[b])
        nr[b] = n
        t = np.sort(rng.integers(0, t_max, size=E)).astype(np.float32)
        if n < E:
            if pad_time == "last":
                t[n:] = t[n - 1] if n > 0 else 0.0
            elif pad_time == "big":
                t[n:] = np.float32(1e12)
        times[b] = t
        src[b] = rng.integers(0, n_addr, size=E)
    return times, src, nr


def stream_of(times, src, nr) -> S.EventStream:
    return S.EventStream(np.asarray(times, np.float32), np.asarray(src, np.int32),
                         np.ones_like(times, dtype=np.float32), np.asarray(nr, np.int32))


def materialised(t, s, n_real, M):
    """Oracle-style stream (pads at 1e12 / 0) from the first entries."""
    t = np.array(t[:M], np.float32)
    s = np.array(s[:M], np.int32)
    k = min(int(n_real), M)
    t[k:] = np.float32(1e12)
    s[k:] = 0
    return t, s
