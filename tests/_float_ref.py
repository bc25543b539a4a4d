"""Independent float64 restatement of a float FC layer's sequential semantics (test-only).

Runs v = a*v + b with fire-and-reset at every event and the chunk step accounting of
salt_core/float/scan.py:67-116 (a step ends at a fire or after chunk_size events; after
max_steps steps the remaining events are dropped).  In float64 it serves as the exact-math
yardstick: it reports, per neuron, how close any processed value came to v_th, so that tests can
set apart the fire decisions that float32 rounding may legitimately flip: `first_near[o]` is the
first event at which neuron o's value came within `near` of v_th (len(times) if never)."""
from __future__ import annotations

import numpy as np


def sequential_float64(layer, w, times, src, n_real, gain=None, tau=None, near=1e-4):
    n_out, n_in = int(layer.n_out), int(layer.n_in)
    L = len(times)
    n_eff = min(max(int(n_real), 0), L)
    C = int(layer.chunk_size)
    max_steps = -(-L // C) + int(layer.max_extra_steps)
    vth = float(layer.v_th)
    taus = np.broadcast_to(np.asarray(layer.tau if tau is None else tau, np.float64), (n_out,))
    base = (1.0 - 1.0 / taus).astype(np.float32).astype(np.float64)
    W = np.asarray(w, np.float64).reshape(n_out, n_in)
    v = np.zeros(n_out)
    phase = np.zeros(n_out, np.int64)
    steps = np.zeros(n_out, np.int64)
    run = np.ones(n_out, bool)
    gap = np.full(n_out, np.inf)
    first_near = np.full(n_out, L, np.int64)
    spikes = [[] for _ in range(n_out)]
    tprev = np.float32(0.0)
    for j in range(n_eff):
        t = np.float32(times[j])
        dt = float(np.float32(t - tprev))
        tprev = t
        s = int(src[j])
        s = s + n_in if s < 0 else s
        s = min(max(s, 0), n_in - 1)
        b = W[:, s] * (1.0 if gain is None else float(np.float32(gain[j])))
        vn = base ** dt * v + b
        v = np.where(run, vn, v)
        d = np.abs(v - vth)
        gap = np.where(run, np.minimum(gap, d), gap)
        first_near = np.where(run & (d < near * abs(vth)) & (first_near == L), j, first_near)
        spike = run & (v >= vth)
        for o in np.nonzero(spike)[0]:
            spikes[o].append(j)
        v[spike] = 0.0
        phase[run] += 1
        end = run & (spike | (phase == C))
        steps[end] += 1
        phase[end] = 0
        run &= steps < max_steps
    return v, spikes, gap, first_near
