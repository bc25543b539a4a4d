"""Split runs of a quantised network on the B200: the per-sample record, capacity growth, the
saved-reference check and the overflow analysis (what example/quant_run.py:54-240 and the check of
example/quantize.py:306-330 provide on the reference side).

Design.  A `SplitRunner` holds one native network plan (capacities are runtime sizes: changing
them re-plans buffers, nothing recompiles) and streams a split through it in fixed-size
batches.  Everything the reference records per sample comes from the plan's device statistics
with one copy per batch: the output layer's registers, and per layer the spike count, the
overflow flag, the unfitted extremes and the needed queue length.

Growth and widening re-run only the samples that need it.  A sample whose needs fit the
capacities gets the same results under any larger capacities (no queue column or output spike
of it is cut), and a sample whose registers never overflowed gets the same results with wider
registers; so growing from the needs of the overflowing samples alone, and re-running only them,
ends exactly where re-running the whole split would.
"""
from __future__ import annotations

import math
from typing import Callable, NamedTuple

import numpy as np

from .capacity import GrowthPolicy, LayerDiag, grown_to_fit
from .layers import is_conv
from .network import InputEvents, Network

REFERENCE_FIELDS = ("v_final_int", "preds", "spike_count", "truncated", "overflowed")
MAX_OVERFLOW_EVENTS = 50   # overflow_events lists at most this many entries


class QuantSplitOutput(NamedTuple):
    """Per-sample record of a split of N samples (the reference's fields)."""
    v_final_int: np.ndarray     # (N, n_out) output-layer registers
    preds: np.ndarray           # (N,)
    spike_count: np.ndarray     # (N, n_layers)
    truncated: np.ndarray       # (N, n_layers) a capacity knob was too small
    overflowed: np.ndarray      # (N, n_layers) a register overflowed
    v_unfitted_min: np.ndarray  # (N, n_layers)
    v_unfitted_max: np.ndarray  # (N, n_layers)
    needed: dict                # layer name -> knob -> (N,) needed capacity

    def rows(self, idx) -> "QuantSplitOutput":
        idx = np.asarray(idx)
        return QuantSplitOutput(*(getattr(self, f)[idx] for f in self._fields[:-1]),
                                {n: {k: v[idx] for k, v in d.items()}
                                 for n, d in self.needed.items()})

    def with_rows(self, idx, other: "QuantSplitOutput") -> "QuantSplitOutput":
        """This record with rows idx replaced by other's rows (in order)."""
        idx = np.asarray(idx)
        fields = []
        for f in self._fields[:-1]:
            a = getattr(self, f).copy()
            a[idx] = getattr(other, f)
            fields.append(a)
        needed = {}
        for n, d in self.needed.items():
            needed[n] = {}
            for k, v in d.items():
                v = v.copy()
                v[idx] = other.needed[n][k]
                needed[n][k] = v
        return QuantSplitOutput(*fields, needed)


def membrane_scores(readout_v_final: np.ndarray) -> np.ndarray:
    """MembraneRegressionDecoder (salt_core/decoder.py:35-51): the read-out potentials are the
    class scores; argmax takes the lowest index on ties."""
    return readout_v_final


def _take(raw: InputEvents, idx) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    idx = np.asarray(idx)
    return (np.asarray(raw.event_times, dtype=np.float32)[idx],
            np.asarray(raw.source_idx, dtype=np.int32)[idx],
            np.asarray(raw.n_real_events, dtype=np.int32)[idx])


class SplitRunner:
    """One network (fixed capacities) compiled for batches of `batch_size` samples of streams
    with `capacity` entries; run() records every sample of a split."""

    def __init__(self, network: Network, params, round_mode, batch_size: int, capacity: int,
                 decode: Callable[[np.ndarray], np.ndarray] = membrane_scores):
        from .plan import NetworkPlan
        self.network, self.params = network, list(params)
        self.layers = list(network.layers)
        self.batch, self.capacity = int(batch_size), int(capacity)
        self.decode = decode
        self.plan = NetworkPlan(self.layers, self.params, self.batch, self.capacity, round_mode)

    def close(self) -> None:
        self.plan.close()

    def _batch(self, times, src, n_real):
        """Device statistics of up to `batch` samples (short batches are padded with empty
        samples, whose rows are dropped)."""
        from .device import to_device
        k = times.shape[0]
        if k < self.batch:
            pad = self.batch - k
            times = np.concatenate([times, np.zeros((pad, times.shape[1]), np.float32)])
            src = np.concatenate([src, np.zeros((pad, src.shape[1]), np.int32)])
            n_real = np.concatenate([n_real, np.zeros(pad, np.int32)])
        logits, stats, _ = self.plan.forward_device(to_device(times, np.float32),
                                                    to_device(src, np.int32),
                                                    to_device(n_real, np.int32))
        return logits.numpy()[:k], stats.numpy()[:, :, :k]

    def record(self, logits: np.ndarray, stats: np.ndarray) -> QuantSplitOutput:
        """The per-sample record from the plan's outputs: stats rows are spike count, overflow,
        unfitted min, unfitted max, needed queue length, each (n_layers, N)."""
        spikes, ovf, vmin, vmax, need_q = (stats[i].T for i in range(5))
        p_last = self.params[-1]
        readout = (logits.astype(np.float32) * np.float32(2.0 ** -p_last.f_V)
                   * np.asarray(p_last.scale, dtype=np.float32))
        needed, truncated = {}, []
        for li, layer in enumerate(self.layers):
            need = {"max_out_spikes": spikes[:, li].astype(np.int32),
                    "max_extra_steps": np.zeros(len(logits), np.int32)}
            if is_conv(layer):
                need = {"max_queue_len": need_q[:, li].astype(np.int32), **need}
            needed[layer.name] = need
            cap = layer.capacity
            truncated.append(np.any([need[k] > cap[k] for k in need], axis=0))
        return QuantSplitOutput(v_final_int=logits, preds=np.argmax(self.decode(readout), axis=1),
                                spike_count=spikes.astype(np.int32),
                                truncated=np.stack(truncated, axis=1), overflowed=ovf != 0,
                                v_unfitted_min=vmin, v_unfitted_max=vmax, needed=needed)

    def run(self, raw: InputEvents, rows=None) -> QuantSplitOutput:
        n = np.asarray(raw.event_times).shape[0]
        rows = np.arange(n) if rows is None else np.asarray(rows)
        logits, stats = [], []
        for start in range(0, len(rows), self.batch):
            lg, st = self._batch(*_take(raw, rows[start:start + self.batch]))
            logits.append(lg)
            stats.append(st)
        if not logits:
            return self.record(np.zeros((0, self.layers[-1].n_neurons), np.int32),
                               np.zeros((5, len(self.layers), 0), np.int32))
        return self.record(np.concatenate(logits), np.concatenate(stats, axis=2))


def quant_forward_split(network: Network, params, round_mode, raw: InputEvents,
                        batch_size: int, *, decode=membrane_scores, rows=None
                        ) -> QuantSplitOutput:
    """Every sample of raw (or the given rows) through the integer forward, batch by batch
    (example/quant_run.py:71-103)."""
    runner = SplitRunner(network, params, round_mode, batch_size,
                         np.asarray(raw.event_times).shape[-1], decode)
    try:
        return runner.run(raw, rows)
    finally:
        runner.close()


def reference_arrays(out: QuantSplitOutput) -> dict[str, np.ndarray]:
    """The arrays a reference.npz records (example/quant_run.py:106-108)."""
    return {k: getattr(out, k) for k in REFERENCE_FIELDS}


def _peak_needs(network: Network, out: QuantSplitOutput, rows) -> list[LayerDiag]:
    return [LayerDiag(0, 0.0, {k: int(np.max(v[rows])) for k, v in out.needed[l.name].items()})
            for l in network.layers]


def grown_for_needed(layers, policies, needed: dict) -> list:
    """Layers with every knob grown to hold the largest need in `needed` (layer name -> knob ->
    per-sample needs), by each layer's GrowthPolicy (example/quant_run.py:111-119)."""
    diags = [LayerDiag(0, 0.0, {k: int(np.max(v)) for k, v in needed[l.name].items()})
             for l in layers]
    return list(grown_to_fit(layers, policies, diags))


def run_until_fits(network: Network, params, round_mode, raw: InputEvents, batch_size: int,
                   policies: dict | None = None, *, max_rounds: int = 16, out=None
                   ) -> tuple[Network, QuantSplitOutput, int]:
    """The split with capacities grown until no sample is truncated (example/quant_run.py:
    122-136).  One full pass; then, while some samples overflow a knob, the knobs grow from
    those samples' device-reported needs and only those samples run again.  Returns (the
    network that fits, the record, the number of re-runs)."""
    policies = policies or {l.name: GrowthPolicy() for l in network.layers}
    if out is None:
        out = quant_forward_split(network, params, round_mode, raw, batch_size)
    reruns = 0
    while True:
        bad = np.nonzero(out.truncated.any(axis=1))[0]
        if bad.size == 0:
            return network, out, reruns
        if reruns >= max_rounds:
            raise RuntimeError(f"capacities still overflow after {max_rounds} regrowths")
        grown = grown_to_fit(network.layers, policies, _peak_needs(network, out, bad))
        network = network.replace_layers(grown)
        out = out.with_rows(bad, quant_forward_split(network, params, round_mode, raw,
                                                     batch_size, rows=bad))
        reruns += 1


def check_against_reference(out: QuantSplitOutput, reference: dict) -> dict[str, np.ndarray]:
    """Per REFERENCE_FIELDS entry, the indices of the samples that differ from the recorded
    reference (all indices when the shapes differ) — the comparison of
    example/quantize.py:320-327."""
    diffs = {}
    for key, got in reference_arrays(out).items():
        want = np.asarray(reference[key])
        if want.shape != got.shape:
            diffs[key] = np.arange(max(len(want), len(got)))
        else:
            diffs[key] = np.flatnonzero((got != want).reshape(len(got), -1).any(axis=1))
    return diffs


def check_quantized(model_path, reference_path, raw: InputEvents, batch_size: int | None = None
                    ) -> tuple[int, dict[str, np.ndarray]]:
    """Re-runs a saved quantised model on the given samples and compares it with a saved
    reference.npz (example/quantize.py:306-330 without the dataset loader).  Returns (0 when
    every field of every sample matches, else 1; the differing sample indices per field)."""
    from .io import load_quantized
    model = load_quantized(model_path)
    with np.load(reference_path) as z:
        reference = {k: z[k] for k in z.files}
    bs = int(batch_size or model.metadata.get("batch_size", 64))
    out = quant_forward_split(model.network, model.params, model.round_mode, raw, bs)
    diffs = check_against_reference(out, reference)
    return int(any(d.size for d in diffs.values())), diffs


# ---------------------------------------------------------------- overflow analysis

def with_extra_i_V(params, extra) -> list:
    """Parameters with extra[i] more integer bits in layer i's register."""
    return [p._replace(i_V=int(p.i_V) + int(e)) for p, e in zip(params, extra)]


def headroom_bits(params, out: QuantSplitOutput) -> list[float | None]:
    """Per layer, the bits between the largest magnitude any register took before fitting and
    the register's range (negative: it overflowed); None when every value was 0
    (example/quant_run.py:144-154)."""
    lo = out.v_unfitted_min.min(axis=0).astype(np.int64)
    hi = out.v_unfitted_max.max(axis=0).astype(np.int64)
    peaks = np.maximum(-lo, hi + 1)
    return [None if peak <= 0 else round(int(p.i_V) + int(p.f_V) - 1 - math.log2(int(peak)), 3)
            for p, peak in zip(params, peaks)]


def min_extra_bits(network: Network, params, round_mode, raw: InputEvents, batch_size: int,
                   policies: dict | None, out: QuantSplitOutput
                   ) -> tuple[list[int], int]:
    """The fewest extra register bits that remove every overflow, found the reference's way
    (example/quant_run.py:157-174): one bit at a time on the most upstream layer that still
    overflows.  Only the samples that overflowed run again (with capacities regrown for them).
    Returns (extra bits per layer, rounds)."""
    extra = np.zeros(len(params), np.int64)
    rows = np.nonzero(out.overflowed.any(axis=1))[0]
    flags = out.overflowed[rows]
    rounds = 0
    while rows.size:
        extra[int(np.argmax(flags.any(axis=0)))] += 1
        rounds += 1
        sub = InputEvents(*_take(raw, rows))
        _, rerun, _ = run_until_fits(network, with_extra_i_V(params, extra), round_mode, sub,
                                     batch_size, policies)
        keep = rerun.overflowed.any(axis=1)
        rows, flags = rows[keep], rerun.overflowed[keep]
    return [int(e) for e in extra], rounds


def _neuron_position(layer, neuron: int) -> tuple[int, int, int]:
    shape = layer.unflatten_neurons(np.zeros(layer.n_neurons)).shape
    return tuple(int(v) for v in np.unravel_index(neuron, shape))


def overflow_events(network: Network, params, round_mode, raw: InputEvents,
                    out: QuantSplitOutput) -> list[dict]:
    """For each overflowing (sample, layer, neuron): its first overflowing column (time, the
    register before and after, whether it fired) and the neuron's unfitted extremes, at most
    MAX_OVERFLOW_EVENTS entries (example/quant_run.py:183-214).  Each overflowing sample runs
    once more through the trace kernels' per-neuron first-overflow records."""
    from .backend import QuantB200Backend
    from .device import DeviceStream
    backend = QuantB200Backend(round_mode)
    events = []
    for i in np.nonzero(out.overflowed.any(axis=1))[0]:
        cur = DeviceStream.from_host(network.input_stream(InputEvents(*_take(raw, [int(i)]))))
        for layer, p in zip(network.layers, params):
            tr = {k: v[0].numpy() for k, v in
                  backend.trace_layer_device(layer, p, cur, dense=False).items()}
            half = 2 ** (int(p.i_V) + int(p.f_V) - 1)
            for neuron in np.flatnonzero(tr["first_overflow"] >= 0):
                ch, y, x = _neuron_position(layer, int(neuron))
                events.append({"sample": int(i), "layer": layer.name, "channel": ch, "y": y,
                               "x": x, "time_ms": float(tr["time_ms"][neuron]),
                               "v_before": int(tr["v_before"][neuron]),
                               "v_after": int(tr["v_after"][neuron]),
                               "spiked": bool(tr["spiked"][neuron]),
                               "true_min": int(tr["v_min"][neuron]),
                               "true_max": int(tr["v_max"][neuron]),
                               "register_range": [-half, half - 1]})
                if len(events) >= MAX_OVERFLOW_EVENTS:
                    return events
            cur = backend.forward_layer_device(layer, p, cur).out
    return events


def overflow_summary(network: Network, params, round_mode, raw: InputEvents, batch_size: int,
                     policies: dict | None, out: QuantSplitOutput) -> dict:
    """Overflowing samples per layer and the headroom; without saturating layers also the
    fewest extra bits and where the overflows happen (example/quant_run.py:217-240)."""
    from .quant import OverflowMode
    names = [l.name for l in network.layers]
    summary = {"overflowed_samples": dict(zip(names, out.overflowed.sum(axis=0).tolist())),
               "headroom_bits": dict(zip(names, headroom_bits(params, out)))}
    if any(OverflowMode(p.overflow_mode) is OverflowMode.SATURATE for p in params):
        return summary
    extra, rounds = min_extra_bits(network, params, round_mode, raw, batch_size, policies, out)
    summary.update(min_extra_bits=dict(zip(names, extra)), min_extra_bits_rounds=rounds,
                   overflow_events=overflow_events(network, params, round_mode, raw, out))
    return summary
