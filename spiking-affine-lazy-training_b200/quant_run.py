"""Whole-split integer forward, capacity growth and the reference-file check, on the B200 backend.

Mirrors example/quant_run.py:54-136 and the check of example/quantize.py:306-330: a split of
input samples runs through the quantised network batch by batch; the per-sample fields that the
reference records in ``reference.npz`` (REFERENCE_FIELDS) come back for comparison, and
``run_until_fits`` grows the capacities until no sample overflows.  Capacities are runtime sizes
here, so growing them re-plans buffers; nothing is recompiled.
"""
from __future__ import annotations

from typing import Callable, NamedTuple

import numpy as np

from .capacity import GrowthPolicy, LayerDiag, grown_to_fit
from .network import InputEvents, Network

REFERENCE_FIELDS = ("v_final_int", "preds", "spike_count", "truncated", "overflowed")
_ARRAY_FIELDS = REFERENCE_FIELDS + ("v_unfitted_min", "v_unfitted_max")


class QuantSplitOutput(NamedTuple):
    """example/quant_run.py:54-64, N samples."""
    v_final_int: np.ndarray     # (N, n_out) output-layer registers
    preds: np.ndarray           # (N,)
    spike_count: np.ndarray     # (N, n_layers)
    truncated: np.ndarray       # (N, n_layers) a capacity knob overflowed
    overflowed: np.ndarray      # (N, n_layers) a register overflowed
    v_unfitted_min: np.ndarray  # (N, n_layers)
    v_unfitted_max: np.ndarray  # (N, n_layers)
    needed: dict                # layer name -> knob -> (N,) needed capacity


def membrane_scores(readout_v_final: np.ndarray) -> np.ndarray:
    """MembraneRegressionDecoder (salt_core/decoder.py:34-50): the read-out v_final are the
    scores; argmax picks the lowest index on ties."""
    return readout_v_final


def _batches(raw: InputEvents, batch_size: int):
    n = np.asarray(raw.event_times).shape[0]
    for start in range(0, n, batch_size):
        sl = slice(start, start + batch_size)
        yield InputEvents(np.asarray(raw.event_times)[sl], np.asarray(raw.source_idx)[sl],
                          np.asarray(raw.n_real_events)[sl])


def quant_forward_split(network: Network, params, round_mode, raw: InputEvents,
                        batch_size: int, *, backend=None,
                        decode: Callable[[np.ndarray], np.ndarray] = membrane_scores
                        ) -> QuantSplitOutput:
    """example/quant_run.py:71-103: every sample of raw through the integer forward."""
    from .backend import QuantB200Backend
    backend = backend or QuantB200Backend(round_mode)
    layers = list(network.layers)
    parts = []
    for rb in _batches(raw, batch_size):
        out = backend.run_network(layers, params, network.input_stream(rb))
        scores = decode(backend.readout(out.last, params[-1]).v_final)
        parts.append({
            "v_final_int": out.last.v_final,
            "preds": np.argmax(scores, axis=1),
            "spike_count": np.stack([r.spike_count for r in out.results], axis=1),
            "truncated": np.stack([~np.asarray(l.capacity.fits(d), dtype=bool)
                                   for l, d in zip(layers, out.diags)], axis=1),
            "overflowed": np.stack([r.overflowed for r in out.results], axis=1),
            "v_unfitted_min": np.stack([r.v_unfitted_min for r in out.results], axis=1),
            "v_unfitted_max": np.stack([r.v_unfitted_max for r in out.results], axis=1),
            "needed": [d.needed for d in out.diags]})
    arrays = {k: np.concatenate([p[k] for p in parts]) for k in _ARRAY_FIELDS}
    needed = {l.name: {knob: np.concatenate([np.atleast_1d(p["needed"][i][knob]) for p in parts])
                       for knob in parts[0]["needed"][i]}
              for i, l in enumerate(layers)}
    return QuantSplitOutput(**arrays, needed=needed)


def reference_arrays(out: QuantSplitOutput) -> dict[str, np.ndarray]:
    """example/quant_run.py:106-108"""
    return {k: getattr(out, k) for k in REFERENCE_FIELDS}


def grown_for_needed(layers, policies, needed: dict) -> list:
    """example/quant_run.py:111-119: grow every knob to its largest need over the samples."""
    diags = [LayerDiag(0, 0.0, {k: int(np.max(v)) for k, v in needed[l.name].items()})
             for l in layers]
    return list(grown_to_fit(layers, policies, diags))


def run_until_fits(network: Network, params, round_mode, raw: InputEvents, batch_size: int,
                   policies: dict | None = None, *, backend=None, max_rounds: int = 16
                   ) -> tuple[Network, QuantSplitOutput, int]:
    """example/quant_run.py:122-136: rerun with grown capacities while a sample overflows.
    Returns (the network that fits, its output, the number of reruns)."""
    policies = policies or {l.name: GrowthPolicy() for l in network.layers}
    n = 0
    out = quant_forward_split(network, params, round_mode, raw, batch_size, backend=backend)
    while out.truncated.any():
        if n >= max_rounds:
            raise RuntimeError(f"capacities still overflow after {max_rounds} regrowths")
        network = network.replace_layers(grown_for_needed(network.layers, policies, out.needed))
        out = quant_forward_split(network, params, round_mode, raw, batch_size, backend=backend)
        n += 1
    return network, out, n


def check_against_reference(out: QuantSplitOutput, reference: dict) -> dict[str, np.ndarray]:
    """example/quantize.py:320-327: per REFERENCE_FIELDS, the indices of the samples whose
    values differ from the recorded reference (empty arrays when everything matches)."""
    diffs = {}
    for key, value in reference_arrays(out).items():
        ref = np.asarray(reference[key])
        if ref.shape != value.shape:
            diffs[key] = np.arange(max(len(ref), len(value)))
            continue
        d = value != ref
        diffs[key] = np.nonzero(d.reshape(d.shape[0], -1).any(axis=1))[0]
    return diffs


def check_quantized(model_path, reference_path, raw: InputEvents, batch_size: int | None = None,
                    *, backend=None) -> tuple[int, dict[str, np.ndarray]]:
    """example/quantize.py:306-330 without the dataset loader: rerun the saved model on the
    given samples and compare with the saved reference.npz.  Returns (0 when every field of
    every sample matches, else 1; the differing sample indices per field)."""
    from .io import load_quantized
    model = load_quantized(model_path)
    with np.load(reference_path) as npz:
        reference = dict(npz)
    bs = int(batch_size or model.metadata.get("batch_size", 64))
    out = quant_forward_split(model.network, model.params, model.round_mode, raw, bs,
                              backend=backend)
    diffs = check_against_reference(out, reference)
    return int(any(len(v) for v in diffs.values())), diffs


# ---------------------------------------------------------------- overflow analysis
# example/quant_run.py:139-240

MAX_OVERFLOW_EVENTS = 50


def with_extra_i_V(params, extra: list[int]) -> list:
    """example/quant_run.py:139-141: each layer's i_V plus extra[i] bits."""
    return [p._replace(i_V=p.i_V + e) for p, e in zip(params, extra)]


def headroom_bits(params, out: QuantSplitOutput) -> list[float | None]:
    """example/quant_run.py:144-154: bits between each layer's unfitted extremes and its
    register range (negative: overflow); None when every value was 0."""
    import math
    res = []
    for i, p in enumerate(params):
        peak = max(-int(out.v_unfitted_min[:, i].min()), int(out.v_unfitted_max[:, i].max()) + 1)
        res.append(None if peak <= 0 else round(p.i_V + p.f_V - 1 - math.log2(peak), 3))
    return res


def min_extra_bits(network: Network, params, round_mode, raw: InputEvents, batch_size: int,
                   policies: dict | None, out: QuantSplitOutput, *, backend=None
                   ) -> tuple[list[int], int]:
    """example/quant_run.py:157-174: widen the most upstream overflowing layer by one bit and
    rerun until no sample overflows.  Returns (extra bits per layer, reruns)."""
    extra = [0] * len(params)
    rounds = 0
    while out.overflowed.any():
        extra[int(np.argmax(out.overflowed.any(axis=0)))] += 1
        _, out, _ = run_until_fits(network, with_extra_i_V(params, extra), round_mode, raw,
                                   batch_size, policies, backend=backend)
        rounds += 1
    return extra, rounds


def _neuron_position(layer, neuron: int) -> tuple[int, int, int]:
    shape = layer.unflatten_neurons(np.zeros(layer.n_neurons)).shape
    return tuple(int(v) for v in np.unravel_index(neuron, shape))


def overflow_events(network: Network, params, round_mode, raw: InputEvents,
                    out: QuantSplitOutput, *, backend=None) -> list[dict]:
    """example/quant_run.py:183-214: for each overflowing (sample, layer, neuron), its first
    overflowing column — the time, the register before and after it, whether it fired — and the
    neuron's unfitted extremes; at most MAX_OVERFLOW_EVENTS entries.  Each overflowing sample
    runs once more on the GPU with the layer traces' per-neuron records."""
    from .backend import QuantB200Backend
    from .device import DeviceStream
    backend = backend or QuantB200Backend(round_mode)
    layers = list(network.layers)
    events = []
    for i in np.nonzero(out.overflowed.any(axis=1))[0]:
        i = int(i)
        one = InputEvents(np.asarray(raw.event_times)[i:i + 1], np.asarray(raw.source_idx)[i:i + 1],
                          np.asarray(raw.n_real_events)[i:i + 1])
        cur = DeviceStream.from_host(network.input_stream(one))
        for layer, p in zip(layers, params):
            tr = backend.trace_layer_device(layer, p, cur, dense=False)
            first = tr["first_overflow"][0].cpu().numpy()
            rec = {k: tr[k][0].cpu().numpy() for k in ("v_before", "v_after", "spiked", "time_ms",
                                                        "v_min", "v_max")}
            half = 2 ** (p.i_V + p.f_V - 1)
            for neuron in np.nonzero(first >= 0)[0]:
                ch, y, x = _neuron_position(layer, int(neuron))
                events.append({"sample": i, "layer": layer.name, "channel": ch, "y": y, "x": x,
                               "time_ms": float(rec["time_ms"][neuron]),
                               "v_before": int(rec["v_before"][neuron]),
                               "v_after": int(rec["v_after"][neuron]),
                               "spiked": bool(rec["spiked"][neuron]),
                               "true_min": int(rec["v_min"][neuron]),
                               "true_max": int(rec["v_max"][neuron]),
                               "register_range": [-half, half - 1]})
                if len(events) >= MAX_OVERFLOW_EVENTS:
                    return events
            cur = backend.forward_layer_device(layer, p, cur).out
    return events


def overflow_summary(network: Network, params, round_mode, raw: InputEvents, batch_size: int,
                     policies: dict | None, out: QuantSplitOutput, *, backend=None) -> dict:
    """example/quant_run.py:217-240: overflowing samples per layer and headroom; without
    saturating layers also the fewest extra bits and where the overflows happen."""
    from .quant import OverflowMode
    names = [l.name for l in network.layers]
    summary = {"overflowed_samples": {n: int(out.overflowed[:, i].sum())
                                      for i, n in enumerate(names)},
               "headroom_bits": dict(zip(names, headroom_bits(params, out)))}
    if any(OverflowMode(getattr(p, "overflow_mode", "wrap")) is OverflowMode.SATURATE
           for p in params):
        return summary
    extra, rounds = min_extra_bits(network, params, round_mode, raw, batch_size, policies, out,
                                   backend=backend)
    return {**summary, "min_extra_bits": dict(zip(names, extra)),
            "min_extra_bits_rounds": rounds,
            "overflow_events": overflow_events(network, params, round_mode, raw, out,
                                               backend=backend)}
