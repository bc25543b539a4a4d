"""Network descriptions and weights, float or quantised, saved with the network as npz.

The file formats are the reference's (salt_core/io.py:16-180), so that models quantised by the
reference's tooling load here unchanged and the other way round:

* ``"__network__"``: a JSON string ``{"format": 1, "input_shape": [...], "layers": [{"type":
  "conv" | "fc", <every layer field>}, ...]}`` (``network_to_dict``, io.py:39-48).
* float weights: one array per layer, keyed by layer name (io.py:80-118).
* quantised models: arrays ``"<layer>/q"``, ``"<layer>/decay_table_int"``, ``"<layer>/v_th_int"``
  (absent when the layer does not fire) and ``"<layer>/scale"``, plus ``"__quant__"``, a JSON
  string ``{"format": 1, "round_mode": ..., "layers": {name: {"f_a", "f_V", "i_V",
  "overflow_mode"}}, "metadata": {...}}`` (io.py:129-180).

Arrays are returned as numpy arrays (the reference returns JAX arrays); the values are the same.
"""
from __future__ import annotations

import dataclasses
import json
import os
from collections.abc import Mapping, Sequence
from typing import Any, NamedTuple

import numpy as np

from .layers import ConvLayer, FCLayer
from .network import Network
from .quant import OverflowMode, QuantizedLayerParams, RoundMode

FORMAT_VERSION = 1
NETWORK_KEY = "__network__"
QUANT_KEY = "__quant__"
_LAYER_TYPES = {"conv": ConvLayer, "fc": FCLayer}


def _layer_type(layer) -> str:
    for name, cls in _LAYER_TYPES.items():
        if type(layer) is cls:
            return name
    raise ValueError(f"{layer.name}: layer type {type(layer).__name__} cannot be serialised")


def network_to_dict(network: Network) -> dict:
    """io.py:39-48: the input grid and every field of every layer (capacities included)."""
    return {"format": FORMAT_VERSION, "input_shape": list(network.input_shape),
            "layers": [{"type": _layer_type(l), **dataclasses.asdict(l)} for l in network.layers]}


def network_from_dict(description: Mapping) -> Network:
    """io.py:51-66; ValueError on another format or an unknown layer type."""
    if description.get("format") != FORMAT_VERSION:
        raise ValueError(f"network description format must be {FORMAT_VERSION}, got "
                         f"{description.get('format')!r}")
    layers = []
    for entry in description["layers"]:
        fields = dict(entry)
        kind = fields.pop("type")
        if kind not in _LAYER_TYPES:
            raise ValueError(f"unknown layer type {kind!r} (known: {list(_LAYER_TYPES)})")
        layers.append(_LAYER_TYPES[kind](**fields))
    return Network(tuple(description["input_shape"]), tuple(layers))


def _checked_layer_names(network: Network, n_per_layer: int, what: str) -> list[str]:
    names = [l.name for l in network.layers]
    if n_per_layer != len(names):
        raise ValueError(f"{n_per_layer} {what} for a network of {len(names)} layers")
    if len(set(names)) != len(names) or NETWORK_KEY in names or QUANT_KEY in names:
        raise ValueError(f"layer names must be distinct and not {NETWORK_KEY!r}: {names}")
    return names


def _network_json(network: Network) -> np.ndarray:
    return np.asarray(json.dumps(network_to_dict(network)))


def _read_network(arrays: Mapping[str, np.ndarray]) -> Network:
    if NETWORK_KEY not in arrays:
        raise ValueError(f"no network description ({NETWORK_KEY!r})")
    return network_from_dict(json.loads(str(arrays[NETWORK_KEY])))


def weights_to_arrays(network: Network, weights: Sequence) -> dict[str, np.ndarray]:
    names = _checked_layer_names(network, len(weights), "weight arrays")
    arrays = {n: np.asarray(w) for n, w in zip(names, weights)}
    arrays[NETWORK_KEY] = _network_json(network)
    return arrays


def weights_from_arrays(arrays: Mapping[str, np.ndarray]) -> tuple[Network, tuple]:
    network = _read_network(arrays)
    return network, tuple(np.asarray(arrays[l.name]) for l in network.layers)


def save_weights(path: str | os.PathLike, network: Network, weights: Sequence) -> None:
    np.savez(path, **weights_to_arrays(network, weights))


def load_weights(path: str | os.PathLike) -> tuple[Network, tuple]:
    with np.load(path) as arrays:
        return weights_from_arrays(arrays)


class QuantizedModel(NamedTuple):
    """io.py:121-126"""
    network: Network
    params: tuple
    round_mode: RoundMode
    metadata: dict[str, Any]


def save_quantized(path: str | os.PathLike, network: Network, params: Sequence,
                   round_mode, metadata: Mapping[str, Any]) -> None:
    """io.py:129-155.  metadata must be JSON-serialisable (TypeError otherwise)."""
    names = _checked_layer_names(network, len(params), "parameter sets")
    arrays = {NETWORK_KEY: _network_json(network)}
    info = {}
    for name, p in zip(names, params):
        arrays[f"{name}/q"] = np.asarray(p.q)
        arrays[f"{name}/decay_table_int"] = np.asarray(p.decay_table_int)
        if p.v_th_int is not None:
            arrays[f"{name}/v_th_int"] = np.asarray(p.v_th_int)
        arrays[f"{name}/scale"] = np.asarray(p.scale)
        info[name] = {"f_a": int(p.f_a), "f_V": int(p.f_V), "i_V": int(p.i_V),
                      "overflow_mode": OverflowMode(getattr(p, "overflow_mode", "wrap")).value}
    arrays[QUANT_KEY] = np.asarray(json.dumps({
        "format": FORMAT_VERSION, "round_mode": RoundMode(round_mode).value, "layers": info,
        "metadata": dict(metadata)}))
    np.savez(path, **arrays)


def load_quantized(path: str | os.PathLike) -> QuantizedModel:
    """io.py:158-180; ValueError without the network or quantisation entries or on another
    format."""
    with np.load(path) as arrays:
        network = _read_network(arrays)
        if QUANT_KEY not in arrays:
            raise ValueError(f"no quantisation settings ({QUANT_KEY!r})")
        quant = json.loads(str(arrays[QUANT_KEY]))
        if quant.get("format") != FORMAT_VERSION:
            raise ValueError(f"quantisation format must be {FORMAT_VERSION}, got "
                             f"{quant.get('format')!r}")
        params = []
        for layer in network.layers:
            name, li = layer.name, quant["layers"][layer.name]
            vkey = f"{name}/v_th_int"
            params.append(QuantizedLayerParams(
                q=np.asarray(arrays[f"{name}/q"]),
                decay_table_int=np.asarray(arrays[f"{name}/decay_table_int"]),
                v_th_int=np.asarray(arrays[vkey]) if vkey in arrays else None,
                scale=np.asarray(arrays[f"{name}/scale"]),
                f_a=li["f_a"], f_V=li["f_V"], i_V=li["i_V"],
                overflow_mode=OverflowMode(li["overflow_mode"])))
    return QuantizedModel(network, tuple(params), RoundMode(quant["round_mode"]),
                          quant["metadata"])
