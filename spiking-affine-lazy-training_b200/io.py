"""Model files: network descriptions, float weights and quantised models as npz archives.

The layouts are the reference's (salt_core/io.py), byte-compatible so that a model quantised by
either implementation loads in the other:

  ``__network__``  0-d string array holding the JSON ``{"format": 1, "input_shape": [...],
                   "layers": [{"type": "conv" | "fc", <every layer field>}, ...]}``
  ``<layer>``      float weights, one array per layer (weight files)
  ``<layer>/<a>``  quantised arrays, ``a`` from ``QUANT_ARRAYS`` (quantised models)
  ``__quant__``    0-d string array holding the JSON ``{"format": 1, "round_mode": ...,
                   "layers": {<layer>: {"f_a", "f_V", "i_V", "overflow_mode"}},
                   "metadata": {...}}`` (quantised models)

Every read and write goes through one schema: the tag table of layer classes, the table of
per-layer quantised arrays and the table of per-layer quantised settings.  Arrays come back as
numpy arrays.
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
RESERVED_KEYS = (NETWORK_KEY, QUANT_KEY)

# type tag of each serialisable layer class
LAYER_TAGS = {"conv": ConvLayer, "fc": FCLayer}

# quantised arrays stored per layer as "<layer>/<name>": (name, may be absent).  An absent
# optional array stands for None (v_th_int of a layer that never fires).
QUANT_ARRAYS = (("q", False), ("decay_table_int", False), ("v_th_int", True), ("scale", False))

# quantised settings stored per layer in the __quant__ document: name -> (encode, decode)
QUANT_SETTINGS = {
    "f_a": (int, int),
    "f_V": (int, int),
    "i_V": (int, int),
    "overflow_mode": (lambda m: OverflowMode(m).value, OverflowMode),
}


# ---------------------------------------------------------------- network descriptions

def _tag_of(layer) -> str:
    tags = [tag for tag, cls in LAYER_TAGS.items() if type(layer) is cls]
    if not tags:
        raise ValueError(f"{layer.name}: layer type {type(layer).__name__} cannot be serialised")
    return tags[0]


def _require_format(doc: Mapping, what: str) -> None:
    if doc.get("format") != FORMAT_VERSION:
        raise ValueError(f"{what} format must be {FORMAT_VERSION}, got {doc.get('format')!r}")


def network_to_dict(network: Network) -> dict:
    """The JSON-ready description: the input grid and every field of every layer, capacities
    included (salt_core/io.py:40-48)."""
    layers = [dict(type=_tag_of(layer), **dataclasses.asdict(layer)) for layer in network.layers]
    return {"format": FORMAT_VERSION, "input_shape": list(network.input_shape), "layers": layers}


def network_from_dict(description: Mapping) -> Network:
    """Inverse of network_to_dict; ValueError on another format or an unknown layer type
    (salt_core/io.py:51-63)."""
    _require_format(description, "network description")
    layers = []
    for entry in description["layers"]:
        fields = {k: v for k, v in entry.items() if k != "type"}
        cls = LAYER_TAGS.get(entry.get("type"))
        if cls is None:
            raise ValueError(f"unknown layer type {entry.get('type')!r} (known: "
                             f"{sorted(LAYER_TAGS)})")
        layers.append(cls(**fields))
    return Network(tuple(description["input_shape"]), tuple(layers))


# ---------------------------------------------------------------- the archive

class _Archive:
    """A flat name -> array mapping with the two JSON documents and per-layer keys."""

    def __init__(self, arrays: Mapping[str, np.ndarray] | None = None):
        self.arrays = dict(arrays or {})

    @staticmethod
    def for_network(network: Network, per_layer: int, what: str) -> "_Archive":
        names = [layer.name for layer in network.layers]
        if per_layer != len(names):
            raise ValueError(f"{per_layer} {what} for a network of {len(names)} layers")
        clash = len(set(names)) != len(names) or any(n in RESERVED_KEYS for n in names)
        if clash:
            raise ValueError(f"layer names must be distinct and not in {RESERVED_KEYS}: {names}")
        archive = _Archive()
        archive.put_doc(NETWORK_KEY, network_to_dict(network))
        return archive

    def put_doc(self, key: str, doc: Mapping) -> None:
        self.arrays[key] = np.asarray(json.dumps(doc))

    def doc(self, key: str, what: str) -> dict:
        if key not in self.arrays:
            raise ValueError(f"no {what} ({key!r})")
        return json.loads(str(self.arrays[key]))

    def network(self) -> Network:
        return network_from_dict(self.doc(NETWORK_KEY, "network description"))

    def save(self, path: str | os.PathLike) -> None:
        np.savez(path, **self.arrays)

    @staticmethod
    def load(path: str | os.PathLike) -> "_Archive":
        with np.load(path) as z:
            return _Archive({k: z[k] for k in z.files})


# ---------------------------------------------------------------- float weights

def weights_to_arrays(network: Network, weights: Sequence) -> dict[str, np.ndarray]:
    """The weight-file mapping: one array per layer name plus the network description
    (salt_core/io.py:87-97)."""
    archive = _Archive.for_network(network, len(weights), "weight arrays")
    for layer, w in zip(network.layers, weights):
        archive.arrays[layer.name] = np.asarray(w)
    return archive.arrays


def weights_from_arrays(arrays: Mapping[str, np.ndarray]) -> tuple[Network, tuple]:
    """(network, weights in layer order) from a weight-file mapping (salt_core/io.py:100-106)."""
    archive = _Archive(arrays)
    network = archive.network()
    return network, tuple(np.asarray(archive.arrays[layer.name]) for layer in network.layers)


def save_weights(path: str | os.PathLike, network: Network, weights: Sequence) -> None:
    _Archive(weights_to_arrays(network, weights)).save(path)


def load_weights(path: str | os.PathLike) -> tuple[Network, tuple]:
    return weights_from_arrays(_Archive.load(path).arrays)


# ---------------------------------------------------------------- quantised models

class QuantizedModel(NamedTuple):
    """A loaded quantised model (salt_core/io.py:121-126)."""
    network: Network
    params: tuple
    round_mode: RoundMode
    metadata: dict[str, Any]


def save_quantized(path: str | os.PathLike, network: Network, params: Sequence,
                   round_mode, metadata: Mapping[str, Any]) -> None:
    """Writes a quantised model (salt_core/io.py:129-153); metadata must be JSON-serialisable
    (TypeError otherwise)."""
    archive = _Archive.for_network(network, len(params), "parameter sets")
    settings = {}
    for layer, p in zip(network.layers, params):
        for name, optional in QUANT_ARRAYS:
            value = getattr(p, name)
            if value is None and optional:
                continue
            archive.arrays[f"{layer.name}/{name}"] = np.asarray(value)
        settings[layer.name] = {name: enc(getattr(p, name))
                                for name, (enc, _) in QUANT_SETTINGS.items()}
    archive.put_doc(QUANT_KEY, {"format": FORMAT_VERSION,
                                "round_mode": RoundMode(round_mode).value,
                                "layers": settings, "metadata": dict(metadata)})
    archive.save(path)


def load_quantized(path: str | os.PathLike) -> QuantizedModel:
    """Reads a quantised model (salt_core/io.py:156-180); ValueError when the network or the
    quantisation document is missing or has another format."""
    archive = _Archive.load(path)
    network = archive.network()
    quant = archive.doc(QUANT_KEY, "quantisation settings")
    _require_format(quant, "quantisation")
    params = []
    for layer in network.layers:
        fields = {}
        for name, optional in QUANT_ARRAYS:
            key = f"{layer.name}/{name}"
            fields[name] = np.asarray(archive.arrays[key]) if (key in archive.arrays
                                                                or not optional) else None
        stored = quant["layers"][layer.name]
        fields.update({name: dec(stored[name]) for name, (_, dec) in QUANT_SETTINGS.items()})
        params.append(QuantizedLayerParams(**fields))
    return QuantizedModel(network, tuple(params), RoundMode(quant["round_mode"]),
                          quant["metadata"])
