"""Importable alias of the ``spiking-affine-lazy-training_b200`` package (its directory name is
not a Python identifier).  ``import salt_b200`` and ``import salt_b200.<module>`` give the very
same module objects as the package itself, so classes compare equal under either name."""
import importlib
import os
import sys

_REAL = "spiking-affine-lazy-training_b200"
_SUBMODULES = ("stream", "quant", "capacity", "layers", "network", "_lib", "device", "backend",
               "plan", "workloads", "float_backend", "sharding", "io", "quant_run", "trace", "build", "calibrate", "comm")

_root = os.path.dirname(os.path.abspath(__file__))
if _root not in sys.path:
    sys.path.insert(0, _root)
_pkg = importlib.import_module(_REAL)
for _name in _SUBMODULES:
    try:
        _mod = importlib.import_module(f"{_REAL}.{_name}")
    except ModuleNotFoundError as e:  # a module that does not exist (yet)
        if e.name != f"{_REAL}.{_name}":
            raise
        continue
    sys.modules[f"{__name__}.{_name}"] = _mod
sys.modules[__name__] = _pkg
