"""Importable alias of the ``spiking-affine-lazy-training_b200`` package (its directory name is
not a Python identifier): ``import salt_b200`` gives that package."""
import importlib
import os
import sys

_root = os.path.dirname(os.path.abspath(__file__))
if _root not in sys.path:
    sys.path.insert(0, _root)
sys.modules[__name__] = importlib.import_module("spiking-affine-lazy-training_b200")
