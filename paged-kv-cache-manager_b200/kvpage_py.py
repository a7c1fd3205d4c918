"""Drop-in for the reference's pybind11 module `kvpage_py` (python/kvpage_py.cpp:12-66 of
prathameshpranjale/paged-kv-cache-manager): the same `KVManager` class -- constructor, method names, argument
names and results, `stats()` readable by attribute -- backed by this library's C++17 KVManager.  Put this
directory on sys.path and the reference's Python harness (python/paged_model.py, model_check.py) imports it
unchanged.  The reference module's CPU attention functions are not provided: this library has no CPU attention
path (its GPU entry points are paged_attention / the decode-step Decoder of the package)."""
import importlib
import os
import sys

_here = os.path.dirname(os.path.abspath(__file__))
if os.path.dirname(_here) not in sys.path:
    sys.path.insert(0, os.path.dirname(_here))
_pkg = importlib.import_module(os.path.basename(_here))

KVManager = _pkg.KVManager
KVStats = _pkg.KVStats

__all__ = ["KVManager", "KVStats"]
