"""Drop-in for the reference's pybind11 module `kvpage_py` (python/kvpage_py.cpp:12-66 of
prathameshpranjale/paged-kv-cache-manager): the same `KVManager` class -- constructor, method names, argument
names and results, `stats()` readable by attribute -- backed by this library's C++17 KVManager -- and the
module's two attention functions with their signatures (python/kvpage_py.cpp:43-66): numpy arrays in, a
numpy array out, computed on the current CUDA device by this library's fp32 kernel (there is no CPU
attention path).  Put this directory on sys.path and the reference's Python harness (python/paged_model.py,
model_check.py, attention_check.py) imports it unchanged."""
import importlib
import os
import sys

_here = os.path.dirname(os.path.abspath(__file__))
if os.path.dirname(_here) not in sys.path:
    sys.path.insert(0, os.path.dirname(_here))
_pkg = importlib.import_module(os.path.basename(_here))

KVManager = _pkg.KVManager
KVStats = _pkg.KVStats


def reference_attention(nh, kvh, hd, bs, q, k, v, tables, lens):
    """The reference module's reference_attention(nh, kvh, hd, bs, q, k, v, tables, lens) -> out."""
    return _pkg.paged_attention_host(nh, kvh, hd, bs, q, k, v, tables, lens, 1)


def paged_attention_cpu(nh, kvh, hd, bs, q, k, v, tables, lens, partitions):
    """The reference module's paged_attention_cpu(nh, kvh, hd, bs, q, k, v, tables, lens, partitions) -> out."""
    return _pkg.paged_attention_host(nh, kvh, hd, bs, q, k, v, tables, lens, partitions)


__all__ = ["KVManager", "KVStats", "reference_attention", "paged_attention_cpu"]
