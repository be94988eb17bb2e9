"""mini-llama B200: quantized weight matmul (q8_0 / q4_0 / q4_1) for sm_100a.

The product is the C-ABI library ``lib/libmlq.so`` (include/mlq.h), built
from ``csrc/`` by ``build.py``.  This Python package is a thin host layer:

* ``mlq``        ctypes bindings of the C ABI (torch CUDA tensors in/out)
* ``cuda_quant`` the reference's cuda_quant.h entry points, same names
* ``synth``      the seeded synthetic-input generator used by tests/bench

The directory name contains a hyphen, so load it by path, e.g.::

    spec = importlib.util.spec_from_file_location(
        "mini_llama_b200", "mini-llama_b200/__init__.py",
        submodule_search_locations=["mini-llama_b200"])
"""
from . import mlq, synth  # noqa: F401

__all__ = ["mlq", "synth"]
