"""runtimed_b200 -- sm_100a quantized-linear hot path of syntropd/runtimed.

The compute lives in libruntimed_b200.so (C ABI: include/rtd.h).  This package
holds the host-side mirror of the reference operator surface (weights.py,
tp.py), the ctypes binding (_lib.py), the build recipe (build.py) and the
seeded random-init weight generators used by tests and benchmarks (synth.py).
"""
from . import _lib  # noqa: F401
from .errors import ConfigError, GgufError, MissingWeight, ModelError, ShapeError  # noqa: F401

__all__ = ["ConfigError", "GgufError", "MissingWeight", "ModelError", "ShapeError"]


def __getattr__(name):
    # torch-dependent modules load lazily so the C-ABI checks run without CUDA.
    if name in ("weights", "tp"):
        import importlib

        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)
