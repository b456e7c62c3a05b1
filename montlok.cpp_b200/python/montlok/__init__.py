"""montlok on NVIDIA B200: tree-ensemble models (GBDT and random forests) run
by CUDA kernels behind montlok's C ABI.

    import montlok

    model = montlok.load("gbdt.montlok")      # tree_ensemble models
    y = model.predict(x)                      # [batch, features] -> [batch, outputs]
    model.predict(x, out=y)                   # into an existing float64 array

The API is the reference package's (montlok.cpp python/montlok/__init__.py):
``load``, ``Model``, ``Stream``, ``FormatError``, thread settings and
``build_info``. :mod:`montlok.export` writes model files (LightGBM and XGBoost
dumps, scikit-learn trees); :mod:`montlok.synth` builds the seeded benchmark
models. Additions: ``Model.predict`` accepts CUDA arrays, ``predict_leaves``
returns leaf indices, ``set_devices`` spreads host batches over GPUs.
"""

from __future__ import annotations

import importlib
import json
import os
import platform
from typing import Any

# The native library loads with the first use of a name that needs it (below),
# so the pure-Python submodules (export, synth) import without it: the
# reference benchmark arm and the CPU checkers use them beside the reference
# runtime without mapping libmontlok.so into their process.
_CORE_NAMES = ("FormatError", "Model", "Stream", "device_count", "devices", "families", "latency_threads",
               "set_devices", "set_latency_threads", "set_threads", "threads")

__all__ = ["FormatError", "Model", "Stream", "__version__", "build_info", "device_count", "devices", "export",
           "families", "latency_threads", "load", "load_plugin", "set_devices", "set_latency_threads",
           "set_threads", "synth", "threads"]

_SUBMODULES = ("export", "synth", "cli")

# The library's montlok_version(); a test checks that the two agree.
__version__ = "0.2.0"


def _native():
    """montlok._core (raises ImportError when libmontlok.so is missing)."""
    core = importlib.import_module("._core", __name__)
    if not hasattr(core.Model, "spec"):
        core.Model.spec = property(lambda self: json.loads(self.spec_json))
    return core


def load(source: Any):
    """Opens a model from a path, the file's bytes, or a binary file object."""
    core = _native()
    if isinstance(source, (bytes, bytearray, memoryview)):
        return core.Model.from_bytes(bytes(source))
    if hasattr(source, "read"):
        return core.Model.from_bytes(source.read())
    return core.Model.open(os.fspath(source))


def load_plugin(path: str | os.PathLike) -> None:
    """Plugin families are CPU code and not part of this build: raises NotImplementedError."""
    _native().load_plugin(os.fspath(path))


def build_info() -> dict:
    """Version, ABI, families, thread and GPU settings, for logs and status pages."""
    core = _native()
    return {"version": core.version(), "abi": core.abi_version(), "families": core.families(),
            "threads": core.threads(), "latency_threads": core.latency_threads(), "devices": core.devices(),
            "device_count": core.device_count(), "machine": platform.machine(),
            "python": platform.python_version(), "rdt_extension": False}


def __getattr__(name: str) -> Any:
    if name in _SUBMODULES:
        return importlib.import_module(f".{name}", __name__)
    if name in _CORE_NAMES or name == "_core":
        core = _native()
        return core if name == "_core" else getattr(core, name)
    raise AttributeError(f"module 'montlok' has no attribute {name!r}")


def __dir__() -> list[str]:
    return sorted(set(globals()) | set(_SUBMODULES) | set(_CORE_NAMES))
