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

from . import _core
from ._core import (FormatError, Model, Stream, device_count, devices, families, latency_threads, set_devices,
                    set_latency_threads, set_threads, threads)

__version__: str = _core.version()

__all__ = ["FormatError", "Model", "Stream", "__version__", "build_info", "device_count", "devices", "export",
           "families", "latency_threads", "load", "load_plugin", "set_devices", "set_latency_threads",
           "set_threads", "synth", "threads"]

_SUBMODULES = ("export", "synth", "cli")


def load(source: Any) -> Model:
    """Opens a model from a path, the file's bytes, or a binary file object."""
    if isinstance(source, (bytes, bytearray, memoryview)):
        return Model.from_bytes(bytes(source))
    if hasattr(source, "read"):
        return Model.from_bytes(source.read())
    return Model.open(os.fspath(source))


def load_plugin(path: str | os.PathLike) -> None:
    """Plugin families are CPU code and not part of this build: raises NotImplementedError."""
    _core.load_plugin(os.fspath(path))


def _spec(self: Model) -> dict:
    return json.loads(self.spec_json)


Model.spec = property(_spec)  # type: ignore[attr-defined]


def build_info() -> dict:
    """Version, ABI, families, thread and GPU settings, for logs and status pages."""
    return {"version": __version__, "abi": _core.abi_version(), "families": families(), "threads": threads(),
            "latency_threads": latency_threads(), "devices": devices(), "device_count": device_count(),
            "machine": platform.machine(), "python": platform.python_version(), "rdt_extension": False}


def __getattr__(name: str) -> Any:
    if name in _SUBMODULES:
        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(f"module 'montlok' has no attribute {name!r}")


def __dir__() -> list[str]:
    return sorted(set(globals()) | set(_SUBMODULES))
