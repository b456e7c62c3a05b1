"""TEST INFRASTRUCTURE ONLY - Python access to the CPU checkers.

* :class:`Oracle` drives the plain-C restatement (tree_oracle.c) of the
  reference's tree_ensemble predict on a model file's own node arrays.
* :class:`Reference` drives the reference runtime itself, compiled from its
  sources into ``_ref/libmontlok_ref.so`` by this directory's Makefile (only
  where the reference sources are present). ``Reference.leaves`` reads the
  reference's leaf selection without touching its code: it re-exports the
  model with every leaf's value replaced by its node index, one output per
  tree, base 0, sum and identity link, so each output is exactly the index of
  the leaf the reference reached (one addition to 0.0 is exact).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the product library never does.
"""

from __future__ import annotations

import ctypes
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "libmontlok_oracle.so"
REF_LIB = HERE / "_ref" / "libmontlok_ref.so"
CONSUMER = HERE / "_ref" / "test_core_consumer"  # the reference's C++ test linked to libmontlok.so


def reference_sources() -> Path | None:
    """The reference's source tree: the directory named by MONTLOK_REFERENCE,
    else a checkout called ``reference`` beside this repository; None when
    neither holds its sources (then nothing of the reference is built)."""
    for where in (os.environ.get("MONTLOK_REFERENCE"), HERE.parent.parent / "reference"):
        if where and (Path(where) / "src" / "core" / "trees.cpp").exists():
            return Path(where)
    return None


REFERENCE_SOURCES = reference_sources()
sys.path.insert(0, str(HERE.parent / "montlok.cpp_b200" / "python"))

from montlok import export  # noqa: E402  (the model-file reader)

_LINKS = {"identity": 0, "sigmoid": 1, "softmax": 2, "exp": 3}


def build(reference: bool = True) -> None:
    """Builds the oracle (and the reference library when its sources exist)."""
    targets = ["oracle"]
    variables = []
    if reference and REFERENCE_SOURCES is not None:
        targets.append("ref")
        if (HERE.parent / "montlok.cpp_b200" / "python" / "montlok" / "libmontlok.so").exists():
            targets.append("consumer")
        variables.append(f"REF={REFERENCE_SOURCES}")
    subprocess.run(["make", "-s", "-C", str(HERE), *variables, *targets], check=True)


class _Forest(ctypes.Structure):
    _fields_ = [("features", ctypes.c_int32), ("outputs", ctypes.c_int32), ("trees", ctypes.c_int32),
                ("nodes", ctypes.c_int32), ("decision_le", ctypes.c_int32), ("cast_f32", ctypes.c_int32),
                ("mean", ctypes.c_int32), ("link", ctypes.c_int32), ("sigmoid_scale", ctypes.c_double),
                ("base", ctypes.c_void_p), ("roots", ctypes.c_void_p), ("tree_output", ctypes.c_void_p),
                ("feature", ctypes.c_void_p), ("threshold", ctypes.c_void_p), ("left", ctypes.c_void_p),
                ("right", ctypes.c_void_p), ("value", ctypes.c_void_p), ("flags", ctypes.c_void_p),
                ("standardize", ctypes.c_int32), ("clip", ctypes.c_int32), ("pre_mean", ctypes.c_void_p),
                ("pre_scale", ctypes.c_void_p), ("clip_lo", ctypes.c_double), ("clip_hi", ctypes.c_double)]


def _input(x) -> tuple[np.ndarray, int]:
    a = np.asarray(x)
    if a.dtype == np.float32:
        return np.ascontiguousarray(a), 1
    return np.ascontiguousarray(a, dtype=np.float64), 2


_oracle_lib = None


def _oracle() -> ctypes.CDLL:
    global _oracle_lib
    if _oracle_lib is None:
        if not ORACLE_LIB.exists():
            build(reference=False)
        lib = ctypes.CDLL(str(ORACLE_LIB))
        for name in ("oracle_predict", "oracle_leaves"):
            getattr(lib, name).restype = None
            getattr(lib, name).argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                           ctypes.c_void_p, ctypes.c_int]
        lib.oracle_exp.restype = ctypes.c_double
        lib.oracle_exp.argtypes = [ctypes.c_double]
        _oracle_lib = lib
    return _oracle_lib


def oracle_exp(x: float) -> float:
    """The restated reference exp of one value."""
    return float(_oracle().oracle_exp(float(x)))


class Oracle:
    """The C restatement over a model file's arrays."""

    def __init__(self, model: bytes) -> None:
        self._lib = _oracle()
        spec, t = export.read(model)
        cfg = spec.get("config", {}) or {}
        p = cfg.get("tensors", "trees")
        self.features = int(spec["inputs"]["features"])
        self.outputs = int(spec["outputs"]["size"])
        self.a = {
            "roots": np.ascontiguousarray(t[p + ".root"], dtype=np.int32),
            "tree_output": np.ascontiguousarray(t[p + ".output"], dtype=np.int32),
            "feature": np.ascontiguousarray(t[p + ".feature"], dtype=np.int32),
            "threshold": np.ascontiguousarray(t[p + ".threshold"], dtype=np.float64),
            "left": np.ascontiguousarray(t[p + ".left"], dtype=np.int32),
            "right": np.ascontiguousarray(t[p + ".right"], dtype=np.int32),
            "value": np.ascontiguousarray(t[p + ".value"], dtype=np.float64),
            "flags": np.ascontiguousarray(t[p + ".flags"], dtype=np.uint8),
        }
        base = cfg.get("base_score", 0.0)
        base = [float(base)] * self.outputs if base is None or np.ndim(base) == 0 else [float(b) for b in base]
        self.a["base"] = np.asarray(base if base else [0.0] * self.outputs, dtype=np.float64)
        pre = spec.get("preprocess") or {}
        self.trees = len(self.a["roots"])
        f = _Forest()
        f.features, f.outputs, f.trees, f.nodes = self.features, self.outputs, self.trees, len(self.a["feature"])
        f.decision_le = int(cfg.get("decision", "le") == "le")
        f.cast_f32 = int(cfg.get("feature_cast", "f64") == "f32")
        f.mean = int(cfg.get("aggregate", "sum") == "mean")
        f.link = _LINKS[cfg.get("link", "identity")]
        f.sigmoid_scale = float(cfg.get("sigmoid_scale", 1.0) if cfg.get("sigmoid_scale") is not None else 1.0)
        for name in ("base", "roots", "tree_output", "feature", "threshold", "left", "right", "value", "flags"):
            setattr(f, name, self.a[name].ctypes.data)
        if pre.get("mean"):
            self.a["pre_mean"] = np.ascontiguousarray(t[pre["mean"]], dtype=np.float64)
            self.a["pre_scale"] = np.ascontiguousarray(t[pre["scale"]], dtype=np.float64)
            f.standardize, f.pre_mean, f.pre_scale = 1, self.a["pre_mean"].ctypes.data, self.a["pre_scale"].ctypes.data
        if pre.get("clip") is not None:
            f.clip, f.clip_lo, f.clip_hi = 1, float(pre["clip"][0]), float(pre["clip"][1])
        self.f = f

    def predict(self, x, threads: int = 1) -> np.ndarray:
        x, dtype = _input(x)
        x2 = x.reshape(-1, self.features)
        out = np.empty((len(x2), self.outputs), dtype=np.float64)
        self._lib.oracle_predict(ctypes.byref(self.f), dtype, x2.ctypes.data, len(x2), out.ctypes.data, threads)
        return out

    def leaves(self, x, threads: int = 1) -> np.ndarray:
        x, dtype = _input(x)
        x2 = x.reshape(-1, self.features)
        out = np.empty((len(x2), self.trees), dtype=np.int32)
        self._lib.oracle_leaves(ctypes.byref(self.f), dtype, x2.ctypes.data, len(x2), out.ctypes.data, threads)
        return out

def available_reference() -> bool:
    return REF_LIB.exists()


class Reference:
    """The reference runtime (oracle/_ref/libmontlok_ref.so) through its own C ABI."""

    _lib = None

    def __init__(self) -> None:
        if Reference._lib is None:
            if not REF_LIB.exists():
                raise FileNotFoundError(f"{REF_LIB} is not built (reference sources absent?)")
            lib = ctypes.CDLL(str(REF_LIB))
            lib.montlok_model_open_memory.restype = ctypes.c_int
            lib.montlok_model_open_memory.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]
            lib.montlok_model_predict.restype = ctypes.c_int
            lib.montlok_model_predict.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                                  ctypes.c_void_p]
            lib.montlok_model_close.argtypes = [ctypes.c_void_p]
            lib.montlok_last_error.restype = ctypes.c_char_p
            lib.montlok_set_threads.argtypes = [ctypes.c_int]
            lib.montlok_threads.restype = ctypes.c_int
            lib.ref_time_calls.restype = ctypes.c_int
            lib.ref_time_calls.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                           ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                           ctypes.c_void_p]
            Reference._lib = lib
        self.lib = Reference._lib

    def set_threads(self, n: int) -> None:
        self.lib.montlok_set_threads(int(n))

    def threads(self) -> int:
        return int(self.lib.montlok_threads())

    def open(self, model: bytes) -> ctypes.c_void_p:
        h = ctypes.c_void_p()
        status = self.lib.montlok_model_open_memory(model, len(model), ctypes.byref(h))
        if status:
            raise ValueError(f"reference rejects the model ({status}): {self.lib.montlok_last_error().decode()}")
        spec, _ = export.read(model)
        self._outputs = getattr(self, "_outputs", {})
        self._outputs[h.value] = int(spec["outputs"]["size"])
        return h

    def close(self, h: ctypes.c_void_p) -> None:
        self.lib.montlok_model_close(h)

    def predict(self, model: bytes, x, outputs: int | None = None) -> np.ndarray:
        x, dtype = _input(x)
        spec, _ = export.read(model)
        K = outputs or int(spec["outputs"]["size"])
        F = int(spec["inputs"]["features"])
        x2 = x.reshape(-1, F)
        out = np.empty((len(x2), K), dtype=np.float64)
        h = self.open(model)
        try:
            status = self.lib.montlok_model_predict(h, dtype, x2.ctypes.data, len(x2), out.ctypes.data)
            if status:
                raise RuntimeError(f"reference predict failed ({status}): {self.lib.montlok_last_error().decode()}")
        finally:
            self.close(h)
        return out

    def predict_handle(self, h: ctypes.c_void_p, x: np.ndarray, out: np.ndarray, dtype: int = 2) -> None:
        K = getattr(self, "_outputs", {}).get(h.value)
        if K is None or out.dtype != np.float64 or not out.flags.c_contiguous or out.size != len(x) * K:
            raise ValueError("out must be a C-contiguous float64 array of rows x outputs")
        status = self.lib.montlok_model_predict(h, dtype, x.ctypes.data, len(x), out.ctypes.data)
        if status:
            raise RuntimeError(f"reference predict failed ({status}): {self.lib.montlok_last_error().decode()}")

    def time_calls(self, h: ctypes.c_void_p, rows: np.ndarray, batch: int, iterations: int,
                   warmup: int) -> np.ndarray:
        """Nanoseconds of each of `iterations` predict calls of `batch` rows
        (float64 rows [count, batch * features] used in turn), after
        `warmup` untimed calls; the loop runs in C (ref_timer.c)."""
        rows = np.ascontiguousarray(rows, dtype=np.float64)
        features = rows.shape[1] // batch
        out = np.empty((batch, 64), dtype=np.float64)
        samples = np.empty(iterations, dtype=np.float64)
        status = self.lib.ref_time_calls(h, rows.ctypes.data, rows.shape[0], batch, features, iterations, warmup,
                                         out.ctypes.data, samples.ctypes.data)
        if status:
            raise RuntimeError(f"reference predict failed ({status}): {self.lib.montlok_last_error().decode()}")
        return samples

    def leaves(self, model: bytes, x, chunk: int = 4096) -> np.ndarray:
        """Leaf node index per (row, tree) as the reference selects them."""
        ids = leaf_id_model(model)
        spec, t = export.read(ids)
        T = int(spec["outputs"]["size"])
        x, _ = _input(x)
        F = int(spec["inputs"]["features"])
        x2 = x.reshape(-1, F)
        out = np.empty((len(x2), T), dtype=np.int32)
        for lo in range(0, len(x2), chunk):
            part = self.predict(ids, x2[lo:lo + chunk])
            out[lo:lo + chunk] = part.astype(np.int32)
            assert np.array_equal(part, out[lo:lo + chunk]), "leaf ids must come back exact"
        return out


def leaf_id_model(model: bytes) -> bytes:
    """The same trees with every leaf valued at its own node index, one output
    per tree, base 0, sum and identity: predict() returns leaf indices."""
    spec, t = export.read(model)
    cfg = dict(spec.get("config", {}) or {})
    p = cfg.get("tensors", "trees")
    T = len(t[p + ".root"])
    t = dict(t)
    value = np.arange(len(t[p + ".feature"]), dtype=np.float64)
    t[p + ".value"] = value
    t[p + ".output"] = np.arange(T, dtype=np.int32)
    cfg.update(aggregate="sum", link="identity", base_score=0.0, sigmoid_scale=1.0)
    spec = json.loads(json.dumps(spec))
    spec["outputs"] = {"size": T}
    spec["config"] = cfg
    return export.encode(spec, t)
