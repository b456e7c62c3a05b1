"""montlok._core: the Python binding, over the C ABI of libmontlok.so.

Mirrors the reference binding (montlok.cpp src/python/module.cpp:304-386):
``Model.open/from_bytes``, the ``family/spec_json/features/sequence/outputs/
streamable/preprocess`` properties, ``predict(x, out=None)``, ``stream()``,
``bench`` and the error mapping (IO -> OSError, UNSUPPORTED ->
NotImplementedError, FORMAT -> FormatError, INVALID/SHAPE -> ValueError,
others -> RuntimeError). Every call goes through ctypes, which releases the
GIL while the library runs.

The library is built in-tree (montlok.cpp_b200/build.py) next to this file;
importing without it raises ImportError: there is no pure-Python path.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Any

import numpy as np

_LIB_PATH = Path(os.environ.get("MONTLOK_LIBRARY", Path(__file__).with_name("libmontlok.so")))
if not _LIB_PATH.exists():
    raise ImportError(f"montlok: {_LIB_PATH} is missing; build it with `python montlok.cpp_b200/build.py`")
lib = ctypes.CDLL(str(_LIB_PATH))

_vp, _sz, _i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int


def _sig(name: str, res, *args) -> None:
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = list(args)


class _Info(ctypes.Structure):
    _fields_ = [("features", ctypes.c_uint32), ("sequence", ctypes.c_uint32), ("outputs", ctypes.c_uint32),
                ("flags", ctypes.c_uint32)]


_sig("montlok_abi_version", ctypes.c_uint32)
_sig("montlok_version", ctypes.c_char_p)
_sig("montlok_last_error", ctypes.c_char_p)
_sig("montlok_set_threads", None, _i32)
_sig("montlok_threads", _i32)
_sig("montlok_set_latency_threads", _i32, _i32)
_sig("montlok_latency_threads", _i32)
_sig("montlok_families", ctypes.c_char_p)
_sig("montlok_model_open", _i32, ctypes.c_char_p, ctypes.POINTER(_vp))
_sig("montlok_model_open_memory", _i32, ctypes.c_char_p, _sz, ctypes.POINTER(_vp))
_sig("montlok_model_close", None, _vp)
_sig("montlok_model_get_info", _i32, _vp, ctypes.POINTER(_Info))
_sig("montlok_model_family", ctypes.c_char_p, _vp)
_sig("montlok_model_spec", ctypes.c_char_p, _vp)
_sig("montlok_model_predict", _i32, _vp, _i32, _vp, _sz, _vp)
_sig("montlok_model_predict_device", _i32, _vp, _i32, _vp, _sz, _vp, _vp)
_sig("montlok_model_predict_leaves", _i32, _vp, _i32, _vp, _sz, _vp)
_sig("montlok_model_predict_leaves_device", _i32, _vp, _i32, _vp, _sz, _vp, _vp)
_sig("montlok_model_trees", _i32, _vp, ctypes.POINTER(ctypes.c_uint32))
_sig("montlok_model_device_status", _i32, _vp)
_sig("montlok_model_kernel", _i32, _vp, _sz, ctypes.POINTER(ctypes.c_char_p))
_sig("montlok_stream_open", _i32, _vp, _sz, ctypes.POINTER(_vp))
_sig("montlok_stream_step", _i32, _vp, _i32, _vp, _vp)
_sig("montlok_stream_reset", _i32, _vp)
_sig("montlok_stream_close", None, _vp)
_sig("montlok_plugin_load", _i32, ctypes.c_char_p)
_sig("montlok_set_devices", _i32, _i32)
_sig("montlok_devices", _i32)
_sig("montlok_device_count", _i32)
_sig("montlok_bench_predict", _i32, _vp, _i32, _vp, _sz, _sz, _sz, _sz, _vp, ctypes.POINTER(ctypes.c_double))

FLOAT32, FLOAT64 = 1, 2


class FormatError(ValueError):
    """A malformed or foreign model file."""


FormatError.__module__ = "montlok._core"


def _raise(status: int) -> None:
    message = (lib.montlok_last_error() or b"").decode(errors="replace")
    if status == 2:
        raise OSError(message)
    if status == 4:
        raise NotImplementedError(message)
    if status == 3:
        raise FormatError(message)
    if status in (1, 5):
        raise ValueError(message)
    raise RuntimeError(message)


def _check(status: int) -> None:
    if status != 0:
        _raise(status)


def version() -> str:
    return lib.montlok_version().decode()


def abi_version() -> int:
    return int(lib.montlok_abi_version())


def set_threads(threads: int) -> None:
    """Host threads that stage pageable inputs; 0 means one per hardware thread."""
    lib.montlok_set_threads(int(threads))


def threads() -> int:
    return int(lib.montlok_threads())


def set_latency_threads(threads: int) -> None:
    _check(lib.montlok_set_latency_threads(int(threads)))


def latency_threads() -> int:
    return int(lib.montlok_latency_threads())


def families() -> list[str]:
    text = lib.montlok_families().decode()
    return [name for name in text.split(",") if name]


def load_plugin(path: str) -> None:
    _check(lib.montlok_plugin_load(os.fsencode(path)))


def set_devices(count: int) -> None:
    """GPUs that host-buffer predictions split their rows over (0: the current one)."""
    _check(lib.montlok_set_devices(int(count)))


def devices() -> int:
    return int(lib.montlok_devices())


def device_count() -> int:
    return int(lib.montlok_device_count())


def _as_input(x: Any) -> np.ndarray:
    a = np.asarray(x)
    if a.dtype == np.float32:
        return np.ascontiguousarray(a)
    return np.ascontiguousarray(a, dtype=np.float64)


def _output(out: Any, shape: tuple[int, ...]) -> np.ndarray:
    size = int(np.prod(shape))
    if out is None:
        return np.empty(shape, dtype=np.float64)
    if not isinstance(out, np.ndarray):
        raise TypeError("out must be a NumPy array")
    if out.dtype != np.float64 or not out.flags.c_contiguous or not out.flags.writeable or out.size != size:
        raise ValueError(f"out must be a writable C-contiguous float64 array of {size} values")
    return out


def _cuda_pointer(a: Any) -> int | None:
    iface = getattr(a, "__cuda_array_interface__", None)
    return None if iface is None else int(iface["data"][0])


class Model:
    """A loaded model (reference module.cpp:350-372)."""

    def __init__(self, handle: ctypes.c_void_p) -> None:
        self._h = handle
        info = _Info()
        _check(lib.montlok_model_get_info(handle, ctypes.byref(info)))
        self._info = info
        trees = ctypes.c_uint32()
        _check(lib.montlok_model_trees(handle, ctypes.byref(trees)))
        self._trees = int(trees.value)

    def __del__(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value and lib is not None:
            lib.montlok_model_close(h)
            self._h = None

    @staticmethod
    def open(path: str) -> "Model":
        h = _vp()
        _check(lib.montlok_model_open(os.fsencode(path), ctypes.byref(h)))
        return Model(h)

    @staticmethod
    def from_bytes(data: bytes) -> "Model":
        data = bytes(data)
        h = _vp()
        _check(lib.montlok_model_open_memory(data, len(data), ctypes.byref(h)))
        return Model(h)

    @property
    def family(self) -> str:
        return lib.montlok_model_family(self._h).decode()

    @property
    def spec_json(self) -> str:
        return lib.montlok_model_spec(self._h).decode()

    @property
    def features(self) -> int:
        return int(self._info.features)

    @property
    def sequence(self) -> int:
        return int(self._info.sequence)

    @property
    def outputs(self) -> int:
        return int(self._info.outputs)

    @property
    def trees(self) -> int:
        return self._trees

    @property
    def streamable(self) -> bool:
        return bool(self._info.flags & 1)

    @property
    def preprocess(self) -> bool:
        return bool(self._info.flags & 2)

    def _rows(self, x: np.ndarray) -> tuple[bool, int]:
        if x.ndim == 1:
            single, batch = True, 1
        elif x.ndim == 2:
            single, batch = False, int(x.shape[0])
        else:
            raise ValueError("expected [batch, features] or [features]")
        if x.shape[-1] != self.features:
            raise ValueError(f"input shape does not match the model: features={self.features}, sequence={self.sequence}")
        return single, batch

    def predict(self, x: Any, out: Any = None) -> Any:
        """[batch, features] (or [features]) -> [batch, outputs] (or [outputs]).
        float32 inputs stay float32, anything else becomes float64. Arrays with
        ``__cuda_array_interface__`` (e.g. torch CUDA tensors, contiguous) run in
        place on the device; ``out`` must then be a float64 device array too."""
        if _cuda_pointer(x) is not None:
            return self._predict_cuda(x, out)
        x = _as_input(x)
        single, batch = self._rows(x)
        shape = (self.outputs,) if single else (batch, self.outputs)
        result = _output(out, shape)
        dtype = FLOAT32 if x.dtype == np.float32 else FLOAT64
        _check(lib.montlok_model_predict(self._h, dtype, x.ctypes.data, batch, result.ctypes.data))
        return result

    def _predict_cuda(self, x: Any, out: Any) -> Any:
        ix = x.__cuda_array_interface__
        typestr = ix["typestr"]
        if typestr not in ("<f4", "<f8"):
            raise ValueError("device inputs must be float32 or float64")
        shape = tuple(ix["shape"])
        if ix.get("strides") not in (None, (shape[-1] * int(typestr[2]), int(typestr[2]))) and len(shape) == 2:
            raise ValueError("device inputs must be C-contiguous")
        batch = 1 if len(shape) == 1 else int(shape[0])
        if shape[-1] != self.features or len(shape) not in (1, 2):
            raise ValueError(f"input shape does not match the model: features={self.features}")
        if out is None or _cuda_pointer(out) is None:
            raise ValueError("device inputs need a float64 device `out` of batch * outputs values")
        io = out.__cuda_array_interface__
        if io["typestr"] != "<f8" or int(np.prod(io["shape"])) != batch * self.outputs:
            raise ValueError(f"out must be a float64 device array of {batch * self.outputs} values")
        stream = ix.get("stream") or 0
        if stream in (1, 2):  # legacy / per-thread default stream markers
            stream = 0
        _check(lib.montlok_model_predict_device(self._h, FLOAT32 if typestr == "<f4" else FLOAT64, ix["data"][0],
                                                batch, io["data"][0], stream))
        return out

    def predict_device(self, x_ptr: int, batch: int, out_ptr: int, dtype: int = FLOAT64, stream: int = 0) -> None:
        """Raw device pointers on the current CUDA device; queued on `stream`."""
        _check(lib.montlok_model_predict_device(self._h, int(dtype), x_ptr, int(batch), out_ptr, stream))

    def check_device_status(self) -> None:
        """Raises RuntimeError when a device-buffer predict on the current
        device gave up waiting for its tree data since the last check (its
        rows were not written); call it after synchronising those calls."""
        _check(lib.montlok_model_device_status(self._h))

    def kernel(self, batch: int) -> str:
        """The kernel a predict of `batch` rows runs on the current device."""
        name = ctypes.c_char_p()
        _check(lib.montlok_model_kernel(self._h, int(batch), ctypes.byref(name)))
        return (name.value or b"").decode()

    def predict_leaves(self, x: Any) -> np.ndarray:
        """int32 node index of the leaf each row reaches in each tree: [batch, trees]."""
        x = _as_input(x)
        single, batch = self._rows(x)
        leaves = np.empty((batch, self.trees), dtype=np.int32)
        dtype = FLOAT32 if x.dtype == np.float32 else FLOAT64
        _check(lib.montlok_model_predict_leaves(self._h, dtype, x.ctypes.data, batch, leaves.ctypes.data))
        return leaves[0] if single else leaves

    def stream(self, batch: int = 1) -> "Stream":
        h = _vp()
        _check(lib.montlok_stream_open(self._h, int(batch), ctypes.byref(h)))
        return Stream(self, h, int(batch))


class Stream:
    """A stateless stream of a tree model (reference trees.cpp:199-208)."""

    def __init__(self, model: Model, handle: ctypes.c_void_p, batch: int) -> None:
        self._model, self._h, self._batch = model, handle, batch

    def __del__(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value and lib is not None:
            lib.montlok_stream_close(h)
            self._h = None

    @property
    def batch(self) -> int:
        return self._batch

    def step(self, x: Any, out: Any = None) -> np.ndarray:
        x = _as_input(x)
        single = x.ndim == 1
        if not (single and self._batch == 1) and not (x.ndim == 2 and x.shape[0] == self._batch):
            raise ValueError("expected [batch, features] (or [features] for a batch of 1)")
        if x.shape[-1] != self._model.features:
            raise ValueError(f"expected {self._model.features} features")
        shape = (self._model.outputs,) if single else (self._batch, self._model.outputs)
        result = _output(out, shape)
        _check(lib.montlok_stream_step(self._h, FLOAT32 if x.dtype == np.float32 else FLOAT64, x.ctypes.data,
                                       result.ctypes.data))
        return result

    def reset(self) -> None:
        _check(lib.montlok_stream_reset(self._h))


def bench(model: Model, rows: Any, batch: int = 1, iterations: int = 20000, stream: bool = False) -> tuple:
    """Per-call latency of montlok_model_predict (reference module.cpp:115-150):
    ``rows`` holds [count, batch * features] inputs used in turn; returns
    (nanoseconds of each timed call, mean nanoseconds of back-to-back calls).
    The timing loop runs inside the library, after max(1000, iterations / 10)
    warm-up calls."""
    rows = np.ascontiguousarray(rows, dtype=np.float64)
    width = batch * model.features
    if batch <= 0 or iterations <= 0 or rows.ndim != 2 or rows.shape[0] == 0 or rows.shape[1] != width:
        raise ValueError(f"rows must be [count, {width}] and batch, iterations positive")
    samples = np.empty(iterations, dtype=np.float64)
    mean = ctypes.c_double()
    warmup = max(1000, iterations // 10)
    _check(lib.montlok_bench_predict(model._h, FLOAT64, rows.ctypes.data, rows.shape[0], batch, iterations, warmup,
                                     samples.ctypes.data, ctypes.byref(mean)))
    return samples, mean.value
