"""The C-ABI library: it loads, exports every entry point include/montlok/montlok.h
declares (and no other montlok_* symbol), and its host-side settings behave
like the reference's (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import montlok
from montlok import _core

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "montlok" / "montlok.h"


def declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"MONTLOK_API\s+[\w\s\*]+?\b(montlok_\w+)\s*\(", text))


def exported() -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(_core._LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.split()[-1].startswith("montlok_")}


def test_every_declared_symbol_is_exported_and_nothing_else():
    names = declared()
    assert len(names) >= 25
    assert names == exported()
    lib = ctypes.CDLL(str(_core._LIB_PATH))
    for name in names:
        assert hasattr(lib, name), name


def test_reference_model_api_is_present():
    # The entry points the reference's bindings call (include/montlok/montlok.h:75-113).
    reference = {"montlok_abi_version", "montlok_version", "montlok_last_error", "montlok_set_threads",
                 "montlok_threads", "montlok_set_latency_threads", "montlok_latency_threads", "montlok_families",
                 "montlok_model_open", "montlok_model_open_memory", "montlok_model_close", "montlok_model_get_info",
                 "montlok_model_family", "montlok_model_spec", "montlok_model_predict", "montlok_stream_open",
                 "montlok_stream_step", "montlok_stream_reset", "montlok_stream_close", "montlok_register_family",
                 "montlok_plugin_load"}
    assert reference <= exported()


def test_versions_and_families():
    info = montlok.build_info()
    assert info["abi"] == 1
    assert info["version"] == montlok.__version__ == "0.2.0"
    assert montlok.families() == ["tree_ensemble"]


def test_thread_settings():
    montlok.set_threads(3)
    assert montlok.threads() == 3
    montlok.set_threads(0)
    assert montlok.threads() >= 1
    for n in (0, 1, 7):
        montlok.set_latency_threads(n)
        assert montlok.latency_threads() == n
    with pytest.raises(ValueError):
        montlok.set_latency_threads(-1)
    with pytest.raises(ValueError):
        montlok.set_latency_threads(257)
    montlok.set_latency_threads(0)


def test_device_settings():
    montlok.set_devices(4)
    assert montlok.devices() == 4
    montlok.set_devices(0)
    assert montlok.devices() == 0
    with pytest.raises(ValueError):
        montlok.set_devices(-1)


def test_plugins_are_not_part_of_this_build():
    with pytest.raises(NotImplementedError):
        montlok.load_plugin("/nonexistent.so")
    lib = ctypes.CDLL(str(_core._LIB_PATH))
    assert lib.montlok_register_family(None) == 4


def test_null_arguments_are_invalid():
    lib = ctypes.CDLL(str(_core._LIB_PATH))
    lib.montlok_last_error.restype = ctypes.c_char_p
    handle = ctypes.c_void_p()
    assert lib.montlok_model_open(None, ctypes.byref(handle)) == 1
    assert lib.montlok_model_open_memory(None, ctypes.c_size_t(4), ctypes.byref(handle)) == 1
    assert lib.montlok_model_predict(None, 2, None, ctypes.c_size_t(1), None) == 1
    assert lib.montlok_model_get_info(None, None) == 1
    assert lib.montlok_stream_step(None, 2, None, None) == 1
    assert b"null" in lib.montlok_last_error()
