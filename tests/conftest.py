"""Test setup: import paths for the package (montlok.cpp_b200/python) and the
CPU oracle (oracle/), the `gpu` marker, and an in-tree build of the library
and the oracle when they are missing."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT / "montlok.cpp_b200" / "python", ROOT / "oracle", ROOT / "tests", ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the CUDA kernels")
    lib = ROOT / "montlok.cpp_b200" / "python" / "montlok" / "libmontlok.so"
    if not lib.exists():
        sys.path.insert(0, str(ROOT / "montlok.cpp_b200"))
        import build  # noqa: PLC0415

        build.build()
    if not (ROOT / "oracle" / "_build" / "libmontlok_oracle.so").exists():
        import oracle  # noqa: PLC0415

        oracle.build()


@pytest.fixture(scope="session")
def gpu():
    """Skips (CPU runs) unless a CUDA device is visible to the library."""
    import montlok

    if montlok.device_count() == 0:
        pytest.skip("no CUDA device")
    return montlok.device_count()
