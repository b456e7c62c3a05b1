"""Builds libmontlok.so: the C ABI (include/montlok/montlok.h) over the CUDA
kernels, for sm_100a only.

    python montlok.cpp_b200/build.py          # incremental
    python montlok.cpp_b200/build.py --clean

Host sources (csrc/core/*.cpp) build with g++ -std=c++17, CUDA sources
(csrc/cuda/*.cu) with nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo,
and the library links the CUDA runtime statically, so it needs only the driver
at run time. The library lands next to the Python package
(python/montlok/libmontlok.so), where montlok._core loads it; objects go to
_build/. Only the montlok_* entry points are exported.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
OUT = HERE / "_build"
LIB = HERE / "python" / "montlok" / "libmontlok.so"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA / "bin" / "nvcc")
CXX = os.environ.get("CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INCLUDES = ["-I", str(REPO / "include"), "-I", str(CSRC)]
CXXFLAGS = ["-std=c++17", "-O2", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra", "-Wno-unused-parameter"]
# -fmad=false: no float multiply-add contraction anywhere in device code, so
# every float64 operation of the sums and link rounds on its own.
NVCCFLAGS = ["-std=c++17", "-O3", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC,-fvisibility=hidden",
             "-Xptxas", "-v"] + ARCH


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], log: Path | None = None) -> None:
    result = subprocess.run(cmd, capture_output=True, text=True)
    if log is not None:
        log.write_text(result.stdout + result.stderr)
    if result.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + result.stdout + result.stderr)
        raise SystemExit(f"build failed: {cmd[0]} exited {result.returncode}")


def build(clean: bool = False, verbose: bool = False) -> Path:
    if clean and OUT.exists():
        shutil.rmtree(OUT)
    OUT.mkdir(parents=True, exist_ok=True)
    headers = sorted(p for pattern in ("*.h", "*.hpp", "*.cuh") for p in CSRC.rglob(pattern)) + sorted(
        (REPO / "include").rglob("*.h"))
    objects = []
    for src in sorted((CSRC / "core").glob("*.cpp")):
        obj = OUT / (src.stem + ".o")
        if _stale(obj, [src, *headers]):
            _run([CXX, *CXXFLAGS, *INCLUDES, "-c", str(src), "-o", str(obj)])
            if verbose:
                print("built", obj.name)
        objects.append(obj)
    for src in sorted((CSRC / "cuda").glob("*.cu")):
        obj = OUT / (src.stem + ".cu.o")
        if _stale(obj, [src, *headers]):
            _run([NVCC, *NVCCFLAGS, *INCLUDES, "-c", str(src), "-o", str(obj)], log=OUT / (src.stem + ".ptxas.txt"))
            if verbose:
                print("built", obj.name)
        objects.append(obj)
    if _stale(LIB, objects):
        _run([CXX, "-shared", "-o", str(LIB), *map(str, objects), "-L", str(CUDA / "lib64"), "-lcudart_static",
              "-lrt", "-ldl", "-lpthread", "-Wl,--exclude-libs,ALL", "-Wl,-soname,libmontlok.so"])
        if verbose:
            print("linked", LIB)
    return LIB


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--clean", action="store_true")
    args = parser.parse_args()
    print(build(clean=args.clean, verbose=True))


if __name__ == "__main__":
    main()
