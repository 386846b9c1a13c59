"""Builds libq38.so, the sm_100a kernels behind include/q38.h, in the package directory.

Each csrc/*.cu is compiled separately (relocatable device code, so the device error word is one
symbol for the whole library) into _build/, then nvcc links the shared library. Only sources newer
than their object are recompiled. nvcc cross-compiles for sm_100a on a machine without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PACKAGE_DIR / "_build"
LIBRARY = PACKAGE_DIR / "libq38.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMPILE_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-rdc=true",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-warn-spills",
]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit's bin on PATH")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers_mtime() -> float:
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in headers), default=0.0)


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc(), *ARCH_FLAGS, *COMPILE_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{result.stdout}\n{result.stderr}")
    if verbose and (result.stdout or result.stderr):
        print(result.stdout + result.stderr, flush=True)
    return obj


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compiles what changed and links libq38.so. Returns the library path."""
    BUILD_DIR.mkdir(exist_ok=True)
    sources = _sources()
    header_time = _headers_mtime()
    stale = []
    for src in sources:
        obj = BUILD_DIR / (src.stem + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, header_time):
            stale.append(src)
    with ThreadPoolExecutor(max_workers=min(8, max(1, len(stale)))) as pool:
        list(pool.map(lambda s: _compile(s, verbose), stale))
    objects = [BUILD_DIR / (s.stem + ".o") for s in sources]
    if stale or not LIBRARY.exists() or LIBRARY.stat().st_mtime < max(o.stat().st_mtime for o in objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-rdc=true", *map(str, objects), "-o", str(tmp), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{result.stdout}\n{result.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose=True))
