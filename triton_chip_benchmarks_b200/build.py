"""Build recipe for libtcb.so, the sm_100a probe library.

Compiles every ``csrc/*.cu`` for ``sm_100a`` with nvcc (object files in
``_build/`` beside this file, incremental on source/header timestamps) and
links them, with the CUDA runtime linked statically, into
``triton_chip_benchmarks_b200/libtcb.so``.  Run ``python -m
triton_chip_benchmarks_b200.build`` or call :func:`build`.
"""

from __future__ import annotations

import concurrent.futures
import os
from pathlib import Path
import shutil
import subprocess
import sys

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PACKAGE_DIR / "_build"
LIBRARY = PACKAGE_DIR / "libtcb.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc_path() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found; set CUDA_HOME or put nvcc on PATH")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in deps)


def _compile(nvcc: str, source: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (source.stem + ".o")
    if not _stale(obj, [source, *_headers()]):
        return obj
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC),
           "-c", str(source), "-o", str(obj)]
    if verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stdout}\n{result.stderr}")
    if verbose and (result.stdout or result.stderr):
        print(result.stdout + result.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile and link libtcb.so; returns its path."""
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
        objects = list(pool.map(lambda src: _compile(nvcc, src, verbose), sources))
    if _stale(LIBRARY, objects):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(LIBRARY),
               *map(str, objects)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
