"""Build the in-tree C-ABI library ``libspecgrove_b200.so`` for sm_100a.

Every ``csrc/*.cu`` file is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared object
next to this file, so the library travels with the source tree.  Objects are
rebuilt only when a source or header is newer than the library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = PACKAGE_DIR.parent / "include"
BUILD_DIR = PACKAGE_DIR / "_build"
LIBRARY = PACKAGE_DIR / "libspecgrove_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(INCLUDE), "-I", str(CSRC),
]


def nvcc() -> str:
    path = shutil.which("nvcc")
    if path is None:
        cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
        if cand.exists():
            return str(cand)
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build specgrove_b200")
    return path


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in deps)


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    if _stale(obj, [src, *_headers()]):
        cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(lambda s: _compile(s, verbose), srcs))
    if _stale(LIBRARY, objs):
        tmp = LIBRARY.with_suffix(".so.tmp")
        # cudart is linked statically; driver entry points are resolved at run
        # time (cudaGetDriverEntryPoint), so the library loads without a GPU.
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
