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
        # The soname lets the torch-op extension's dependency resolve to the
        # copy ctypes already loaded (one set of library state per process).
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-Xlinker", f"-soname={LIBRARY.name}", "-o", str(tmp),
               *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIBRARY)
    build_torch_ops(verbose)
    return LIBRARY


TORCH_OPS_SOURCE = CSRC / "torch_ops.cpp"
TORCH_OPS = PACKAGE_DIR / "_torch_ops.so"


def build_torch_ops(verbose: bool = False) -> Path:
    """The torch custom-op extension (torch.ops.specgrove_b200.*): host C++
    compiled by g++ against torch's headers, linked to the C-ABI library."""
    if not _stale(TORCH_OPS, [TORCH_OPS_SOURCE, LIBRARY, *sorted(INCLUDE.glob("*.h"))]):
        return TORCH_OPS
    import torch
    from torch.utils import cpp_extension as ce
    torch_dir = Path(torch.__file__).resolve().parent
    includes = [torch_dir / "include", torch_dir / "include" / "torch" / "csrc" / "api" / "include",
                Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include", INCLUDE]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_OPS.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_torch_ops", *[f"-I{p}" for p in includes], str(TORCH_OPS_SOURCE),
           "-o", str(tmp), f"-L{torch_dir / 'lib'}", f"-L{PACKAGE_DIR}", f"-l:{LIBRARY.name}",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_dir / 'lib'}"]
    del ce
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, TORCH_OPS)
    return TORCH_OPS


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
