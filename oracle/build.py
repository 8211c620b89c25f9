"""TEST INFRASTRUCTURE — build the CPU oracle library ``oracle/_build/libsg_oracle.so``.

The oracle is the checker for the CUDA path (tests, smoke, bench CPU baseline);
the product never loads it.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
BUILD_DIR = ORACLE_DIR / "_build"
LIBRARY = BUILD_DIR / "libsg_oracle.so"
SOURCES = [ORACLE_DIR / "sg_oracle.c"]


def build(verbose: bool = False) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    if LIBRARY.exists() and all(LIBRARY.stat().st_mtime >= s.stat().st_mtime for s in SOURCES):
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = ["gcc", "-O2", "-std=c11", "-fopenmp", "-fPIC", "-shared", "-o", str(tmp),
           *map(str, SOURCES), "-lm"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose=True))
