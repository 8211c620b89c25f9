"""TEST INFRASTRUCTURE — compile the reference's own CUDA tree samplers into
``oracle/_ref/`` so GPU parity tests can run them beside the B200 kernels.

The reference ships its sampler kernels as the source strings ``CPP_SOURCE``
and ``CUDA_SOURCE`` of ``gbv_experiments/fused_tree_sampling.py``
(:10-100, :103-2058) and builds them with ``load_inline`` (:2061-2086).  This
recipe compiles those strings, unmodified, where they lie in a reference
checkout, for sm_100a (``TORCH_CUDA_ARCH_LIST=10.0a``), writing only into
``oracle/_ref/``.  The resulting extension module travels with the tree and is
loaded by path (``load_reference_sampler``); nothing reads the reference
checkout at run time.

    python oracle/build_ref.py --reference <specgrove checkout>
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import time
from pathlib import Path

REF_DIR = Path(__file__).resolve().parent / "_ref"
MODULE = "specgrove_reference_sampler"
FUNCTIONS = ["fused_tree_sample_scan_cuda", "fused_tree_sample_sparse_exit_batched_cuda",
             "fused_tree_follow_cuda", "fused_tree_sample_logits_scan_batched_cuda"]


def build(reference: str) -> Path:
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    sys.path.insert(0, str(Path(reference) / "code" / "natural" / "src"))
    from gbv_experiments import fused_tree_sampling as fts
    from torch.utils.cpp_extension import load_inline
    REF_DIR.mkdir(exist_ok=True)
    t0 = time.time()
    load_inline(name=MODULE, cpp_sources=[fts.CPP_SOURCE], cuda_sources=[fts.CUDA_SOURCE],
                functions=FUNCTIONS, extra_cflags=["-O3"], extra_cuda_cflags=["-O3"], with_cuda=True,
                verbose=False, build_directory=str(REF_DIR))
    print(f"built {MODULE} in {time.time() - t0:.0f}s")
    return library_path()


def library_path() -> Path:
    return REF_DIR / f"{MODULE}.so"


def load_reference_sampler():
    """Import the prebuilt reference extension (None when it was not built)."""
    path = library_path()
    if not path.exists():
        return None
    import torch  # noqa: F401  (libtorch symbols)
    spec = importlib.util.spec_from_file_location(MODULE, str(path))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    print(build(ap.parse_args().reference))
