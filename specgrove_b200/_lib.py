"""ctypes binding of the in-tree C-ABI library ``libspecgrove_b200.so``.

The library is the only compute path: there is no CPU fallback.  Importing a
function from here when the library has not been built raises immediately.
"""
from __future__ import annotations

import ctypes
from ctypes import c_double, c_int32, c_int64, c_uint64, c_void_p
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "libspecgrove_b200.so"

SG_OK = 0
SG_ERR_INVALID_ARGUMENT = 1
SG_ERR_CUDA = 2
SG_ERR_TREE = 3
SG_ERR_PROBABILITY = 4
SG_ERR_CAPACITY = 5
SG_ERR_UNSUPPORTED = 6
SG_ERR_WORKSPACE = 7

SG_RULE_SCAN = 0
SG_RULE_SPARSE_EXIT = 1

# name -> (restype, argtypes); mirrors include/specgrove_b200.h
_SIGNATURES = {
    "sg_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "sg_last_error": (ctypes.c_char_p, []),
    "sg_version": (ctypes.c_int, []),
    "sg_launch_count": (c_uint64, []),
    "sg_tree_accept_probs": (ctypes.c_int, [
        c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
        c_void_p, c_int32, c_uint64, c_void_p, c_void_p, c_void_p, c_void_p]),
    "sg_tree_accept_logits": (ctypes.c_int, [
        c_void_p, c_int32, c_int64, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_double,
        c_void_p, c_int32, c_uint64, c_void_p, c_void_p, c_void_p, c_void_p]),
    "sg_tree_follow": (ctypes.c_int, [
        c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p,
        c_void_p]),
    "sg_kv_commit": (ctypes.c_int, [
        c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
        c_int32, c_int32, c_void_p, c_void_p]),
    "sg_kv_commit_accepted": (ctypes.c_int, [
        c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
        c_int32, c_int32, c_void_p, c_void_p]),
    "sg_gemm_bf16": (ctypes.c_int, [
        c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32, c_int32, c_int32,
        c_void_p, c_int64, c_void_p, c_void_p]),
    "sg_tree_verify_terminal_mass_workspace_bytes": (ctypes.c_size_t, [c_int64]),
    "sg_tree_verify_terminal_mass": (ctypes.c_int, [
        c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int32, c_int64, c_int32, c_void_p, c_int32, c_uint64,
        c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_void_p]),
    "sg_gemm_split_workspace_bytes": (ctypes.c_size_t, []),
    "sg_gemm_split_workspace_init": (ctypes.c_int, [c_void_p, ctypes.c_size_t, c_void_p]),
    "sg_gemm_bf16_ws": (ctypes.c_int, [
        c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32, c_int32, c_int32,
        c_void_p, c_int64, c_void_p, c_void_p, ctypes.c_size_t, c_void_p]),
    "sg_allocate_tiers": (ctypes.c_int, [
        c_int32, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_double, c_void_p, c_void_p, c_int32,
        c_void_p]),
    "sg_allocate_tiers_device_workspace_bytes": (ctypes.c_size_t, [c_int32, c_int32]),
    "sg_allocate_tiers_device": (ctypes.c_int, [
        c_int32, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_double, c_void_p, c_void_p, c_int32,
        c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_void_p]),
    "sg_proposal_topk": (ctypes.c_int, [
        c_void_p, c_int32, c_int64, c_int32, c_int64, c_int32, c_int32, c_int32, c_double, c_void_p, c_void_p,
        c_void_p, c_void_p]),
    "sg_build_draft_trees": (ctypes.c_int, [
        c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_double,
        c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "sg_pack_tree_wave": (ctypes.c_int, [
        c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_int64, c_void_p, c_void_p, c_void_p,
        c_void_p, c_void_p]),
    "sg_lm_head_sample_workspace_bytes": (ctypes.c_size_t, [c_int32, c_int32, c_int32]),
    "sg_lm_head_sample": (ctypes.c_int, [
        c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, ctypes.c_float, c_void_p, c_void_p, c_uint64,
        ctypes.c_float, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_void_p]),
    "sg_lm_head_sample_bf16": (ctypes.c_int, [
        c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_uint64, ctypes.c_float, c_void_p,
        c_void_p, c_void_p, ctypes.c_size_t, c_void_p]),
    "sg_lm_head_sample_static": (ctypes.c_int, [
        c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, ctypes.c_float, c_void_p, c_void_p, c_uint64,
        ctypes.c_float, c_void_p, c_void_p, c_void_p]),
}

SG_EPI_STORE_BF16 = 0
SG_EPI_STORE_F32 = 1
SG_EPI_RESIDUAL = 2
SG_EPI_SWIGLU = 3

_lib = None


class SpecgroveError(RuntimeError):
    """A non-zero sg_status returned by the C ABI."""

    def __init__(self, status: int, where: str):
        lib = load()
        detail = lib.sg_last_error().decode(errors="replace")
        text = lib.sg_status_string(status).decode(errors="replace")
        super().__init__(f"{where}: {text} (status {status}){': ' + detail if detail else ''}")
        self.status = status


def load() -> ctypes.CDLL:
    """Load the library once; raise if it was not built."""
    global _lib
    if _lib is None:
        if not LIBRARY_PATH.exists():
            raise ImportError(
                f"{LIBRARY_PATH.name} is not built; run `python -m specgrove_b200.build` "
                "(the CUDA library is required, there is no CPU fallback)")
        lib = ctypes.CDLL(str(LIBRARY_PATH))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def check(status: int, where: str) -> None:
    if status != SG_OK:
        raise SpecgroveError(status, where)


# Entry points taking struct descriptors; bound with their ctypes structures
# in specgrove_b200.engine.
STRUCT_SYMBOLS = ["sg_engine_create", "sg_engine_destroy", "sg_engine_workspace_bytes", "sg_verify_pass",
                  "sg_draft_engine_create", "sg_draft_pass"]


def exported_symbols() -> list[str]:
    return list(_SIGNATURES) + STRUCT_SYMBOLS


def ptr(tensor) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if tensor is None else tensor.data_ptr()


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def launch_count() -> int:
    return int(load().sg_launch_count())
