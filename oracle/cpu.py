"""TEST INFRASTRUCTURE — numpy/ctypes front end of the C oracle (``sg_oracle.c``).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may call
these functions.  Argument meaning follows include/specgrove_b200.h, with host
numpy arrays instead of device pointers.
"""
from __future__ import annotations

import ctypes
from ctypes import c_double, c_float, c_int32, c_int64, c_uint64, c_void_p, POINTER

import numpy as np

from . import build as _build

RULE_SCAN = 0
RULE_SPARSE_EXIT = 1
ARITH_EXACT = 0
ARITH_FP64 = 1

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.LIBRARY
        if not path.exists():
            path = _build.build()
        L = ctypes.CDLL(str(path))
        L.sgo_tree_accept_probs.restype = ctypes.c_int
        L.sgo_tree_accept_probs.argtypes = [
            c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p,
            c_int32, c_uint64, c_void_p, c_int32, c_void_p]
        L.sgo_tree_accept_logits.restype = ctypes.c_int
        L.sgo_tree_accept_logits.argtypes = [
            c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_double, c_void_p, c_int32,
            c_uint64, c_void_p, c_int32, c_void_p]
        L.sgo_tree_follow.restype = ctypes.c_int
        L.sgo_tree_follow.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                      c_void_p]
        L.sgo_kv_commit.restype = ctypes.c_int
        L.sgo_kv_commit.argtypes = [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64,
                                    c_void_p, c_void_p, c_int64]
        L.sgo_tree_verify_terminal_mass.restype = ctypes.c_int
        L.sgo_tree_verify_terminal_mass.argtypes = [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int32,
                                                    c_int32, c_void_p, c_int32, c_uint64, c_void_p, c_void_p]
        L.sgo_node_uniforms.restype = None
        L.sgo_node_uniforms.argtypes = [c_uint64, c_uint64, ctypes.c_uint32, POINTER(c_double),
                                        POINTER(c_double)]
        L.sgo_mass_of.restype = ctypes.c_int
        L.sgo_mass_of.argtypes = [c_float, POINTER(c_uint64), POINTER(c_uint64)]
        L.sgo_mass_scale.restype = None
        L.sgo_mass_scale.argtypes = [c_double, c_uint64, c_uint64, POINTER(c_uint64),
                                     POINTER(c_uint64)]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def accept_probs(probs: np.ndarray, row_offsets, parents, tokens, max_depth: int, rule: int = RULE_SCAN,
                 uniforms: np.ndarray | None = None, seed: int = 0, request_ids=None,
                 arith: int = ARITH_EXACT) -> tuple[np.ndarray, int]:
    """Batched acceptance walk; returns (out [trees, max_depth+2] int64, status)."""
    probs = np.ascontiguousarray(probs, dtype=np.float32)
    row_offsets = np.ascontiguousarray(row_offsets, dtype=np.int64)
    parents = np.ascontiguousarray(parents, dtype=np.int64)
    tokens = np.ascontiguousarray(tokens, dtype=np.int64)
    trees = len(row_offsets) - 1
    stride = 0
    if uniforms is not None:
        uniforms = np.ascontiguousarray(uniforms, dtype=np.float64).reshape(trees, -1)
        stride = uniforms.shape[1]
    if request_ids is not None:
        request_ids = np.ascontiguousarray(request_ids, dtype=np.int64)
    out = np.full((trees, max_depth + 2), -1, dtype=np.int64)
    st = lib().sgo_tree_accept_probs(_p(probs), probs.shape[1], _p(row_offsets), _p(parents),
                                     _p(tokens), trees, max_depth, rule, _p(uniforms), stride,
                                     seed, _p(request_ids), arith, _p(out))
    return out, st


def accept_logits(logits: np.ndarray, row_offsets, parents, tokens, max_depth: int, temperature: float = 1.0,
                  uniforms: np.ndarray | None = None, seed: int = 0, request_ids=None,
                  arith: int = ARITH_EXACT) -> tuple[np.ndarray, int]:
    """Direct-logits walk (fp32 logits; bf16 widened exactly by the caller);
    returns (out [trees, max_depth+2] int64, status)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    row_offsets = np.ascontiguousarray(row_offsets, dtype=np.int64)
    parents = np.ascontiguousarray(parents, dtype=np.int64)
    tokens = np.ascontiguousarray(tokens, dtype=np.int64)
    trees = len(row_offsets) - 1
    stride = 0
    if uniforms is not None:
        uniforms = np.ascontiguousarray(uniforms, dtype=np.float64).reshape(trees, -1)
        stride = uniforms.shape[1]
    if request_ids is not None:
        request_ids = np.ascontiguousarray(request_ids, dtype=np.int64)
    out = np.full((trees, max_depth + 2), -1, dtype=np.int64)
    st = lib().sgo_tree_accept_logits(_p(logits), logits.shape[1], _p(row_offsets), _p(parents), _p(tokens), trees,
                                      max_depth, float(temperature), _p(uniforms), stride, seed, _p(request_ids),
                                      arith, _p(out))
    return out, st


def terminal_mass(probs: np.ndarray, row_offsets, parents, tokens, max_depth: int,
                  uniforms: np.ndarray | None = None, seed: int = 0, request_ids=None) -> tuple[np.ndarray, int]:
    """Terminal-mass verifier (sampling.py:542-735) over packed rows; returns
    (out [trees, max_depth+2] int64, status)."""
    probs = np.ascontiguousarray(probs, dtype=np.float32)
    row_offsets = np.ascontiguousarray(row_offsets, dtype=np.int64)
    parents = np.ascontiguousarray(parents, dtype=np.int64)
    tokens = np.ascontiguousarray(tokens, dtype=np.int64)
    trees = len(row_offsets) - 1
    stride = 0
    if uniforms is not None:
        uniforms = np.ascontiguousarray(uniforms, dtype=np.float64).reshape(trees, -1)
        stride = uniforms.shape[1]
    if request_ids is not None:
        request_ids = np.ascontiguousarray(request_ids, dtype=np.int64)
    out = np.full((trees, max_depth + 2), -1, dtype=np.int64)
    st = lib().sgo_tree_verify_terminal_mass(_p(probs), probs.shape[1], _p(row_offsets), _p(parents), _p(tokens),
                                             trees, max_depth, _p(uniforms), stride, seed, _p(request_ids), _p(out))
    return out, st


def follow(posterior, row_offsets, parents, tokens, max_depth: int) -> np.ndarray:
    posterior = np.ascontiguousarray(posterior, dtype=np.int64)
    row_offsets = np.ascontiguousarray(row_offsets, dtype=np.int64)
    parents = np.ascontiguousarray(parents, dtype=np.int64)
    tokens = np.ascontiguousarray(tokens, dtype=np.int64)
    trees = len(row_offsets) - 1
    out = np.full((trees, max_depth + 2), -1, dtype=np.int64)
    lib().sgo_tree_follow(_p(posterior), _p(row_offsets), _p(parents), _p(tokens), trees, max_depth,
                          _p(out))
    return out


def kv_commit(dst: np.ndarray, src: np.ndarray, src_rows, dst_rows) -> int:
    """In-place commit on [planes, rows, ...] arrays (dst may be src)."""
    assert dst.flags.c_contiguous and src.flags.c_contiguous
    src_rows = np.ascontiguousarray(src_rows, dtype=np.int64)
    dst_rows = np.ascontiguousarray(dst_rows, dtype=np.int64)
    planes = dst.shape[0]
    row_bytes = dst[0, 0].nbytes
    return lib().sgo_kv_commit(_p(dst), dst.shape[1], _p(src), src.shape[1], planes, row_bytes,
                               _p(src_rows), _p(dst_rows), len(src_rows))


def node_uniforms(seed: int, request: int, node: int) -> tuple[float, float]:
    a, b = c_double(), c_double()
    lib().sgo_node_uniforms(seed, request, node, ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


def mass_of(p: float) -> tuple[int, int]:
    lo, hi = c_uint64(), c_uint64()
    bad = lib().sgo_mass_of(p, ctypes.byref(lo), ctypes.byref(hi))
    return (hi.value << 64) | lo.value, bad


def mass_scale(u: float, total: int) -> int:
    lo, hi = c_uint64(), c_uint64()
    lib().sgo_mass_scale(u, total & ((1 << 64) - 1), total >> 64, ctypes.byref(lo), ctypes.byref(hi))
    return (hi.value << 64) | lo.value
