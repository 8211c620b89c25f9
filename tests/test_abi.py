"""The C-ABI library loads without a GPU and exports every declared symbol."""
import ctypes
import re
from pathlib import Path

import pytest

from specgrove_b200 import _lib

HEADER_DIR = Path(__file__).resolve().parents[1] / "include"


def declared_symbols():
    names = set()
    for header in HEADER_DIR.glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"SG_API\s+[\w\s\*]+?\b(sg_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("sg_tree_accept_probs", "sg_tree_follow", "sg_kv_commit", "sg_status_string"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    assert set(declared_symbols()) <= set(_lib.exported_symbols())


def test_status_strings_without_gpu():
    lib = _lib.load()
    assert lib.sg_status_string(0) == b"ok"
    assert b"capacity" in lib.sg_status_string(5)
    assert lib.sg_version() >= 1


def test_argument_errors_are_reported_without_gpu():
    lib = _lib.load()
    # null pointers are rejected before any CUDA call
    st = lib.sg_tree_accept_probs(None, 10, None, None, None, 1, 4, 2, 0, None, 0, 0, None, None,
                                  None, None)
    assert st == _lib.SG_ERR_INVALID_ARGUMENT
    assert b"null" in lib.sg_last_error()
    st = lib.sg_kv_commit(None, 1, None, 1, 1, 16, None, None, None, 1, 1, None, None)
    assert st == _lib.SG_ERR_INVALID_ARGUMENT


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIBRARY_PATH", tmp_path / "absent.so")
    with pytest.raises(ImportError, match="no CPU fallback"):
        _lib.load()
