"""The C ABI library loads without a GPU and exports every entry point that
include/qwen_b200.h declares (no compute calls here)."""
import ctypes
import os
import re

from qweninferenceengine_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "qwen_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qwen_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "qwen_gemv_q4_0" in names and "qwen_engine_generate" in names
    assert len(names) >= 30


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    names = set(declared_functions())
    bound = set(_lib.SIGNATURES)
    # every bound name exists in the header; the binding may skip none of the engine calls
    assert bound <= names, bound - names
    assert {n for n in names if n.startswith("qwen_engine_")} <= bound


def test_error_reporting_without_gpu():
    L = _lib.lib()
    rc = L.qwen_gemv_q4_0(None, None, None, None, 32, None, 16, None)
    assert rc == _lib.QWEN_ERR_INVALID_ARGUMENT
    assert b"null" in L.qwen_last_error()
    rc = L.qwen_engine_create(None, None)
    assert rc == _lib.QWEN_ERR_INVALID_ARGUMENT
