"""The C-ABI library loads without a GPU and exports every symbol that
include/q3t.h declares (no compute calls)."""
import ctypes
import os
import re

import q3t

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "q3t.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(q3t_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(q3t.LIB_PATH)
    syms = header_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_python_mirror_binds_every_declared_symbol():
    assert sorted(q3t.EXPORTS) == header_symbols()


def test_version_and_error_without_gpu():
    L = q3t.lib()
    assert b"sm_100a" in L.q3t_version()
    assert isinstance(L.q3t_last_error(), bytes)
    assert L.q3t_kernel_launches() >= 0
