"""The C-ABI library loads on a CPU-only host and exports every function include/*.h declares."""
import ctypes
import glob
import os
import re

from suika_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(rs_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_the_path():
    names = declared_functions()
    for n in ("rs_plan_build", "rs_program_build", "rs_program_resolve", "rs_copy_launch", "rs_peer_open"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding knows the signature of each of them
    assert declared_functions() <= set(_lib.SIGNATURES)


def test_version_and_error_string():
    lib = _lib.load()
    a, b = ctypes.c_int32(), ctypes.c_int32()
    assert lib.rs_version(ctypes.byref(a), ctypes.byref(b)) == 0 and (a.value, b.value) >= (1, 1)
    assert lib.rs_plan_num_ops(None, None) == _lib.RS_ERR_ARG
    assert b"NULL" in lib.rs_last_error()


def test_copy_workspace_size_without_gpu():
    lib = _lib.load()
    n = ctypes.c_uint64()
    assert lib.rs_copy_workspace_bytes(1000, ctypes.byref(n)) == 0
    assert n.value >= 1000 * 72 and n.value % 256 == 0
