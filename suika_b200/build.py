"""Build recipe for libsuika_reshard.so (the C ABI declared in include/suika_reshard.h).

The library is compiled in-tree with nvcc for sm_100a only; the resulting .so sits next to this
file so that it travels with the source tree. `python -m suika_b200.build` rebuilds it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_NAME = "libsuika_reshard.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
SOURCES = [os.path.join(CSRC, "plan.cpp"), os.path.join(CSRC, "act.cpp"), os.path.join(CSRC, "exec.cu")]
DEPS = SOURCES + [os.path.join(CSRC, "internal.h"), os.path.join(REPO_DIR, "include", "suika_reshard.h")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-Wall",
    "-shared",
]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libsuika_reshard.so")


def is_stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if it is missing or older than its sources; return its path."""
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, *SOURCES, "-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"building {LIB_NAME} failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
