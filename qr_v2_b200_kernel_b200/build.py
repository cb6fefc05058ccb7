"""Build the in-tree CUDA library ``libqrb200.so`` for sm_100a with nvcc.

The library exposes only the C ABI declared in ``include/qrb200.h`` (no torch types), so it
is compiled directly with nvcc rather than through a torch extension. Run as
``python -m qr_v2_b200_kernel_b200.build`` or call :func:`build`.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_NAME = "libqrb200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
SOURCES = ["qrb200.cu", "noalloc.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the qrb200 CUDA library cannot be built")


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h"))]
    files.append(os.path.join(REPO_DIR, "include", "qrb200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile ``libqrb200.so`` next to this file if any source is newer; return its path."""
    if not force and up_to_date():
        return LIB_PATH
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-Xptxas", "-v" if verbose else "-O3",
           "-I", os.path.join(REPO_DIR, "include"), "-o", LIB_PATH + ".tmp"]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr}\n{res.stdout}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
