"""Build the sm_100a C-ABI library in-tree.

``python -m unchainkv_b200._build`` (or ``__graft_entry__.build()``) compiles
``csrc/splitzip.cu`` with nvcc for sm_100a into
``unchainkv_b200/lib/libunchain_kv_splitzip_cuda.so``.  The file name is the
reference's (native/unchain_kv/CMakeLists.txt:21), so the reference's own
ctypes wrapper can load it through ``UNCHAIN_KV_SPLITZIP_LIB``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
LIB_DIR = PACKAGE / "lib"
LIB_NAME = "libunchain_kv_splitzip_cuda.so"
LIB_PATH = LIB_DIR / LIB_NAME
INCLUDE = PACKAGE.parent / "include"
SOURCES = [CSRC / "splitzip.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-I", str(INCLUDE),
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return str(Path(cuda) / "bin" / "nvcc")


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(src.stat().st_mtime > built for src in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, *(str(s) for s in SOURCES), "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    tmp.replace(LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
