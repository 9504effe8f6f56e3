"""Build recipe for the test-side checkers (TEST INFRASTRUCTURE ONLY).

* ``oracle/_build/libsplitzip_oracle.so``: the C restatement in
  ``splitzip_oracle.c`` (gcc, OpenMP).
* ``oracle/_ref/libref_splitzip_cuda.so``: the reference's own CUDA codec
  compiled unchanged from ``native/unchain_kv/kvq_splitzip_cuda.cu`` where it
  lies in the reference checkout (nvcc, sm_100a).  The GPU tests use it to
  cross-check the new kernels against the reference kernels (modulo the
  canonical-form differences documented in splitzip_oracle.c).  It is built
  only when the reference checkout is present; the GPU box reuses the file
  that travelled with the repository snapshot.

Nothing here is imported by the product package.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libsplitzip_oracle.so"
REF_SO = HERE / "_ref" / "libref_splitzip_cuda.so"
# The reference checkout: UNCHAIN_KV_REFERENCE_ROOT, else a checkout named
# `reference` beside this repository.
REFERENCE_ROOT = Path(os.environ.get("UNCHAIN_KV_REFERENCE_ROOT") or HERE.parents[1] / "reference")
REFERENCE_CU = REFERENCE_ROOT / "native" / "unchain_kv" / "kvq_splitzip_cuda.cu"


def _stale(target: Path, *sources: Path) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(src.stat().st_mtime > mtime for src in sources if src.exists())


def build_oracle(force: bool = False) -> Path:
    src = HERE / "splitzip_oracle.c"
    if force or _stale(ORACLE_SO, src):
        ORACLE_SO.parent.mkdir(parents=True, exist_ok=True)
        tmp = ORACLE_SO.with_suffix(".so.tmp")
        subprocess.run(
            ["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-shared", "-fPIC",
             "-std=c11", "-Wall", "-Wextra", "-Wno-unused-parameter",
             str(src), "-o", str(tmp)],
            check=True,
        )
        tmp.replace(ORACLE_SO)
    return ORACLE_SO


def build_reference(force: bool = False) -> Path | None:
    """Compile the reference CUDA codec from its own source, if present."""
    if not REFERENCE_CU.exists():
        return REF_SO if REF_SO.exists() else None
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if force or _stale(REF_SO, REFERENCE_CU):
        REF_SO.parent.mkdir(parents=True, exist_ok=True)
        tmp = REF_SO.with_suffix(".so.tmp")
        subprocess.run(
            [nvcc, "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
             "-gencode", "arch=compute_100a,code=sm_100a",
             str(REFERENCE_CU), "-o", str(tmp)],
            check=True,
        )
        tmp.replace(REF_SO)
    return REF_SO


def build(force: bool = False) -> None:
    build_oracle(force)
    build_reference(force)


if __name__ == "__main__":
    build(force=True)
    print(ORACLE_SO, REF_SO if REF_SO.exists() else "(reference not built)")
