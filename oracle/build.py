"""Build recipe for the test-side checkers (TEST INFRASTRUCTURE ONLY).

* ``oracle/_build/libsplitzip_oracle.so``: the C restatement in
  ``splitzip_oracle.c`` (gcc, OpenMP).
* ``baseline/_ref``: the reference's own Python package installed from the
  checkout, with its wrapper tests (``reference_tests/``): the GPU tests run
  them against this repository's library.
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


REF_PACKAGE = HERE.parent / "baseline" / "_ref"
REF_TESTS = REF_PACKAGE / "reference_tests"
REFERENCE_WRAPPER = REFERENCE_ROOT / "src" / "unchain_kv" / "splitzip_cuda.py"
REFERENCE_WRAPPER_TESTS = REFERENCE_ROOT / "tests" / "test_splitzip_cuda.py"


def build_reference_package(force: bool = False) -> Path | None:
    """Install the reference's own Python package (pure Python, no
    dependencies) into baseline/_ref with an offline pip, from a temporary
    copy of the checkout (its build writes into the source tree), and put the
    reference's wrapper tests beside it in baseline/_ref/reference_tests.
    The GPU tests run those tests, and the reference's ctypes wrapper, against
    this repository's library (UNCHAIN_KV_SPLITZIP_LIB).  Only when the
    checkout is present; the GPU box reuses the copy that travelled."""
    installed = REF_PACKAGE / "unchain_kv" / "splitzip_cuda.py"
    if not REFERENCE_WRAPPER.exists():
        return REF_PACKAGE if installed.exists() else None
    if force or _stale(installed, REFERENCE_WRAPPER) or not (REF_TESTS / REFERENCE_WRAPPER_TESTS.name).exists():
        import sys
        import tempfile

        with tempfile.TemporaryDirectory() as tmp:
            src = Path(tmp) / "reference"
            shutil.copytree(REFERENCE_ROOT, src, ignore=shutil.ignore_patterns(".git", "build", "*.egg-info"))
            subprocess.run(
                [sys.executable, "-m", "pip", "install", "--quiet", "--no-index", "--no-deps",
                 "--no-build-isolation", "--upgrade", "--target", str(REF_PACKAGE), str(src)],
                check=True,
            )
        REF_TESTS.mkdir(parents=True, exist_ok=True)
        shutil.copy2(REFERENCE_WRAPPER_TESTS, REF_TESTS / REFERENCE_WRAPPER_TESTS.name)
    return REF_PACKAGE


def build(force: bool = False) -> None:
    build_oracle(force)
    build_reference(force)
    build_reference_package(force)


if __name__ == "__main__":
    build(force=True)
    print(ORACLE_SO, REF_SO if REF_SO.exists() else "(reference not built)")
