"""The C-ABI library loads and exports every entry point include/*.h declares
(no compute calls: this runs without a GPU)."""

import ctypes
import re
from pathlib import Path

import pytest

from unchainkv_b200 import splitzip_cuda

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        text = header.read_text()
        names += re.findall(r"KVQ_API\s+[\w\s\*]+?\b(kvq_\w+)\s*\(", text)
    return names


def test_header_declares_reference_entry_points():
    names = set(declared_symbols())
    reference = {
        "kvq_splitzip_last_error", "kvq_splitzip_bf16_encode_mode", "kvq_splitzip_bf16_encode",
        "kvq_splitzip_bf16_decode_fixed6_blocks", "kvq_splitzip_bf16_decode_fixed6",
        "kvq_splitzip_bf16_encode_top16", "kvq_splitzip_bf16_decode_top16_blocks",
        "kvq_splitzip_bf16_decode_top16",
    }
    assert reference <= names


def test_library_exports_every_declared_symbol():
    path = splitzip_cuda.library_path()
    if not path.exists():
        pytest.skip("library not built (python -m unchainkv_b200._build)")
    lib = ctypes.CDLL(str(path))
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_operator_module_binds_every_declared_symbol():
    assert splitzip_cuda.available(), splitzip_cuda.load_error()
    lib = splitzip_cuda._load()
    for name in declared_symbols():
        assert getattr(lib, name) is not None


def test_last_error_is_empty_before_any_failure():
    lib = splitzip_cuda._load()
    assert lib.kvq_splitzip_last_error() in (b"",)


def test_declines_without_touching_the_device():
    lib = splitzip_cuda._load()
    # null pointers / zero counts / bad bits are declined before any CUDA call
    assert lib.kvq_splitzip_bf16_encode_top16(0, 0, 0, 0, 0, 0) == 0
    assert lib.kvq_splitzip_bf16_encode_mode(1, 1, 0, 10, 0, 6) == 0
    assert lib.kvq_splitzip_bf16_encode_mode(1, 1, 100, 10, 0, 4) == 0
    assert lib.kvq_splitzip_bf16_decode_top16_blocks(1, 10, 1, 7, 2, 2, 8, 2, 0, 0, 1, 0) == 0
    assert lib.kvq_splitzip_bf16_decode_fixed6(1, 10, 1, 8, 2, 2, 8, 2, 0, 0) == 0
    # capacity too small for a 4096-word top16 stream
    assert lib.kvq_splitzip_bf16_encode_top16(16, 16, 4096, 100, 16, 0) == 0
    # count beyond the 32-bit position field
    assert lib.kvq_splitzip_bf16_encode_top16(16, 16, 1 << 32, 1 << 40, 16, 0) == 0


def test_attention_request_layout_matches_the_header():
    """ABI revision 3: kvq_splitzip_attn_request gained tables_ptr; the
    Python mirror's struct must have the header's fields in its order."""
    lib = splitzip_cuda._load()
    assert lib.kvq_splitzip_abi_version() == 3
    text = (ROOT / "include" / "unchain_kv_splitzip.h").read_text()
    body = re.search(r"typedef struct kvq_splitzip_attn_request \{(.*?)\}", text, re.S).group(1)
    fields = re.findall(r"unsigned long long (\w+);", body)
    assert [name for name, _ in splitzip_cuda.KvqAttnRequest._fields_] == fields
    assert ctypes.sizeof(splitzip_cuda.KvqAttnRequest) == 8 * len(fields) == 56
