"""Operator API of the splitzip bf16 KV codec, backed by the sm_100a library.

Mirrors ``unchain_kv.splitzip_cuda`` of the reference
(src/unchain_kv/splitzip_cuda.py:159-393): same function names, arguments,
return values (int bytes, or None when a call does not apply or the library
declines) and errors (ValueError for bad ``bits``, RuntimeError with the
library's message when a launch fails).  Calls run on
``torch.cuda.current_stream(device)`` and never synchronise.

Differences, all additive:

* the library is the in-tree ``lib/libunchain_kv_splitzip_cuda.so`` (or
  ``UNCHAIN_KV_SPLITZIP_LIB``); when it cannot be loaded, a call with CUDA
  tensors raises instead of returning None -- there is no other backend;
* ``register_top16_codebooks`` installs per-layer palettes (the reference's
  32-layer table is the default);
* fused gather entry points (``encode_top16_blocks``, ``encode_bf16_blocks``)
  encode straight from the paged cache, replacing the
  ``torch.index_select`` pack of vllm_connector.py:2854-2866;
* ``top16_tables`` / ``encode_top16_tables`` take an explicit 544-byte table.
"""

from __future__ import annotations

import ctypes
import math
import os
import threading
from pathlib import Path

_LIB = None
_LOAD_ERROR: str | None = None
_LOAD_LOCK = threading.Lock()
_TOP16_TABLE_CACHE: dict = {}

# Default top-16 exponent codebooks: 32 layers x (16 K + 16 V) exponents,
# code = rank.  This is the reference's interface table
# (src/unchain_kv/splitzip_cuda.py:11-31, Llama-3-8B traces); receivers and
# senders must agree on it byte for byte, so it is carried unchanged.
_DEFAULT_TOP16_CODEBOOKS = bytes.fromhex(
    "7f7e7d807c81857b827a8483867978777c7d7b7a79787e7776757f74737280717f807e817d827c7b837a8479788577767b7c7a797d787776"
    "7e7574737f7271707f807e7d817c7b827a798378777675747c7d7b7a797e7877767f7574807372717f807e7d817c7b7a8283798478857776"
    "7c7d7b7e7a79787f77767574737280717f7e807d7c7b817a79827877767574737d7c7b7e7a79787f77768075817473727f7e807d7c7b7a81"
    "82797877767583747d7e7c7b7f7a797880777675747372717e7f7d807c7b817a82797877767574737d7c7e7b7a7f79787780767574738172"
    "7f7e807d7c7b817a82797877837675747d7e7c7b7f7a797877807675747372717f7e807d7c817b7a79827877767574737d7e7c7b7f7a7980"
    "78777681757473727f7e807d7c7b817a82797877767574737d7e7c7b7f7a797877807675747372717f7e807d7c7b817a8279787776758374"
    "7d7e7c7b7f7a797877807675747372717f7e807d7c7b817a79827877768375747d7e7c7b7f7a797880777675747381727f7e807d7c7b817a"
    "82797877767574737e7d7c7f7b7a797877807675747372717f7e807d7c817b7a82797883778476757d7e7c7b7f7a79788077767574737271"
    "7f7e807d7c7b817a79827877767574737d7e7c7f7b7a798078777675817473727f7e807d7c7b817a79827883777675747e7d7f7c7b7a8079"
    "78777675747372717f7e807d7c817b7a82797877767574737e7d7c7f7b7a798078777675748173727f7e807d7c7b817a7982787776757473"
    "7e7d7c7f7b7a798078777675747372717f7e7d807c7b817a79827877837675747e7d7f7c7b7a807978777675747381727f7e807d7c817b7a"
    "82797877847675837e7d7f7c7b7a807978777675748173727f7e807d7c7b817a79827877767574737e7d7f7c7b7a80797877767574737281"
    "7f7e807d7c7b817a82797877768375747e7d7f7c7b807a7978778176757473727f7e807d7c817b7a82797877767574737e7f7d7c807b7a79"
    "78817776757473727f7e807d7c7b817a82797877767574737f7e7d807c7b817a79787776757482737f7e807d7c7b817a8279787783767574"
    "7f7e7d807c7b817a79787776758274737f7e807d7c7b817a79827877768375747f7e807d817c7b7a79827877767574737f7e807d7c7b817a"
    "7982787776837574807f817e7d827c7b7a797877837675747f7e7d807c7b817a828679838785847880817f7e7d827c7b7a79788377767574"
    "7f807e7d7c817b7a82798378770076757d7c7e7b7a79787f77767580740073727f807e7d7c817b7a79828378770076757d7c7e7b7a7f7978"
    "77807675740073727f807e7d7c817b827a797877830076757d7e7c7b7f7a797877807675007473727f807e7d817c7b7a82797877007675837d7e7c7b7f7a79788077767500747381"
)
_TOP16_CODEBOOKS = _DEFAULT_TOP16_CODEBOOKS

_U64 = ctypes.c_ulonglong
_SIGNATURES = {
    "kvq_splitzip_bf16_encode": [_U64] * 5,
    "kvq_splitzip_bf16_encode_mode": [_U64] * 5 + [ctypes.c_int],
    "kvq_splitzip_bf16_decode_fixed6": [_U64] * 10,
    "kvq_splitzip_bf16_decode_fixed6_blocks": [_U64] * 11,
    "kvq_splitzip_bf16_encode_top16": [_U64] * 6,
    "kvq_splitzip_bf16_decode_top16": [_U64] * 11,
    "kvq_splitzip_bf16_decode_top16_blocks": [_U64] * 12,
    "kvq_splitzip_bf16_encode_top16_blocks": [_U64] * 11,
    "kvq_splitzip_bf16_encode_mode_blocks": [_U64] * 10 + [ctypes.c_int],
    "kvq_splitzip_bf16_encode_top16_noalloc": [_U64] * 6,
    "kvq_splitzip_top16_tables_from_histograms": [_U64] * 5,
    "kvq_splitzip_device_errors": [],
    "kvq_splitzip_device_errors_reset": [],
    "kvq_splitzip_test_encode_mode_skip_arrival": [_U64] * 5 + [ctypes.c_int, _U64],
    "kvq_splitzip_abi_version": [],
}
_BATCH_SIGNATURES = {
    "kvq_splitzip_bf16_encode_top16_batch": None,
    "kvq_splitzip_bf16_encode_mode_batch": ctypes.c_int,
    "kvq_splitzip_bf16_encode_auto_batch": None,
    "kvq_splitzip_bf16_decode_top16_batch": None,
    "kvq_splitzip_bf16_decode_fixed6_batch": None,
    "kvq_splitzip_bf16_decode_auto_batch": None,
    "kvq_splitzip_bf16_exponent_histogram_batch": None,
    "kvq_splitzip_bf16_decode_any_batch": None,
    "kvq_splitzip_bf16_encode_torchop_batch": None,
    "kvq_splitzip_writeback_batch": None,
}


class KvqJob(ctypes.Structure):
    """``kvq_splitzip_job`` of include/unchain_kv_splitzip.h: one call of a batch."""

    _fields_ = [
        (name, ctypes.c_ulonglong)
        for name in (
            "cache_ptr", "plane_stride", "block_stride", "block_words", "block_ids_ptr",
            "block_start", "block_count", "stream_ptr", "stream_bytes", "tables_ptr",
        )
    ]


class KvqAttnRequest(ctypes.Structure):
    """``kvq_splitzip_attn_request`` of include/unchain_kv_splitzip.h: one
    request of a decode-attention batch."""

    _fields_ = [
        (name, ctypes.c_ulonglong)
        for name in ("stream_ptr", "stream_bytes", "blocks", "ctx_tokens", "q_ptr", "out_ptr", "tables_ptr")
    ]


def library_path() -> Path:
    """The in-tree build of the sm_100a library."""
    return Path(__file__).resolve().parent / "lib" / "libunchain_kv_splitzip_cuda.so"


def _candidate_paths() -> list[str]:
    env = os.environ.get("UNCHAIN_KV_SPLITZIP_LIB")
    if env:
        return [env]
    return [str(library_path())]


def _load():
    global _LIB, _LOAD_ERROR
    if _LIB is not None:
        return _LIB
    with _LOAD_LOCK:
        if _LIB is not None:
            return _LIB
        errors = []
        for path in _candidate_paths():
            try:
                lib = ctypes.CDLL(path)
            except OSError as exc:
                errors.append(str(exc))
                continue
            for name, argtypes in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = ctypes.c_longlong
            for name, extra in _BATCH_SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = [ctypes.POINTER(KvqJob), _U64, _U64] + ([extra] if extra else [])
                fn.restype = ctypes.c_longlong
            lib.kvq_splitzip_attention_workspace_bytes.argtypes = [ctypes.POINTER(KvqAttnRequest), _U64, _U64]
            lib.kvq_splitzip_attention_workspace_bytes.restype = ctypes.c_longlong
            lib.kvq_splitzip_attention_decode.argtypes = [ctypes.POINTER(KvqAttnRequest)] + [_U64] * 5
            lib.kvq_splitzip_attention_decode.restype = ctypes.c_longlong
            _bytes64 = ctypes.POINTER(ctypes.c_ubyte)
            for name, argtypes, restype in (
                ("kvq_splitzip_ipc_alloc", [_U64], _U64),
                ("kvq_splitzip_ipc_free", [_U64], ctypes.c_longlong),
                ("kvq_splitzip_ipc_get_handle", [_U64, _bytes64], ctypes.c_longlong),
                ("kvq_splitzip_ipc_open", [_bytes64], _U64),
                ("kvq_splitzip_ipc_close", [_U64], ctypes.c_longlong),
                ("kvq_splitzip_peer_access", [ctypes.c_longlong], ctypes.c_longlong),
            ):
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = restype
            lib.kvq_splitzip_last_error.argtypes = []
            lib.kvq_splitzip_last_error.restype = ctypes.c_char_p
            lib.kvq_splitzip_profile_enable.argtypes = [ctypes.c_int]
            lib.kvq_splitzip_profile_enable.restype = ctypes.c_longlong
            lib.kvq_splitzip_profile_collect.argtypes = []
            lib.kvq_splitzip_profile_collect.restype = ctypes.c_longlong
            lib.kvq_splitzip_profile_name.argtypes = [ctypes.c_int]
            lib.kvq_splitzip_profile_name.restype = ctypes.c_char_p
            lib.kvq_splitzip_profile_ms.argtypes = [ctypes.c_int]
            lib.kvq_splitzip_profile_ms.restype = ctypes.c_double
            lib.kvq_splitzip_profile_launches.argtypes = [ctypes.c_int]
            lib.kvq_splitzip_profile_launches.restype = ctypes.c_longlong
            _LIB = lib
            _LOAD_ERROR = None
            return lib
        _LOAD_ERROR = "; ".join(errors[-2:])
        return None


def available() -> bool:
    return _load() is not None


def load_error() -> str | None:
    _load()
    return _LOAD_ERROR


def _require_lib():
    """The library, or a loud failure: a CUDA call has no other backend."""
    lib = _load()
    if lib is None:
        raise RuntimeError(
            "unchainkv_b200: the sm_100a splitzip library is not loadable "
            f"({_LOAD_ERROR}); build it with `python -m unchainkv_b200._build`"
        )
    return lib


def _is_cuda(tensor) -> bool:
    return getattr(getattr(tensor, "device", None), "type", "") == "cuda"


def _raise_last(lib, default: str):
    error = lib.kvq_splitzip_last_error()
    raise RuntimeError(error.decode() if error else default)


# --------------------------------------------------------------- tables


def build_top16_tables(codebooks: bytes) -> bytes:
    """The 544-byte device table of one layer from its 32 codebook bytes:
    [0,256) K exponent->code, [256,512) V, 255 = escape, later duplicates win;
    then the 32 codebook bytes (splitzip_cuda.py:290-295 of the reference)."""
    if len(codebooks) != 32:
        raise ValueError("a layer's top16 codebooks are 32 bytes (16 K + 16 V)")
    values = bytearray([255]) * 512
    for plane in range(2):
        for code, exponent in enumerate(codebooks[plane * 16 : (plane + 1) * 16]):
            values[plane * 256 + exponent] = code
    values.extend(codebooks)
    return bytes(values)


def rank_top16(histogram) -> list[int]:
    """Top-16 exponents of a 256-bin histogram ranked by (-count, exponent),
    observed exponents only; code = rank (trace.py:30-33 and
    scripts/extract_llama_top16_codebooks.py:39-40 of the reference)."""
    counts = [int(v) for v in histogram]
    ranked = sorted((e for e in range(len(counts)) if counts[e] > 0), key=lambda e: (-counts[e], e))
    return ranked[:16]


def register_top16_codebooks(codebooks: bytes) -> int:
    """Install per-layer top16 codebooks (32 bytes per layer, K then V).

    Replaces the module's ``_TOP16_CODEBOOKS`` (so the layer bound of
    ``_top16_tables`` follows it) and drops cached device tables.  Returns
    the number of layers.  ``register_top16_codebooks(None)`` restores the
    reference's default table."""
    global _TOP16_CODEBOOKS
    if codebooks is None:
        codebooks = _DEFAULT_TOP16_CODEBOOKS
    codebooks = bytes(codebooks)
    if not codebooks or len(codebooks) % 32:
        raise ValueError("codebooks must be a non-empty multiple of 32 bytes")
    _TOP16_CODEBOOKS = codebooks
    _TOP16_TABLE_CACHE.clear()
    return len(codebooks) // 32


def _top16_tables(layer_index: int, device, torch):
    if not 0 <= layer_index < len(_TOP16_CODEBOOKS) // 32:
        return None
    key = (str(device), layer_index, id(_TOP16_CODEBOOKS))
    cached = _TOP16_TABLE_CACHE.get(key)
    if cached is not None:
        return cached
    values = build_top16_tables(_TOP16_CODEBOOKS[layer_index * 32 : (layer_index + 1) * 32])
    cached = torch.tensor(list(values), dtype=torch.uint8, device=device)
    _TOP16_TABLE_CACHE[key] = cached
    return cached


def top16_tables(layer_index: int, device):
    """Public form of ``_top16_tables``: the layer's 544-byte uint8 device table."""
    import torch

    return _top16_tables(layer_index, device, torch)


# --------------------------------------------------------------- encode


def encode_bf16(source, out, bits: int = 6) -> int | None:
    """fixed6 (bits 6) / fixed5 (bits 5) encode of a contiguous bf16 tensor
    into the uint8 tensor ``out``; returns the stream length or None."""
    if not _is_cuda(source):
        return None
    lib = _require_lib()
    if bits not in {5, 6}:
        raise ValueError("splitzip bf16 bits must be 5 or 6")
    import torch

    stream = torch.cuda.current_stream(source.device).cuda_stream
    encoded = lib.kvq_splitzip_bf16_encode_mode(
        int(source.data_ptr()),
        int(out.data_ptr()),
        int(source.numel()),
        int(out.numel()),
        int(stream),
        int(bits),
    )
    if encoded < 0:
        _raise_last(lib, "splitzip cuda encode failed")
    return int(encoded)


def encode_top16(source, out, layer_index: int) -> int | None:
    """top16 encode of a contiguous bf16 tensor with layer ``layer_index``'s
    codebooks; returns the stream length, or None if declined."""
    if not _is_cuda(source):
        return None
    if source.device != getattr(out, "device", None):
        return None
    lib = _require_lib()
    import torch

    if source.dtype != torch.bfloat16 or out.dtype != torch.uint8:
        return None
    if not source.is_contiguous() or not out.is_contiguous():
        return None
    tables = _top16_tables(layer_index, source.device, torch)
    if tables is None:
        return None
    return encode_top16_tables(source, out, tables, _lib=lib)


def encode_top16_tables(source, out, tables, _lib=None) -> int | None:
    """top16 encode with an explicit 544-byte uint8 device table."""
    lib = _lib or _require_lib()
    import torch

    stream = torch.cuda.current_stream(source.device).cuda_stream
    encoded = lib.kvq_splitzip_bf16_encode_top16(
        int(source.data_ptr()),
        int(out.data_ptr()),
        int(source.numel()),
        int(out.numel()),
        int(tables.data_ptr()),
        int(stream),
    )
    if encoded < 0:
        _raise_last(lib, "splitzip top16 encode failed")
    return int(encoded) or None


def _block_layout(kv_layer, block_ids, torch):
    """(plane_stride, block_stride, block_words, ids tensor|None, start, count)
    for a paged layer [2, num_blocks, ...] whose blocks are contiguous."""
    if kv_layer.dim() < 3 or kv_layer.shape[0] != 2:
        return None
    block_words = 1
    for size in kv_layer.shape[2:]:
        block_words *= int(size)
    expected = 1
    for dim in range(kv_layer.dim() - 1, 1, -1):
        if kv_layer.shape[dim] != 1 and kv_layer.stride(dim) != expected:
            return None
        expected *= int(kv_layer.shape[dim])
    if isinstance(block_ids, torch.Tensor):
        ids = block_ids.to(device=kv_layer.device, dtype=torch.int64).contiguous()
        return (int(kv_layer.stride(0)), int(kv_layer.stride(1)), block_words, ids, 0, int(ids.numel()))
    block_ids = [int(b) for b in block_ids]
    if not block_ids:
        return None
    start = block_ids[0]
    if block_ids == list(range(start, start + len(block_ids))):
        return (int(kv_layer.stride(0)), int(kv_layer.stride(1)), block_words, None, start, len(block_ids))
    ids = torch.tensor(block_ids, dtype=torch.int64, device=kv_layer.device)
    return (int(kv_layer.stride(0)), int(kv_layer.stride(1)), block_words, ids, 0, len(block_ids))


def encode_top16_blocks(kv_layer, block_ids, out, layer_index: int = 0, tables=None) -> int | None:
    """Fused gather + top16 encode straight from the paged cache.

    Produces the bytes of ``encode_top16(index_select(kv_layer, 1, ids), out,
    layer)`` without the packed copy.  ``block_ids`` is a list of ints or an
    int64 tensor."""
    if not _is_cuda(kv_layer):
        return None
    lib = _require_lib()
    import torch

    if kv_layer.dtype != torch.bfloat16 or out.dtype != torch.uint8 or not out.is_contiguous():
        return None
    layout = _block_layout(kv_layer, block_ids, torch)
    if layout is None:
        return None
    if tables is None:
        tables = _top16_tables(layer_index, kv_layer.device, torch)
        if tables is None:
            return None
    plane_stride, block_stride, block_words, ids, start, count = layout
    current = torch.cuda.current_stream(kv_layer.device)
    encoded = lib.kvq_splitzip_bf16_encode_top16_blocks(
        int(kv_layer.data_ptr()), plane_stride, block_stride, block_words,
        int(ids.data_ptr()) if ids is not None else 0, start, count,
        int(out.data_ptr()), int(out.numel()), int(tables.data_ptr()), int(current.cuda_stream),
    )
    if ids is not None and not isinstance(block_ids, torch.Tensor):
        ids.record_stream(current)
    if encoded < 0:
        _raise_last(lib, "splitzip top16 encode failed")
    return int(encoded) or None


def encode_bf16_blocks(kv_layer, block_ids, out, bits: int = 6) -> int | None:
    """Fused gather + fixed6/fixed5 encode straight from the paged cache."""
    if not _is_cuda(kv_layer):
        return None
    lib = _require_lib()
    if bits not in {5, 6}:
        raise ValueError("splitzip bf16 bits must be 5 or 6")
    import torch

    if kv_layer.dtype != torch.bfloat16 or out.dtype != torch.uint8 or not out.is_contiguous():
        return None
    layout = _block_layout(kv_layer, block_ids, torch)
    if layout is None:
        return None
    plane_stride, block_stride, block_words, ids, start, count = layout
    current = torch.cuda.current_stream(kv_layer.device)
    encoded = lib.kvq_splitzip_bf16_encode_mode_blocks(
        int(kv_layer.data_ptr()), plane_stride, block_stride, block_words,
        int(ids.data_ptr()) if ids is not None else 0, start, count,
        int(out.data_ptr()), int(out.numel()), int(current.cuda_stream), int(bits),
    )
    if ids is not None and not isinstance(block_ids, torch.Tensor):
        ids.record_stream(current)
    if encoded < 0:
        _raise_last(lib, "splitzip cuda encode failed")
    return int(encoded) or None


# --------------------------------------------------------------- decode


def _decode_layout(source, out, block_ids, raw_bytes, torch):
    """Validation and layout of the reference decoder wrappers
    (splitzip_cuda.py:200-230): same rules, same None results."""
    if not block_ids or raw_bytes <= 0 or raw_bytes % 2:
        return None
    if not _is_cuda(source):
        return None
    if source.device != getattr(out, "device", None):
        return None
    if source.dtype != torch.uint8 or out.dtype != torch.bfloat16:
        return None
    if not source.is_contiguous() or not out.is_contiguous():
        return None
    if out.dim() < 3 or out.shape[0] != 2:
        return None
    if len(set(block_ids)) != len(block_ids) or any(
        block < 0 or block >= out.shape[1] for block in block_ids
    ):
        return None
    start = block_ids[0]
    contiguous = block_ids == list(range(start, start + len(block_ids)))
    count_words = raw_bytes // 2
    divisor = 2 * len(block_ids)
    if count_words % divisor:
        return None
    block_words = count_words // divisor
    current = torch.cuda.current_stream(out.device)
    block_ids_tensor = None
    if not contiguous:
        block_ids_tensor = torch.tensor(block_ids, dtype=torch.int64, device=out.device)
    return count_words, block_words, start, current, block_ids_tensor


def decode_fixed6(source, out, block_ids: list[int], raw_bytes: int) -> int | None:
    """Decode a mode-3 stream and scatter it into ``out``'s blocks."""
    if not _is_cuda(source):
        return None
    lib = _require_lib()
    import torch

    layout = _decode_layout(source, out, block_ids, raw_bytes, torch)
    if layout is None:
        return None
    count_words, block_words, start, current, block_ids_tensor = layout
    if block_ids_tensor is not None:
        copied = lib.kvq_splitzip_bf16_decode_fixed6_blocks(
            int(source.data_ptr()), int(source.numel()), int(out.data_ptr()), count_words,
            len(block_ids), block_words, int(out.stride(0)), int(out.stride(1)), start,
            int(block_ids_tensor.data_ptr()), int(current.cuda_stream),
        )
        block_ids_tensor.record_stream(current)
    else:
        copied = lib.kvq_splitzip_bf16_decode_fixed6(
            int(source.data_ptr()), int(source.numel()), int(out.data_ptr()), count_words,
            len(block_ids), block_words, int(out.stride(0)), int(out.stride(1)), start,
            int(current.cuda_stream),
        )
    if copied < 0:
        _raise_last(lib, "splitzip cuda decode failed")
    return int(copied) or None


def decode_top16(source, out, block_ids: list[int], raw_bytes: int, layer_index: int) -> int | None:
    """Decode a mode-5 stream with layer ``layer_index``'s codebooks and
    scatter it into ``out``'s blocks."""
    if not _is_cuda(source):
        return None
    lib = _require_lib()
    import torch

    layout = _decode_layout(source, out, block_ids, raw_bytes, torch)
    if layout is None:
        return None
    tables = _top16_tables(layer_index, source.device, torch)
    if tables is None:
        return None
    return _decode_top16_with(lib, source, out, block_ids, layout, tables)


def decode_top16_tables(source, out, block_ids: list[int], raw_bytes: int, tables) -> int | None:
    """decode_top16 with an explicit 544-byte uint8 device table."""
    if not _is_cuda(source):
        return None
    lib = _require_lib()
    import torch

    layout = _decode_layout(source, out, block_ids, raw_bytes, torch)
    if layout is None:
        return None
    return _decode_top16_with(lib, source, out, block_ids, layout, tables)


def _decode_top16_with(lib, source, out, block_ids, layout, tables):
    count_words, block_words, start, current, block_ids_tensor = layout
    if block_ids_tensor is not None:
        copied = lib.kvq_splitzip_bf16_decode_top16_blocks(
            int(source.data_ptr()), int(source.numel()), int(out.data_ptr()), count_words,
            len(block_ids), block_words, int(out.stride(0)), int(out.stride(1)), start,
            int(block_ids_tensor.data_ptr()), int(tables.data_ptr()), int(current.cuda_stream),
        )
        block_ids_tensor.record_stream(current)
    else:
        copied = lib.kvq_splitzip_bf16_decode_top16(
            int(source.data_ptr()), int(source.numel()), int(out.data_ptr()), count_words,
            len(block_ids), block_words, int(out.stride(0)), int(out.stride(1)), start,
            int(tables.data_ptr()), int(current.cuda_stream),
        )
    if copied < 0:
        _raise_last(lib, "splitzip top16 decode failed")
    return int(copied) or None


def device_errors() -> int:
    """Device-side bounded waits that ran out since load or the last
    device_errors_reset() (0 normally)."""
    lib = _require_lib()
    value = lib.kvq_splitzip_device_errors()
    if value < 0:
        _raise_last(lib, "splitzip device error query failed")
    return int(value)


def device_errors_reset() -> None:
    lib = _require_lib()
    if lib.kvq_splitzip_device_errors_reset() < 0:
        _raise_last(lib, "splitzip device error reset failed")


# ------------------------------------------------------ decode attention

ATTN_KV_HEADS = 8
ATTN_HEAD_DIM = 128
ATTN_BLOCK_TOKENS = 16


def attention_stream_buffer(nbytes: int, device):
    """A uint8 CUDA buffer of ``nbytes`` whose first byte sits at an address
    15 mod 16: a fixed6 or raw stream placed there has its planes on 16-byte
    boundaries, so attention_decode reads them with plain 16-byte loads."""
    import torch

    raw = torch.empty(nbytes + 32, dtype=torch.uint8, device=device)
    start = (15 - raw.data_ptr()) % 16
    return raw[start : start + nbytes]


def attention_requests(q, streams, ctx_tokens, out, tables=None):
    """The ``kvq_splitzip_attn_request`` array of a batch (see attention_decode)."""
    reqs = (KvqAttnRequest * len(streams))()
    for i, (stream, ctx) in enumerate(zip(streams, ctx_tokens)):
        r = reqs[i]
        r.stream_ptr = stream.data_ptr()
        r.stream_bytes = stream.numel() * stream.element_size()
        r.ctx_tokens = int(ctx)
        r.blocks = (int(ctx) + ATTN_BLOCK_TOKENS - 1) // ATTN_BLOCK_TOKENS
        r.q_ptr = q[i].data_ptr()
        r.out_ptr = out[i].data_ptr()
        table = tables[i] if tables is not None else None
        r.tables_ptr = table.data_ptr() if table is not None else 0
    return reqs


def attention_decode(q, streams, ctx_tokens, out, workspace=None, stream=None, tables=None) -> int | None:
    """Decode attention straight over splitzip streams (extension: the
    reference decodes each stream into its paged cache and attends over the
    bf16 copy, scripts/bench_codec_attention.py:155-157).

    ``q`` and ``out``: bf16 CUDA tensors [requests, 8 * group, 128] (q head
    ``kv_head * group + i`` uses kv head ``kv_head``).  ``streams``: per
    request a uint8 CUDA tensor holding that request's layer stream (fixed6
    mode 3, raw mode 6, or top16 mode 5) of ceil(ctx/16) paged blocks of
    [16, 8, 128].  ``tables``: per request the layer's 544-byte top16 table
    (a uint8 CUDA tensor) or None; a top16 stream needs its table, and its
    escape entries sorted by position (as this library's encoders write
    them).
    ``ctx_tokens``: valid tokens per request.  ``out[r, h]`` =
    softmax(q[r, h] K^T / sqrt(128)) V, fp32 accumulation.  Returns the number
    of requests, or None when the batch is declined."""
    import torch

    lib = _require_lib()
    heads = q.shape[1]
    if q.dtype != torch.bfloat16 or out.dtype != torch.bfloat16 or heads % ATTN_KV_HEADS:
        return None
    if not (q.is_contiguous() and out.is_contiguous()) or q.shape != out.shape or q.shape[2] != ATTN_HEAD_DIM:
        return None
    if len(streams) != q.shape[0] or len(ctx_tokens) != q.shape[0]:
        return None
    group = heads // ATTN_KV_HEADS
    if tables is not None and len(tables) != q.shape[0]:
        return None
    reqs = attention_requests(q, streams, ctx_tokens, out, tables)
    need = lib.kvq_splitzip_attention_workspace_bytes(reqs, len(streams), group)
    if need <= 0:
        return None
    s = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
        if stream is not None:  # keep it from the allocator until that stream is done
            workspace.record_stream(torch.cuda.ExternalStream(stream, device=q.device))
    res = lib.kvq_splitzip_attention_decode(reqs, len(streams), group, workspace.data_ptr(), workspace.numel(), s)
    if res < 0:
        _raise_last(lib, "splitzip attention failed")
    return int(res) if res else None


# --------------------------------------------------------------- batches


def top16_stream_bytes(n: int) -> int:
    """Length of a top16 (mode 5) stream of n words."""
    return 5 + n + (n + 1) // 2 + 5 * ((n + 199) // 200)


def fixed6_stream_bytes(n: int) -> int:
    """Length of a fixed6 (mode 3) stream of n words."""
    return 65 + n + ((n + 3) // 4) * 3


def stream_bytes(mode: int, n: int) -> int | None:
    """Length of a stream of n words from its mode byte (None: no stream)."""
    if mode == 5:
        return top16_stream_bytes(n)
    if mode == 3:
        return fixed6_stream_bytes(n)
    if mode == 6:
        return 1 + 2 * n
    return None


def stream_length(header: bytes, n: int) -> int | None:
    """Length of a stream of n words from its first bytes (at least 5), for
    every form: modes 5, 3, 6 from the mode byte, the torch-op forms 2, 0,
    1 from their widths, fixed5 (4).  None: not a stream."""
    mode = header[0]
    if mode in (5, 3, 6):
        return stream_bytes(mode, n)
    if mode == 4:
        return 33 + n + (5 * n + 7) // 8
    if mode == 2:
        return 3 + n + (n + 7) // 8 + (n * header[1] + 7) // 8
    if mode == 0:
        return 258 + n + (n * header[1] + 7) // 8
    if mode == 1:
        return 69 + sum((n * w + 7) // 8 for w in header[1:5])
    return None


# Words per tile of the library's kernels (kTileWords): the auto encode's
# statistics scratch holds a 16-byte record of escape counts per tile.
TILE_WORDS = 16384


def torchop_capacity(n: int) -> int:
    """Stream-buffer bytes for encode_torchop_batch: raw mode 6 (the largest
    form) plus the job's 416-byte plan."""
    return (1 + 2 * n + 15) // 16 * 16 + 416 + 16


def top16_capacity(n: int) -> int:
    """Least stream-buffer bytes the top16 encoders accept
    (kvq_splitzip_bf16_encode_top16 and its _blocks / _batch / _noalloc
    forms): the reference's rule, align4(stream) + 8
    (native/unchain_kv/kvq_splitzip_cuda.cu:390-394)."""
    return (top16_stream_bytes(n) + 3) // 4 * 4 + 8


def auto_capacity(n: int, raw: bool = True) -> int:
    """Stream-buffer bytes for encode_auto_batch: room for the largest form
    (raw mode 6 when ``raw``) plus the statistics scratch."""
    tiles = (n + TILE_WORDS - 1) // TILE_WORDS
    scratch = 64 + (8 * ((tiles + 31) // 32) + 15) // 16 * 16 + 16 * tiles
    largest = 1 + 2 * n if raw else max(top16_stream_bytes(n), fixed6_stream_bytes(n))
    return ((largest + 15) // 16) * 16 + scratch + 16


def make_job(kv_layer, block_ids, stream_buffer, stream_bytes_: int | None = None, tables=None,
             block_start: int = 0, block_count: int | None = None) -> KvqJob:
    """Describe one call: ``kv_layer`` [2, num_blocks, ...] (bf16, blocks
    contiguous), ``block_ids`` an int64 device tensor (or None with
    ``block_start``/``block_count`` for a contiguous run), ``stream_buffer``
    a uint8 device tensor (its size is the capacity unless
    ``stream_bytes_`` is given), ``tables`` the layer's 544-byte table."""
    block_words = 1
    for size in kv_layer.shape[2:]:
        block_words *= int(size)
    if block_ids is not None:
        block_count = int(block_ids.numel())
    job = KvqJob()
    job.cache_ptr = int(kv_layer.data_ptr())
    job.plane_stride = int(kv_layer.stride(0))
    job.block_stride = int(kv_layer.stride(1))
    job.block_words = block_words
    job.block_ids_ptr = int(block_ids.data_ptr()) if block_ids is not None else 0
    job.block_start = int(block_start)
    job.block_count = int(block_count)
    job.stream_ptr = int(stream_buffer.data_ptr())
    job.stream_bytes = int(stream_bytes_ if stream_bytes_ is not None else stream_buffer.numel())
    job.tables_ptr = int(tables.data_ptr()) if tables is not None else 0
    return job


def job_array(jobs) -> "ctypes.Array":
    array = (KvqJob * len(jobs))()
    for i, job in enumerate(jobs):
        array[i] = job
    return array


def _run_batch(name: str, jobs, stream=None, extra=None) -> int | None:
    lib = _require_lib()
    import torch

    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    array = jobs if isinstance(jobs, ctypes.Array) else job_array(list(jobs))
    args = [array, len(array), int(stream)] + ([extra] if extra is not None else [])
    result = getattr(lib, name)(*args)
    if result < 0:
        _raise_last(lib, f"{name} failed")
    return int(result) or None


def encode_top16_batch(jobs, stream=None) -> int | None:
    """Fused gather + top16 encode of every job in one launch; returns the
    total encoded bytes, None if any job is declined (nothing launched)."""
    return _run_batch("kvq_splitzip_bf16_encode_top16_batch", jobs, stream)


def encode_bf16_batch(jobs, bits: int = 6, stream=None) -> int | None:
    if bits not in {5, 6}:
        raise ValueError("splitzip bf16 bits must be 5 or 6")
    return _run_batch("kvq_splitzip_bf16_encode_mode_batch", jobs, stream, int(bits))


def encode_auto_batch(jobs, stream=None) -> int | None:
    """Device-chosen codec per job (top16, else fixed6, else raw, else 255);
    byte 0 of each stream tells which (see ``stream_bytes``)."""
    return _run_batch("kvq_splitzip_bf16_encode_auto_batch", jobs, stream)


def decode_top16_batch(jobs, stream=None) -> int | None:
    return _run_batch("kvq_splitzip_bf16_decode_top16_batch", jobs, stream)


def decode_fixed6_batch(jobs, stream=None) -> int | None:
    return _run_batch("kvq_splitzip_bf16_decode_fixed6_batch", jobs, stream)


def decode_auto_batch(jobs, stream=None) -> int | None:
    """Decode each job's stream by its mode byte (5, 3 or 6) on the device."""
    return _run_batch("kvq_splitzip_bf16_decode_auto_batch", jobs, stream)


def writeback_job(kv_layer, stream_buffer, stream_bytes_: int, block_start: int, block_count: int) -> KvqJob:
    """A writeback job: the first ``stream_bytes_`` of ``stream_buffer`` go
    over the layer's blocks [block_start, block_start + block_count)."""
    return make_job(kv_layer, None, stream_buffer, stream_bytes_, None, block_start, block_count)


def writeback_batch(jobs, stream=None) -> int | None:
    """Codec writeback (the reference's ``_try_splitzip_writeback``): copy
    each job's stream over its own blocks, K-plane run first, then the
    V-plane run, in one launch.  Like the reference, declines (None) a job
    whose blocks are not one contiguous run of adjacent blocks or whose
    stream overlaps them.  Returns the bytes written."""
    return _run_batch("kvq_splitzip_writeback_batch", jobs, stream)


def writeback_segments(kv_layer, block_start: int, block_count: int):
    """The byte views a writeback fills, in order (the reference's
    ``_kv_writeback_segments`` for one run): K-plane blocks, V-plane blocks."""
    import torch

    return [kv_layer[plane, block_start:block_start + block_count].reshape(-1).view(torch.uint8)
            for plane in range(2)]


def encode_torchop_batch(jobs, stream=None) -> int | None:
    """The reference's torch-op encoder on the GPU, every job in one batch:
    the first of sign/magnitude (mode 2), high-byte palette (mode 0) and
    nibble planes (mode 1) that is smaller than raw, else raw (mode 6).
    Capacity: ``torchop_capacity(n)``.  Returns the sum of 1 + 2n over the
    jobs; each stream's length follows from its header (``stream_length``)."""
    return _run_batch("kvq_splitzip_bf16_encode_torchop_batch", jobs, stream)


def decode_any_batch(jobs, stream=None) -> int | None:
    """Decode each job's stream whatever its mode: 5, 3 and 6 as
    ``decode_auto_batch``, and the receiver's other forms (the reference's
    torch-op modes 0, 1, 2 and fixed5, mode 4) with the receiver's checks.
    ``stream_bytes`` must be the stream's exact length for modes 0, 1, 2
    and 4; a stream that fails its checks leaves its blocks untouched."""
    return _run_batch("kvq_splitzip_bf16_decode_any_batch", jobs, stream)


# ------------------------------------------------------------ calibration
#
# GPU form of the reference's exponent trace (vllm_connector.py:2871-2904)
# and of its codebook ranking (trace.py:27-58,
# scripts/extract_llama_top16_codebooks.py:39-40): histograms of
# (w >> 7) & 0xFF per plane, gathered from the paged cache on the device,
# then the top16 tables built on the device, so palettes can be calibrated
# online without a host round trip.


def histogram_job(kv_layer, block_ids, hist, block_start: int = 0, block_count: int | None = None) -> KvqJob:
    """A calibration job: the layer's blocks (as ``make_job``) counted into
    ``hist``, a [2, 256] int32 device tensor (K plane, then V)."""
    if hist.dtype.itemsize != 4 or hist.numel() != 512 or not hist.is_contiguous():
        raise ValueError("hist must be a contiguous [2, 256] 32-bit tensor")
    return make_job(kv_layer, block_ids, hist, 2048, None, block_start, block_count)


def exponent_histogram_batch(jobs, stream=None) -> int | None:
    """Add the exponent counts of every job's words to its histogram (one
    launch; counts accumulate across calls).  Returns the number of jobs,
    None if any job is declined (nothing launched)."""
    return _run_batch("kvq_splitzip_bf16_exponent_histogram_batch", jobs, stream)


def top16_tables_from_histograms(hist, tables=None, observed=None, stream=None):
    """Top16 device tables of ``hist`` ([layers, 2, 256] int32 counts):
    returns (tables [layers, 544] uint8, observed [layers, 2] int32), the
    tables in the layout ``_top16_tables`` gives and ``observed`` the number
    of exponents with a nonzero count per plane.  A plane with fewer than
    16 gets the unobserved exponents in ascending order as its last codes."""
    lib = _require_lib()
    import torch

    if hist.dim() != 3 or tuple(hist.shape[1:]) != (2, 256) or hist.dtype.itemsize != 4 or not hist.is_contiguous():
        raise ValueError("hist must be a contiguous [layers, 2, 256] 32-bit tensor")
    layers = int(hist.shape[0])
    if tables is None:
        tables = torch.empty((layers, 544), dtype=torch.uint8, device=hist.device)
    if observed is None:
        observed = torch.empty((layers, 2), dtype=torch.int32, device=hist.device)
    if stream is None:
        stream = torch.cuda.current_stream(hist.device).cuda_stream
    result = lib.kvq_splitzip_top16_tables_from_histograms(
        int(hist.data_ptr()), layers, int(tables.data_ptr()), int(observed.data_ptr()), int(stream))
    if result < 0:
        _raise_last(lib, "kvq_splitzip_top16_tables_from_histograms failed")
    if result == 0:
        return None
    return tables, observed


def codebooks_from_tables(tables, observed) -> bytes:
    """The 32 codebook bytes per layer (K then V) of device tables, for
    ``register_top16_codebooks``.  Like the reference's extractor, raises
    ValueError when a plane has fewer than 16 observed exponents."""
    seen = observed.cpu().tolist()
    for layer, planes in enumerate(seen):
        for plane, count in zip("kv", planes):
            if count < 16:
                raise ValueError(f"layer {layer} {plane} has only {count} observed exponents")
    return bytes(tables[:, 512:544].contiguous().cpu().numpy().tobytes())


def summarize_symbol_counts(counts) -> dict:
    """The exponent summary the reference's trace records for a 256-bin
    histogram (trace.py:27-58): words, histogram, distinct exponents,
    entropy in bits, and for the top 8 and 16 exponents by (-count,
    exponent) the list, the covered fraction and the escapes."""
    histogram = [int(v) for v in counts]
    words = sum(histogram)
    order = sorted((e for e, c in enumerate(histogram) if c > 0), key=lambda e: (-histogram[e], e))
    # sum() of floats is compensated (as the trace's own summary is)
    entropy = -sum((c / words) * math.log2(c / words) for c in histogram if c > 0) if words else 0.0
    summary = {"words": words, "histogram": histogram, "unique_exponents": len(order), "entropy_bits": entropy}
    for k in (8, 16):
        covered = sum(histogram[e] for e in order[:k])
        summary[f"top{k}_exponents"] = order[:k]
        summary[f"top{k}_coverage"] = covered / words if words else 0.0
        summary[f"top{k}_escape_count"] = words - covered
        summary[f"top{k}_escape_rate"] = (words - covered) / words if words else 0.0
    return summary


# --------------------------------------------------------------- profiler


def profile_enable(on: bool = True) -> None:
    """Start (or stop) bracketing this library's kernel launches with CUDA
    events; clears earlier records."""
    _require_lib().kvq_splitzip_profile_enable(1 if on else 0)


def profile_collect() -> dict[str, tuple[float, int]]:
    """Wait for the recorded launches; {kernel: (total device ms, launches)}."""
    lib = _require_lib()
    count = lib.kvq_splitzip_profile_collect()
    if count < 0:
        _raise_last(lib, "profile collect failed")
    return {
        lib.kvq_splitzip_profile_name(i).decode(): (
            float(lib.kvq_splitzip_profile_ms(i)), int(lib.kvq_splitzip_profile_launches(i)))
        for i in range(count)
    }
