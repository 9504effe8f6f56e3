"""ctypes binding of the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle restates the reference codec (native/unchain_kv/kvq_splitzip_cuda.cu)
on the CPU in canonical form; see splitzip_oracle.c for the file:line map.
Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use it -- as
the checker, never as the product path.

All functions take and return numpy arrays.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import build as _build

_LIB = None
_u64 = ctypes.c_uint64
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p


def lib():
    global _LIB
    if _LIB is None:
        path = _build.ORACLE_SO
        if not path.exists():
            _build.build_oracle()
        handle = ctypes.CDLL(str(path))
        sigs = {
            "orc_top16_capacity": (_u64, [_u64]),
            "orc_top16_encoded_bytes": (_u64, [_u64]),
            "orc_fixed_encoded_bytes": (_u64, [_u64, ctypes.c_int]),
            "orc_encode_top16": (_i64, [_vp, _u64, _vp, _u64, _vp]),
            "orc_encode_top16_blocks": (_i64, [_vp, _u64, _u64, _u64, _vp, _u64, _u64, _vp, _u64, _vp]),
            "orc_top16_escape_count": (_u64, [_vp, _u64, _vp]),
            "orc_decode_top16_blocks": (_i64, [_vp, _u64, _vp, _u64, _u64, _u64, _u64, _u64, _u64, _vp, _vp]),
            "orc_encode_mode": (_i64, [_vp, _u64, _vp, _u64, ctypes.c_int]),
            "orc_encode_mode_blocks": (_i64, [_vp, _u64, _u64, _u64, _vp, _u64, _u64, _vp, _u64, ctypes.c_int]),
            "orc_decode_fixed6_blocks": (_i64, [_vp, _u64, _vp, _u64, _u64, _u64, _u64, _u64, _u64, _vp]),
            "orc_encode_top16_blocks_mt": (_i64, [_vp, _u64, _u64, _u64, _vp, _u64, _u64, _vp, _u64, _vp, ctypes.c_int]),
            "orc_encode_mode_blocks_mt": (_i64, [_vp, _u64, _u64, _u64, _vp, _u64, _u64, _vp, _u64, ctypes.c_int, ctypes.c_int]),
            "orc_decode_fixed6_blocks_mt": (_i64, [_vp, _u64, _vp, _u64, _u64, _u64, _u64, _u64, _u64, _vp, ctypes.c_int]),
            "orc_decode_top16_blocks_mt": (_i64, [_vp, _u64, _vp, _u64, _u64, _u64, _u64, _u64, _u64, _vp, _vp, ctypes.c_int]),
            "orc_max_threads": (ctypes.c_int, []),
            "orc_encode_torchop_blocks": (_i64, [_vp, _u64, _u64, _u64, _vp, _u64, _u64, _vp, _u64]),
            "orc_decode_modes_blocks": (_i64, [_vp, _u64, _vp, _u64, _u64, _u64, _u64, _u64, _vp]),
        }
        for name, (restype, argtypes) in sigs.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _LIB = handle
    return _LIB


def _ptr(array) -> int | None:
    return None if array is None else int(array.ctypes.data)


def _u16(array) -> np.ndarray:
    array = np.ascontiguousarray(array)
    if array.dtype != np.uint16:
        array = array.view(np.uint16)
    return array


def top16_encoded_bytes(n: int) -> int:
    return int(lib().orc_top16_encoded_bytes(n))


def top16_capacity(n: int) -> int:
    return int(lib().orc_top16_capacity(n))


def fixed_encoded_bytes(n: int, bits: int = 6) -> int:
    return int(lib().orc_fixed_encoded_bytes(n, bits))


def encode_top16(words, tables, capacity: int | None = None):
    """Return (result, stream): result is the reference return value."""
    words = _u16(words).reshape(-1)
    n = words.size
    size = max(2 * n, top16_encoded_bytes(n) + 16) if capacity is None else capacity
    out = np.zeros(size, dtype=np.uint8)
    tables = np.ascontiguousarray(tables, dtype=np.uint8)
    result = lib().orc_encode_top16(_ptr(words), n, _ptr(out), size, _ptr(tables))
    return int(result), out[: max(int(result), 0)]


def encode_top16_blocks(cache, block_ids, tables, block_start: int = 0, capacity: int | None = None):
    """Fused gather+encode over a cache shaped [2, num_blocks, ...] (uint16 view)."""
    cache = _u16(cache)
    plane_stride = int(np.prod(cache.shape[1:]))
    block_words = int(np.prod(cache.shape[2:]))
    ids = None if block_ids is None else np.ascontiguousarray(block_ids, dtype=np.int64)
    block_count = len(ids) if ids is not None else int(capacity or 0)
    n = 2 * block_count * block_words
    size = max(2 * n, top16_encoded_bytes(n) + 16) if capacity is None else capacity
    out = np.zeros(size, dtype=np.uint8)
    tables = np.ascontiguousarray(tables, dtype=np.uint8)
    result = lib().orc_encode_top16_blocks(
        _ptr(cache), plane_stride, block_words, block_words, _ptr(ids), block_start,
        block_count, _ptr(out), size, _ptr(tables))
    return int(result), out[: max(int(result), 0)]


def escape_count(words, tables) -> int:
    words = _u16(words).reshape(-1)
    tables = np.ascontiguousarray(tables, dtype=np.uint8)
    return int(lib().orc_top16_escape_count(_ptr(words), words.size, _ptr(tables)))


def decode_top16_blocks(stream, cache, block_ids, tables, raw_words: int | None = None, block_start: int = 0):
    """Decode into ``cache`` (a uint16 numpy array, modified in place)."""
    stream = np.ascontiguousarray(stream, dtype=np.uint8)
    plane_stride = int(np.prod(cache.shape[1:]))
    block_words = int(np.prod(cache.shape[2:]))
    ids = None if block_ids is None else np.ascontiguousarray(block_ids, dtype=np.int64)
    block_count = len(ids)
    n = 2 * block_count * block_words if raw_words is None else raw_words
    tables = np.ascontiguousarray(tables, dtype=np.uint8)
    return int(lib().orc_decode_top16_blocks(
        _ptr(stream), stream.size, _ptr(cache), n, block_count, block_words,
        plane_stride, block_words, block_start, _ptr(ids), _ptr(tables)))


def encode_mode(words, bits: int = 6, capacity: int | None = None):
    words = _u16(words).reshape(-1)
    n = words.size
    size = max(2 * n, fixed_encoded_bytes(n, 6) + 1040) if capacity is None else capacity
    out = np.zeros(size, dtype=np.uint8)
    result = lib().orc_encode_mode(_ptr(words), n, _ptr(out), size, bits)
    return int(result), out[: max(int(result), 0)]


def encode_mode_blocks(cache, block_ids, bits: int = 6, block_start: int = 0, capacity: int | None = None):
    cache = _u16(cache)
    plane_stride = int(np.prod(cache.shape[1:]))
    block_words = int(np.prod(cache.shape[2:]))
    ids = np.ascontiguousarray(block_ids, dtype=np.int64)
    n = 2 * len(ids) * block_words
    size = max(2 * n, fixed_encoded_bytes(n, 6) + 1040) if capacity is None else capacity
    out = np.zeros(size, dtype=np.uint8)
    result = lib().orc_encode_mode_blocks(
        _ptr(cache), plane_stride, block_words, block_words, _ptr(ids), block_start,
        len(ids), _ptr(out), size, bits)
    return int(result), out[: max(int(result), 0)]


def decode_fixed6_blocks(stream, cache, block_ids, block_start: int = 0):
    stream = np.ascontiguousarray(stream, dtype=np.uint8)
    plane_stride = int(np.prod(cache.shape[1:]))
    block_words = int(np.prod(cache.shape[2:]))
    ids = np.ascontiguousarray(block_ids, dtype=np.int64)
    n = 2 * len(ids) * block_words
    return int(lib().orc_decode_fixed6_blocks(
        _ptr(stream), stream.size, _ptr(cache), n, len(ids), block_words,
        plane_stride, block_words, block_start, _ptr(ids)))


def encode_torchop_blocks(cache, block_ids, block_start: int = 0):
    """The reference's torch-op encoder (modes 2, 0, 1 in that order) over the
    blocks; (length, stream), length 0 when no form is smaller than raw."""
    cache = _u16(cache)
    plane_stride = int(np.prod(cache.shape[1:]))
    block_words = int(np.prod(cache.shape[2:]))
    ids = np.ascontiguousarray(block_ids, dtype=np.int64)
    n = 2 * len(ids) * block_words
    out = np.zeros(2 * n + 512, dtype=np.uint8)
    result = lib().orc_encode_torchop_blocks(
        _ptr(cache), plane_stride, block_words, block_words, _ptr(ids), block_start, len(ids), _ptr(out), out.size)
    return int(result), out[: max(int(result), 0)]


def decode_modes_blocks(stream, cache, block_ids, block_start: int = 0):
    """Receiver decode of a mode 0/1/2/4 stream into ``cache`` (in place);
    returns 2n, or 0 when the stream is declined."""
    stream = np.ascontiguousarray(stream, dtype=np.uint8)
    plane_stride = int(np.prod(cache.shape[1:]))
    block_words = int(np.prod(cache.shape[2:]))
    ids = np.ascontiguousarray(block_ids, dtype=np.int64)
    return int(lib().orc_decode_modes_blocks(
        _ptr(stream), stream.size, _ptr(cache), len(ids), block_words, plane_stride, block_words,
        block_start, _ptr(ids)))


def encode_auto_blocks(cache, block_ids, tables, raw_ok: bool = True, threads: int | None = None) -> np.ndarray:
    """The reference producer's codec chain on one job, in canonical form:
    top16 when the escapes fit its capacity (vllm_connector.py:3104-3118),
    else fixed6 when at most 64 high bytes occur, else raw mode 6 ([6] + the
    words) when ``raw_ok`` (vllm_connector.py:4557-4633), else the fixed6
    overflow stream (mode 255).  Multi-threaded (OpenMP) over the job's
    words.  Returns the stream bytes."""
    cache = _u16(cache)
    plane_stride = int(np.prod(cache.shape[1:]))
    block_words = int(np.prod(cache.shape[2:]))
    ids = np.ascontiguousarray(block_ids, dtype=np.int64)
    n = 2 * len(ids) * block_words
    threads = threads or max_threads()
    tables = np.ascontiguousarray(tables, dtype=np.uint8)
    out = np.zeros(2 * n + 4096, dtype=np.uint8)
    res = lib().orc_encode_top16_blocks_mt(_ptr(cache), plane_stride, block_words, block_words, _ptr(ids), 0,
                                           len(ids), _ptr(out), out.size, _ptr(tables), threads)
    if res > 0 and out[0] == 5:
        return out[:res].copy()
    res = lib().orc_encode_mode_blocks_mt(_ptr(cache), plane_stride, block_words, block_words, _ptr(ids), 0,
                                          len(ids), _ptr(out), out.size, 6, threads)
    if res > 0 and out[0] == 3:
        return out[:res].copy()
    if raw_ok:
        words = np.ascontiguousarray(cache[:, ids]).reshape(-1)
        return np.concatenate([np.array([6], dtype=np.uint8), words.view(np.uint8)])
    return out[:max(int(res), 0)].copy()


def max_threads() -> int:
    return int(lib().orc_max_threads())


def reference_library_path() -> Path | None:
    """Path of the reference CUDA codec compiled from source, if built."""
    path = _build.REF_SO
    return path if path.exists() else None
