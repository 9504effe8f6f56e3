"""Byte chunking of block payloads (host side, no GPU work).

Same API and behaviour as src/unchain_kv/tensor_blocks.py:6-20 of the
reference, which the legacy chunk path of the connector uses
(vllm_connector.py:2325).
"""

from __future__ import annotations

from collections.abc import Iterable, Iterator


def split_block_bytes(data: bytes, chunk_size: int) -> Iterator[tuple[int, bytes]]:
    """Yield (offset, chunk) pairs covering ``data`` in ``chunk_size`` pieces;
    the last piece may be shorter."""
    if chunk_size <= 0:
        raise ValueError("chunk_size must be positive")
    view = bytes(data)
    offset = 0
    while offset < len(view):
        yield offset, view[offset : offset + chunk_size]
        offset += chunk_size


def merge_block_bytes(size: int, chunks: Iterable[tuple[int, bytes]]) -> bytes:
    """Reassemble ``size`` bytes from (offset, chunk) pairs; bytes no chunk
    covers stay zero.  A chunk reaching outside [0, size) raises ValueError."""
    buffer = bytearray(size)
    for offset, chunk in chunks:
        stop = offset + len(chunk)
        if offset < 0 or stop > size:
            raise ValueError("chunk outside block")
        buffer[offset:stop] = chunk
    return bytes(buffer)
