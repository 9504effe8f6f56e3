import pytest

from unchainkv_b200.tensor_blocks import merge_block_bytes, split_block_bytes


def test_split_and_merge_block_bytes():
    data = b"abcdefghijkl"
    chunks = list(split_block_bytes(data, chunk_size=5))
    assert chunks == [(0, b"abcde"), (5, b"fghij"), (10, b"kl")]
    assert merge_block_bytes(len(data), chunks) == data


def test_split_rejects_nonpositive_chunk_and_merge_rejects_outside():
    with pytest.raises(ValueError):
        list(split_block_bytes(b"abc", 0))
    with pytest.raises(ValueError):
        merge_block_bytes(4, [(2, b"abc")])
    assert merge_block_bytes(4, [(1, b"x")]) == b"\x00x\x00\x00"
    assert list(split_block_bytes(b"", 3)) == []
