"""Host-side behaviour of unchainkv_b200.splitzip_cuda without a GPU.

Restates the ABI marshalling checks of the reference's
tests/test_splitzip_cuda.py:10-90, 187-336 (argument order of every call, the
layer bound of the codebook table, record_stream of the block-id tensor)
against this package's operator API, using fake libraries and tensors."""

import sys
from types import SimpleNamespace
from unittest.mock import patch

import pytest

import unchainkv_b200.splitzip_cuda as splitzip_cuda


class FakeTensor:
    def __init__(self, ptr, shape, stride, dtype, device):
        self._ptr = ptr
        self.shape = shape
        self._stride = stride
        self.dtype = dtype
        self.device = device

    def data_ptr(self):
        return self._ptr

    def numel(self):
        result = 1
        for size in self.shape:
            result *= size
        return result

    def dim(self):
        return len(self.shape)

    def stride(self, dim):
        return self._stride[dim]

    def is_contiguous(self):
        return True


class FakeBlockIds(FakeTensor):
    def __init__(self, device, int64):
        super().__init__(55, (2,), (1,), int64, device)
        self.streams = []

    def record_stream(self, stream):
        self.streams.append(stream)


@pytest.fixture
def fake_env():
    device = SimpleNamespace(type="cuda")
    uint8, bfloat16, int64 = object(), object(), object()
    current = SimpleNamespace(cuda_stream=99)
    block_map = FakeBlockIds(device, int64)
    torch = SimpleNamespace(
        uint8=uint8, bfloat16=bfloat16, int64=int64,
        tensor=lambda *_a, **_k: block_map,
        cuda=SimpleNamespace(current_stream=lambda _device: current),
    )
    return SimpleNamespace(device=device, uint8=uint8, bfloat16=bfloat16, torch=torch,
                           current=current, block_map=block_map)


def with_lib(lib):
    old = splitzip_cuda._LIB
    splitzip_cuda._LIB = lib

    class Restore:
        def __enter__(self):
            return lib

        def __exit__(self, *exc):
            splitzip_cuda._LIB = old

    return Restore()


def test_top16_layer_bound_follows_codebook_count():
    layers = len(splitzip_cuda._TOP16_CODEBOOKS) // 32
    assert layers == 32
    assert splitzip_cuda._top16_tables(layers, "cuda", object()) is None
    assert splitzip_cuda._top16_tables(-1, "cuda", object()) is None


def test_top16_wrappers_pass_static_tables_to_cuda(fake_env):
    encode_calls, decode_calls = [], []

    class FakeLib:
        def kvq_splitzip_bf16_encode_top16(self, *args):
            encode_calls.append(args)
            return 13

        def kvq_splitzip_bf16_decode_top16(self, *args):
            decode_calls.append(args)
            return 16

    e = fake_env
    source = FakeTensor(11, (8,), (1,), e.bfloat16, e.device)
    encoded = FakeTensor(22, (32,), (1,), e.uint8, e.device)
    target = FakeTensor(33, (2, 8, 2), (16, 2, 1), e.bfloat16, e.device)
    tables = FakeTensor(44, (544,), (1,), e.uint8, e.device)
    with with_lib(FakeLib()), patch.dict(sys.modules, {"torch": e.torch}), patch.object(
        splitzip_cuda, "_top16_tables", return_value=tables
    ):
        assert splitzip_cuda.encode_top16(source, encoded, 7) == 13
        assert splitzip_cuda.decode_top16(encoded, target, [3, 4], 16, 7) == 16
    assert encode_calls == [(11, 22, 8, 32, 44, 99)]
    assert decode_calls == [(22, 32, 33, 8, 2, 2, 16, 2, 3, 44, 99)]


def test_decode_fixed6_passes_contiguous_native_layout_to_cuda(fake_env):
    calls = []

    class FakeLib:
        def kvq_splitzip_bf16_decode_fixed6(self, *args):
            calls.append(args)
            return 16

    e = fake_env
    source = FakeTensor(11, (79,), (1,), e.uint8, e.device)
    target = FakeTensor(22, (2, 8, 2), (16, 2, 1), e.bfloat16, e.device)
    with with_lib(FakeLib()), patch.dict(sys.modules, {"torch": e.torch}):
        assert splitzip_cuda.decode_fixed6(source, target, [3, 4], 16) == 16
    assert calls == [(11, 79, 22, 8, 2, 2, 16, 2, 3, 99)]


def test_native_decoders_pass_noncontiguous_block_map_to_cuda(fake_env):
    fixed_calls, top16_calls = [], []

    class FakeLib:
        def kvq_splitzip_bf16_decode_fixed6(self, *_args):
            raise AssertionError("contiguous decoder used")

        def kvq_splitzip_bf16_decode_fixed6_blocks(self, *args):
            fixed_calls.append(args)
            return 16

        def kvq_splitzip_bf16_decode_top16(self, *_args):
            raise AssertionError("contiguous decoder used")

        def kvq_splitzip_bf16_decode_top16_blocks(self, *args):
            top16_calls.append(args)
            return 16

    e = fake_env
    source = FakeTensor(11, (79,), (1,), e.uint8, e.device)
    target = FakeTensor(22, (2, 8, 2), (16, 2, 1), e.bfloat16, e.device)
    tables = FakeTensor(44, (544,), (1,), e.uint8, e.device)
    with with_lib(FakeLib()), patch.dict(sys.modules, {"torch": e.torch}), patch.object(
        splitzip_cuda, "_top16_tables", return_value=tables
    ):
        fixed = splitzip_cuda.decode_fixed6(source, target, [3, 5], 16)
        top16 = splitzip_cuda.decode_top16(source, target, [3, 5], 16, 7)
    assert (fixed, top16) == (16, 16)
    assert fixed_calls == [(11, 79, 22, 8, 2, 2, 16, 2, 3, 55, 99)]
    assert top16_calls == [(11, 79, 22, 8, 2, 2, 16, 2, 3, 55, 44, 99)]
    assert e.block_map.streams == [e.current, e.current]


def test_encode_bf16_rejects_bad_bits_and_non_cuda(fake_env):
    class FakeLib:
        def kvq_splitzip_bf16_encode_mode(self, *args):
            return 100

    e = fake_env
    source = FakeTensor(11, (8,), (1,), e.bfloat16, e.device)
    out = FakeTensor(22, (32,), (1,), e.uint8, e.device)
    cpu = FakeTensor(11, (8,), (1,), e.bfloat16, SimpleNamespace(type="cpu"))
    with with_lib(FakeLib()), patch.dict(sys.modules, {"torch": e.torch}):
        assert splitzip_cuda.encode_bf16(cpu, out) is None
        with pytest.raises(ValueError):
            splitzip_cuda.encode_bf16(source, out, bits=4)
        assert splitzip_cuda.encode_bf16(source, out, bits=5) == 100


def test_decode_layout_rejections_match_reference(fake_env):
    class FakeLib:
        def kvq_splitzip_bf16_decode_fixed6(self, *args):
            raise AssertionError("should have been rejected")

    e = fake_env
    source = FakeTensor(11, (79,), (1,), e.uint8, e.device)
    target = FakeTensor(22, (2, 8, 2), (16, 2, 1), e.bfloat16, e.device)
    with with_lib(FakeLib()), patch.dict(sys.modules, {"torch": e.torch}):
        assert splitzip_cuda.decode_fixed6(source, target, [], 16) is None  # no blocks
        assert splitzip_cuda.decode_fixed6(source, target, [3, 3], 16) is None  # duplicates
        assert splitzip_cuda.decode_fixed6(source, target, [3, 8], 16) is None  # out of range
        assert splitzip_cuda.decode_fixed6(source, target, [3, 4], 15) is None  # odd bytes
        assert splitzip_cuda.decode_fixed6(source, target, [3, 4], 12) is None  # 6 words / 4


def test_launch_failure_raises_library_message(fake_env):
    class FakeLib:
        def kvq_splitzip_bf16_encode_top16(self, *args):
            return -1

        def kvq_splitzip_last_error(self):
            return b"EncodeTop16Kernel: invalid argument"

    e = fake_env
    source = FakeTensor(11, (8,), (1,), e.bfloat16, e.device)
    out = FakeTensor(22, (32,), (1,), e.uint8, e.device)
    tables = FakeTensor(44, (544,), (1,), e.uint8, e.device)
    with with_lib(FakeLib()), patch.dict(sys.modules, {"torch": e.torch}), patch.object(
        splitzip_cuda, "_top16_tables", return_value=tables
    ):
        with pytest.raises(RuntimeError, match="EncodeTop16Kernel: invalid argument"):
            splitzip_cuda.encode_top16(source, out, 0)


def test_missing_library_fails_loudly_for_cuda_tensors(fake_env, monkeypatch):
    e = fake_env
    monkeypatch.setenv("UNCHAIN_KV_SPLITZIP_LIB", "/nonexistent/libnothing.so")
    old = splitzip_cuda._LIB
    splitzip_cuda._LIB = None
    try:
        assert not splitzip_cuda.available()
        assert "libnothing" in (splitzip_cuda.load_error() or "")
        source = FakeTensor(11, (8,), (1,), e.bfloat16, e.device)
        out = FakeTensor(22, (32,), (1,), e.uint8, e.device)
        with patch.dict(sys.modules, {"torch": e.torch}):
            with pytest.raises(RuntimeError, match="not loadable"):
                splitzip_cuda.encode_top16(source, out, 0)
    finally:
        splitzip_cuda._LIB = old
        splitzip_cuda._LOAD_ERROR = None


def test_register_codebooks_changes_layer_bound_and_tables():
    books = bytes(range(32)) * 3
    try:
        assert splitzip_cuda.register_top16_codebooks(books) == 3
        assert len(splitzip_cuda._TOP16_CODEBOOKS) // 32 == 3
        assert splitzip_cuda._top16_tables(3, "cuda", object()) is None
        tables = splitzip_cuda.build_top16_tables(books[32:64])
        assert tables[:16] == bytes(range(16)) and tables[16:256] == b"\xff" * 240
        with pytest.raises(ValueError):
            splitzip_cuda.register_top16_codebooks(b"\x00" * 33)
    finally:
        splitzip_cuda.register_top16_codebooks(None)
    assert len(splitzip_cuda._TOP16_CODEBOOKS) // 32 == 32


def test_table_builder_later_duplicates_win():
    books = bytes([5] * 16 + list(range(100, 116)))
    tables = splitzip_cuda.build_top16_tables(books)
    assert tables[5] == 15  # last code mapping to exponent 5
    assert tables[256 + 100] == 0 and tables[256 + 115] == 15
