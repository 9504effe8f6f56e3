"""GPU parity of the sm_100a codec against the CPU oracle (bit-exact), through
the C ABI, plus cross-checks against the reference's own CUDA codec compiled
from its source (oracle/_ref) where that library is present."""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from unchainkv_b200 import splitzip_cuda, workloads  # noqa: E402

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

def tables_for(layer: int) -> np.ndarray:
    return np.frombuffer(
        splitzip_cuda.build_top16_tables(splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[layer * 32 : layer * 32 + 32]),
        dtype=np.uint8,
    )


def dev(array) -> "torch.Tensor":
    return torch.from_numpy(np.array(array, copy=True, order="C")).cuda()


def words_dev(words: np.ndarray) -> "torch.Tensor":
    return dev(words.view(np.int16)).view(torch.bfloat16)


def host_u16(t) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def lib():
    handle = splitzip_cuda._load()
    assert handle is not None, splitzip_cuda.load_error()
    return handle


def book_words(rng, shape, books: bytes, escape_rate=0.0, plane_axis_first=True):
    """bf16 words whose exponents come from the plane's book, with escapes."""
    n = int(np.prod(shape))
    flat_plane = (np.arange(n) >= n // 2).astype(np.int64)
    book = np.frombuffer(books, dtype=np.uint8).reshape(2, 16)
    exp = book[flat_plane, rng.integers(0, 16, size=n)].astype(np.int64)
    outside = np.array([v for v in range(256) if v not in set(books)], dtype=np.int64)
    if escape_rate:
        mask = rng.random(n) < escape_rate
        exp[mask] = rng.choice(outside, size=int(mask.sum()))
    words = (rng.integers(0, 2, size=n) << 15) | (exp << 7) | rng.integers(0, 128, size=n)
    return words.astype(np.uint16).reshape(shape)


def gpu_encode_top16(words: np.ndarray, tables: np.ndarray, capacity=None):
    n = words.size
    cap = capacity if capacity is not None else 2 * n
    src = words_dev(words.reshape(-1))
    out = torch.full((cap,), 0xAB, dtype=torch.uint8, device="cuda")
    tab = dev(tables)
    res = lib().kvq_splitzip_bf16_encode_top16(src.data_ptr(), out.data_ptr(), n, cap,
                                                tab.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return res, out.cpu().numpy()[: max(res, 0)]


# ---------------------------------------------------------------- top16 encode

@pytest.mark.parametrize("n", [22, 256, 1000, 1001, 8192, 8195, 3 * 8192 + 100, 16384, 16384 + 3, 3 * 16384 + 100, 1 << 20])
@pytest.mark.parametrize("rate", [0.0, 0.002, 0.0049, 0.03])
def test_top16_encode_flat_matches_oracle(n, rate):
    rng = np.random.Generator(np.random.PCG64(n * 7 + int(rate * 1e4)))
    tables = tables_for(n % 32)
    words = book_words(rng, (n,), splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[(n % 32) * 32:][:32], rate)
    capacity = max(2 * n, splitzip_cuda.top16_capacity(n))
    expected_res, expected = oracle.encode_top16(words, tables, capacity=capacity)
    res, stream = gpu_encode_top16(words, tables, capacity=capacity)
    assert res == expected_res > 0
    assert np.array_equal(stream, expected), (n, rate, np.flatnonzero(stream != expected)[:10])


def test_top16_encode_declines_like_reference():
    tables = tables_for(0)
    assert gpu_encode_top16(np.zeros(21, np.uint16), tables)[0] == 0   # does not compress
    n = 1 << 16
    enc = oracle.top16_encoded_bytes(n)
    # the reference's rule: align4(encoded) + 8 <= capacity (.cu:390-394)
    words = np.zeros(n, np.uint16)
    need = splitzip_cuda.top16_capacity(n)
    assert need == (enc + 3) // 4 * 4 + 8
    assert gpu_encode_top16(words, tables, capacity=need)[0] == enc
    assert gpu_encode_top16(words, tables, capacity=need - 1)[0] == 0
    assert gpu_encode_top16(words, tables, capacity=enc + 4)[0] == 0


@pytest.mark.parametrize("n", [22, 47, 1000, 8192, 8192 + 30, 8192 + 47, 8192 + 63, 5 * 8192 + 4096, 16384 + 30,
                               16384 + 47, 16384 + 63, 3 * 16384 + 8192, 1 << 20])
@pytest.mark.parametrize("rate", [0.002, 0.0049, 0.03])
@pytest.mark.parametrize("shift", [0, 3, 11])
def test_top16_encode_at_the_reference_capacity(n, rate, shift):
    """A buffer of exactly align4(encoded) + 8 bytes, at any byte alignment:
    the stream equals the oracle's, and no byte past the buffer changes (the
    encoder keeps its per-tile counts inside the stream's own regions)."""
    rng = np.random.Generator(np.random.PCG64(n * 13 + shift + int(rate * 1e4)))
    tables = tables_for(n % 32)
    words = book_words(rng, (n,), splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[(n % 32) * 32:][:32], rate)
    cap = splitzip_cuda.top16_capacity(n)
    expected_res, expected = oracle.encode_top16(words, tables, capacity=cap)
    assert expected_res == oracle.top16_encoded_bytes(n)
    src = words_dev(words.reshape(-1))
    arena = torch.full((cap + 64,), 0xA5, dtype=torch.uint8, device="cuda")
    out = arena[shift:shift + cap]
    tab = dev(tables)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # the second call finds the first one's bytes in the buffer
        res = lib().kvq_splitzip_bf16_encode_top16(src.data_ptr(), out.data_ptr(), n, cap, tab.data_ptr(), stream)
        torch.cuda.synchronize()
        assert res == expected_res
        got = arena.cpu().numpy()
        assert np.array_equal(got[shift:shift + res], expected), np.flatnonzero(got[shift:shift + res] != expected)[:8]
        assert (got[:shift] == 0xA5).all() and (got[shift + cap:] == 0xA5).all()


@pytest.mark.parametrize("shape,pool", [((16, 8, 128), 96), ((16, 1, 128), 300), ((3, 5), 50), ((16, 2, 64), 40)])
@pytest.mark.parametrize("contiguous", [False, True])
def test_top16_fused_gather_matches_index_select_then_encode(shape, pool, contiguous):
    rng = np.random.Generator(np.random.PCG64(sum(shape) + pool))
    blocks = pool // 3
    ids = np.arange(5, 5 + blocks) if contiguous else rng.permutation(pool)[:blocks]
    books = splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[64:96]
    cache = book_words(rng, (2, pool) + shape, books, 0.003)
    tables = tables_for(2)
    expected_res, expected = oracle.encode_top16_blocks(cache, ids, tables)
    assert expected_res > 0
    kv = words_dev(cache)
    out = torch.zeros(4 * cache[:, ids].size, dtype=torch.uint8, device="cuda")
    block_ids = list(map(int, ids))
    res = splitzip_cuda.encode_top16_blocks(kv, block_ids, out, tables=dev(tables))
    torch.cuda.synchronize()
    assert res == expected_res
    assert np.array_equal(out.cpu().numpy()[:res], expected)


# ---------------------------------------------------------------- top16 decode

def gpu_decode_top16(stream: np.ndarray, cache_shape, ids, tables, fill=0x1234):
    cache = torch.full(cache_shape, fill, dtype=torch.int16, device="cuda").view(torch.bfloat16)
    src = dev(stream)
    block_words = int(np.prod(cache_shape[2:]))
    n = 2 * len(ids) * block_words
    ids_t = dev(np.asarray(ids, dtype=np.int64))
    res = lib().kvq_splitzip_bf16_decode_top16_blocks(
        src.data_ptr(), stream.size, cache.data_ptr(), n, len(ids), block_words,
        cache.stride(0), cache.stride(1), 0, ids_t.data_ptr(), dev(tables).data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return res, host_u16(cache)


@pytest.mark.parametrize("shape,pool,rate", [((16, 8, 128), 40, 0.003), ((16, 1, 128), 200, 0.0049),
                                              ((7, 3), 30, 0.004), ((16, 8, 128), 20, 0.0)])
def test_top16_decode_scatter_matches_oracle(shape, pool, rate):
    rng = np.random.Generator(np.random.PCG64(pool + int(rate * 1e5)))
    blocks = pool // 2
    ids = rng.permutation(pool)[:blocks]
    books = splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[96:128]
    tables = tables_for(3)
    cache = book_words(rng, (2, pool) + shape, books, rate)
    res, stream = oracle.encode_top16_blocks(cache, ids, tables)
    assert res > 0 and stream[0] == 5
    expected = np.full(cache.shape, 0x1234, dtype=np.uint16)
    assert oracle.decode_top16_blocks(stream, expected, ids, tables) == 2 * cache[:, ids].size
    got_res, got = gpu_decode_top16(stream, cache.shape, ids, tables)
    assert got_res == 2 * cache[:, ids].size
    assert np.array_equal(got, expected)
    assert np.array_equal(got[:, ids], cache[:, ids])  # lossless round trip


def test_top16_decode_accepts_unsorted_escape_entries():
    """Reference streams list escapes in atomic (arbitrary) order."""
    rng = np.random.Generator(np.random.PCG64(99))
    pool, blocks, shape = 64, 40, (16, 8, 128)
    ids = rng.permutation(pool)[:blocks]
    tables = tables_for(4)
    cache = book_words(rng, (2, pool) + shape, splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[128:160], 0.004)
    res, stream = oracle.encode_top16_blocks(cache, ids, tables)
    n = 2 * blocks * int(np.prod(shape))
    count = int.from_bytes(stream[1:5].tobytes(), "little")
    assert count > 100
    entries_at = 5 + n + (n + 1) // 2
    entries = stream[entries_at : entries_at + 5 * count].reshape(count, 5).copy()
    shuffled = stream.copy()
    shuffled[entries_at : entries_at + 5 * count] = entries[rng.permutation(count)].reshape(-1)
    for _ in range(3):  # the fallback state is reset between calls
        got_res, got = gpu_decode_top16(shuffled, cache.shape, ids, tables)
        assert got_res == 2 * n
        assert np.array_equal(got[:, ids], cache[:, ids])
    # a sorted stream still decodes after unsorted ones
    assert np.array_equal(gpu_decode_top16(stream, cache.shape, ids, tables)[1][:, ids], cache[:, ids])


def test_top16_decode_ignores_overflow_streams_and_bad_lengths():
    rng = np.random.Generator(np.random.PCG64(3))
    pool, blocks, shape = 16, 8, (16, 8, 128)
    ids = rng.permutation(pool)[:blocks]
    tables = tables_for(0)
    cache = book_words(rng, (2, pool) + shape, splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[:32], 0.05)
    res, stream = oracle.encode_top16_blocks(cache, ids, tables)
    assert stream[0] == 255
    got_res, got = gpu_decode_top16(stream, cache.shape, ids, tables)
    n = 2 * blocks * int(np.prod(shape))
    assert got_res == 2 * n  # reference quirk: reports bytes, writes nothing
    assert (got == 0x1234).all()
    assert gpu_decode_top16(stream[:-1], cache.shape, ids, tables)[0] == 0


def test_top16_overflow_stream_is_canonical():
    rng = np.random.Generator(np.random.PCG64(8))
    n = 5 * 8192 + 17
    words = book_words(rng, (n,), splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[:32], 0.02)
    tables = tables_for(0)
    expected_res, expected = oracle.encode_top16(words, tables)
    assert expected[0] == 255
    res, stream = gpu_encode_top16(words, tables)
    assert res == expected_res and np.array_equal(stream, expected)


# ---------------------------------------------------------------- fixed6/fixed5

def distinct_words(rng, n, distinct):
    highs = np.sort(rng.choice(256, size=distinct, replace=False)).astype(np.uint16)
    return ((highs[rng.integers(0, distinct, size=n)] << 8) | rng.integers(0, 256, size=n)).astype(np.uint16)


@pytest.mark.parametrize("bits", [6, 5])
@pytest.mark.parametrize("n,distinct", [(400, 5), (8192, 64), (8195, 30), (3 * 8192 + 999, 33), (1 << 20, 36)])
def test_fixed_encode_flat_matches_oracle(bits, n, distinct):
    if bits == 5:
        distinct = min(distinct, 32)
    rng = np.random.Generator(np.random.PCG64(n + distinct + bits))
    words = distinct_words(rng, n, distinct)
    cap = max(2 * n, oracle.fixed_encoded_bytes(n, bits) + 1040)
    expected_res, expected = oracle.encode_mode(words, bits=bits, capacity=cap)
    assert expected_res > 0
    src = words_dev(words)
    out = torch.full((cap,), 0xCD, dtype=torch.uint8, device="cuda")
    res = lib().kvq_splitzip_bf16_encode_mode(src.data_ptr(), out.data_ptr(), n, cap,
                                               torch.cuda.current_stream().cuda_stream, bits)
    torch.cuda.synchronize()
    assert res == expected_res
    assert np.array_equal(out.cpu().numpy()[:res], expected)


@pytest.mark.parametrize("bits,limit", [(6, 64), (5, 32)])
def test_fixed_overflow_header_and_palette(bits, limit):
    rng = np.random.Generator(np.random.PCG64(bits))
    n = 20000
    words = distinct_words(rng, n, limit + 7)
    expected_res, expected = oracle.encode_mode(words, bits=bits)
    assert expected[0] == 255
    src = words_dev(words)
    out = torch.zeros((2 * n,), dtype=torch.uint8, device="cuda")
    res = lib().kvq_splitzip_bf16_encode_mode(src.data_ptr(), out.data_ptr(), n, 2 * n,
                                               torch.cuda.current_stream().cuda_stream, bits)
    torch.cuda.synchronize()
    assert res == expected_res
    got = out.cpu().numpy()
    assert np.array_equal(got[: 1 + limit], expected[: 1 + limit])


@pytest.mark.parametrize("shape,pool", [((16, 8, 128), 64), ((16, 1, 128), 256), ((5, 31), 20)])
def test_fixed6_fused_gather_and_decode_scatter(shape, pool):
    rng = np.random.Generator(np.random.PCG64(pool))
    blocks = pool // 2
    ids = rng.permutation(pool)[:blocks]
    cache = distinct_words(rng, 2 * pool * int(np.prod(shape)), 40).reshape((2, pool) + shape)
    expected_res, expected = oracle.encode_mode_blocks(cache, ids, bits=6)
    kv = words_dev(cache)
    out = torch.zeros(4 * cache[:, ids].size, dtype=torch.uint8, device="cuda")
    res = splitzip_cuda.encode_bf16_blocks(kv, list(map(int, ids)), out, bits=6)
    torch.cuda.synchronize()
    assert res == expected_res
    assert np.array_equal(out.cpu().numpy()[:res], expected)
    # decode into a second cache with a different block table
    ids2 = rng.permutation(pool)[:blocks]
    target = torch.zeros_like(kv)
    copied = splitzip_cuda.decode_fixed6(out[:res], target, list(map(int, ids2)), 2 * cache[:, ids].size)
    torch.cuda.synchronize()
    assert copied == 2 * cache[:, ids].size
    ref_target = np.zeros_like(cache)
    oracle.decode_fixed6_blocks(expected, ref_target, ids2)
    assert np.array_equal(host_u16(target), ref_target)
    assert np.array_equal(host_u16(target)[:, ids2], cache[:, ids])


def test_misaligned_source_uses_plain_loads():
    rng = np.random.Generator(np.random.PCG64(21))
    n = 3 * 8192 + 5
    words = book_words(rng, (n + 3,), splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[:32], 0.003)
    tables = tables_for(0)
    full = words_dev(words)
    src = full[3:]  # 6-byte offset: not 16-byte aligned
    out = torch.zeros(2 * n, dtype=torch.uint8, device="cuda")
    res = lib().kvq_splitzip_bf16_encode_top16(src.data_ptr(), out.data_ptr(), n, 2 * n,
                                                dev(tables).data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    expected_res, expected = oracle.encode_top16(words[3:], tables)
    assert res == expected_res and np.array_equal(out.cpu().numpy()[:res], expected)
    fout = torch.zeros(2 * n, dtype=torch.uint8, device="cuda")
    res6 = lib().kvq_splitzip_bf16_encode_mode(src.data_ptr(), fout.data_ptr(), n, 2 * n,
                                                torch.cuda.current_stream().cuda_stream, 6)
    torch.cuda.synchronize()
    e6, s6 = oracle.encode_mode(words[3:], bits=6)
    assert res6 == e6
    assert np.array_equal(fout.cpu().numpy()[: 1 + 64], s6[: 1 + 64])
    if s6[0] == 3:
        assert np.array_equal(fout.cpu().numpy()[:res6], s6)


# ---------------------------------------------------------------- API round trips

def test_reference_api_round_trips_like_reference_tests():
    """The scenarios of the reference's GPU tests
    (tests/test_splitzip_cuda.py:92-185) through this package's API."""
    count = 2 * 128 * 2048
    index = torch.arange(count, dtype=torch.int32, device="cuda")
    palette = torch.tensor([0x3F, 0x40, 0xBF, 0xC0], device="cuda")
    high = palette[torch.remainder(index, 4)]
    words = torch.bitwise_or(torch.bitwise_left_shift(high, 8), torch.remainder(index, 251)).to(torch.uint16)
    source = words.view(torch.bfloat16).reshape(2, 128, 2048)
    raw_bytes = source.numel() * 2
    encoded = torch.empty(raw_bytes, dtype=torch.uint8, device="cuda")
    encoded_bytes = splitzip_cuda.encode_bf16(source, encoded)
    assert encoded_bytes
    target = torch.zeros((2, 256, 2048), dtype=torch.bfloat16, device="cuda")
    block_ids = list(range(64, 128)) + list(range(192, 256))
    copied = splitzip_cuda.decode_fixed6(encoded[:encoded_bytes], target, block_ids, raw_bytes)
    torch.cuda.synchronize()
    assert copied == raw_bytes
    assert torch.equal(target[:, block_ids].view(torch.uint16), source.view(torch.uint16))

    for block_count, target_blocks, ids in ((1, 4, [3]), (128, 256, list(range(0, 256, 2)))):
        count = 2 * block_count * 2048
        index = torch.arange(count, dtype=torch.int32, device="cuda")
        codebooks = torch.tensor(list(splitzip_cuda._TOP16_CODEBOOKS[:32]), device="cuda").reshape(2, 16)
        plane = torch.div(index, count // 2, rounding_mode="floor")
        exponent = codebooks[plane.long(), torch.remainder(index, 16).long()]
        exponent[::400] = 100
        words = torch.bitwise_or(
            torch.bitwise_left_shift(torch.remainder(index, 2), 15),
            torch.bitwise_or(torch.bitwise_left_shift(exponent.to(torch.int32), 7), torch.remainder(index, 128)),
        ).to(torch.uint16)
        source = words.view(torch.bfloat16).reshape(2, block_count, 2048)
        raw_bytes = source.numel() * 2
        encoded = torch.empty(raw_bytes, dtype=torch.uint8, device="cuda")
        encoded_bytes = splitzip_cuda.encode_top16(source, encoded, 0)
        assert encoded_bytes
        target = torch.zeros((2, target_blocks, 2048), dtype=torch.bfloat16, device="cuda")
        copied = splitzip_cuda.decode_top16(encoded[:encoded_bytes], target, ids, raw_bytes, 0)
        torch.cuda.synchronize()
        assert raw_bytes / encoded_bytes >= 1.30
        assert int(encoded[0].item()) == 5
        assert copied == raw_bytes
        assert torch.equal(target[:, ids].view(torch.uint16), source.view(torch.uint16))


def test_config0_pipeline_matches_oracle():
    cfg = workloads.CONFIG0
    pool = cfg.blocks * cfg.pool_factor
    ids = workloads.block_table(pool, cfg.blocks, 3000)
    cache = workloads.paged_cache_host(cfg, 0, ids)
    books = workloads.layer_codebooks(0)
    tables = np.frombuffer(splitzip_cuda.build_top16_tables(books), np.uint8)
    kv = words_dev(cache)
    out = torch.zeros(2 * cfg.words_per_layer, dtype=torch.uint8, device="cuda")
    res = splitzip_cuda.encode_top16_blocks(kv, list(map(int, ids)), out, tables=dev(tables))
    torch.cuda.synchronize()
    eres, estream = oracle.encode_top16_blocks(cache, ids, tables)
    assert res == eres and np.array_equal(out.cpu().numpy()[:res], estream)
    assert estream[0] == 255  # this distribution overflows the 0.5% escape capacity
    res6 = splitzip_cuda.encode_bf16_blocks(kv, list(map(int, ids)), out, bits=6)
    torch.cuda.synchronize()
    e6, s6 = oracle.encode_mode_blocks(cache, ids, bits=6)
    assert res6 == e6 and s6[0] == 3 and np.array_equal(out.cpu().numpy()[:res6], s6)
    ids2 = workloads.block_table(pool, cfg.blocks, 3001)
    target = torch.zeros_like(kv)
    assert splitzip_cuda.decode_fixed6(out[:res6], target, list(map(int, ids2)), 2 * cfg.words_per_layer)
    torch.cuda.synchronize()
    assert np.array_equal(host_u16(target)[:, ids2], cache[:, ids])


# ------------------------------------------------ reference kernels (from source)

def ref_lib():
    path = oracle.reference_library_path()
    if path is None:
        pytest.skip("reference CUDA codec not built (oracle/build.py)")
    handle = ctypes.CDLL(str(path))
    for name in ("kvq_splitzip_bf16_encode_top16", "kvq_splitzip_bf16_decode_top16_blocks",
                 "kvq_splitzip_bf16_encode_mode", "kvq_splitzip_bf16_decode_fixed6_blocks"):
        getattr(handle, name).restype = ctypes.c_longlong
    handle.kvq_splitzip_bf16_encode_top16.argtypes = [ctypes.c_ulonglong] * 6
    handle.kvq_splitzip_bf16_decode_top16_blocks.argtypes = [ctypes.c_ulonglong] * 12
    handle.kvq_splitzip_bf16_encode_mode.argtypes = [ctypes.c_ulonglong] * 5 + [ctypes.c_int]
    handle.kvq_splitzip_bf16_decode_fixed6_blocks.argtypes = [ctypes.c_ulonglong] * 11
    return handle


def test_cross_check_with_reference_kernels():
    ref = ref_lib()
    rng = np.random.Generator(np.random.PCG64(1234))
    pool, blocks, shape = 80, 48, (16, 8, 128)
    ids = rng.permutation(pool)[:blocks]
    tables = tables_for(7)
    cache = book_words(rng, (2, pool) + shape, splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[224:256], 0.0045)
    packed = np.ascontiguousarray(cache[:, ids])
    n = packed.size
    stream_ref = torch.zeros(2 * n, dtype=torch.uint8, device="cuda")
    src = words_dev(packed.reshape(-1))
    tab = dev(tables)
    s = torch.cuda.current_stream().cuda_stream
    r_ref = ref.kvq_splitzip_bf16_encode_top16(src.data_ptr(), stream_ref.data_ptr(), n, 2 * n, tab.data_ptr(), s)
    res, mine = gpu_encode_top16(packed.reshape(-1), tables)
    torch.cuda.synchronize()
    theirs = stream_ref.cpu().numpy()[:r_ref]
    assert r_ref == res
    count = int.from_bytes(theirs[1:5].tobytes(), "little")
    ent = 5 + n + (n + 1) // 2
    assert theirs[0] == mine[0] == 5
    assert np.array_equal(theirs[:ent], mine[:ent])  # header, body, codes identical
    set_ref = {bytes(theirs[ent + 5 * i : ent + 5 * i + 5]) for i in range(count)}
    set_mine = {bytes(mine[ent + 5 * i : ent + 5 * i + 5]) for i in range(count)}
    assert set_ref == set_mine  # escape entries equal as a set
    # my decoder on the reference stream; the reference decoder on mine
    _, got = gpu_decode_top16(theirs, cache.shape, ids, tables)
    assert np.array_equal(got[:, ids], packed)
    target = torch.zeros(cache.shape, dtype=torch.int16, device="cuda").view(torch.bfloat16)
    ids_t = dev(ids.astype(np.int64))
    bw = int(np.prod(shape))
    r = ref.kvq_splitzip_bf16_decode_top16_blocks(dev(mine).data_ptr(), mine.size, target.data_ptr(), n, blocks, bw,
                                                   target.stride(0), target.stride(1), 0, ids_t.data_ptr(), tab.data_ptr(), s)
    torch.cuda.synchronize()
    assert r == 2 * n
    assert np.array_equal(host_u16(target)[:, ids], packed)
    # fixed6: identical header layout and remapped codes; both decoders agree
    words6 = distinct_words(rng, n, 40)
    src6 = words_dev(words6)
    out_ref = torch.zeros(2 * n, dtype=torch.uint8, device="cuda")
    r6 = ref.kvq_splitzip_bf16_encode_mode(src6.data_ptr(), out_ref.data_ptr(), n, 2 * n, s, 6)
    out_mine = torch.zeros(2 * n, dtype=torch.uint8, device="cuda")
    m6 = lib().kvq_splitzip_bf16_encode_mode(src6.data_ptr(), out_mine.data_ptr(), n, 2 * n, s, 6)
    torch.cuda.synchronize()
    assert r6 == m6
    theirs6 = out_ref.cpu().numpy()[:r6]
    mine6 = out_mine.cpu().numpy()[:m6]
    assert theirs6[0] == mine6[0] == 3
    assert np.array_equal(theirs6[65 : 65 + n], mine6[65 : 65 + n])  # low plane
    assert sorted(theirs6[1:41]) == list(mine6[1:41])  # same palette, canonical order
    for stream in (theirs6, mine6):
        tgt = torch.zeros(cache.shape, dtype=torch.int16, device="cuda").view(torch.bfloat16)
        ref.kvq_splitzip_bf16_decode_fixed6_blocks(dev(stream).data_ptr(), stream.size, tgt.data_ptr(), n, blocks, bw,
                                                  tgt.stride(0), tgt.stride(1), 0, ids_t.data_ptr(), s)
        torch.cuda.synchronize()
        assert np.array_equal(host_u16(tgt)[:, ids].reshape(-1), words6)


def test_no_device_errors_recorded():
    assert splitzip_cuda.device_errors() == 0
