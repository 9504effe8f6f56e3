"""GPU decode of every form the reference's receiver takes
(vllm_connector.py:5098-5313) through ``decode_any_batch``: the torch-op
modes 0 (palette), 1 (nibble planes) and 2 (sign/magnitude), fixed5 (mode
4), and modes 5, 3 and 6, in one call.  The streams come from the reference's
own encoder (the committed golden fixtures) and from the CPU oracle, which is
pinned to it; the decoded caches must equal the words bit for bit, and a
stream that fails the receiver's checks must leave its blocks untouched."""

import zlib
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from unchainkv_b200 import splitzip_cuda as S  # noqa: E402

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

GOLDEN = Path(__file__).resolve().parent / "golden"
ARRAYS = np.load(GOLDEN / "golden.npz")
TABLE = np.frombuffer(S.build_top16_tables(S._DEFAULT_TOP16_CODEBOOKS[:32]), np.uint8)


def dev(a):
    return torch.from_numpy(np.array(a, copy=True, order="C")).cuda()


def decode_all(cases):
    """cases: (stream, target cache shape, ids) -> decoded caches (numpy)."""
    keep, jobs, outs = [], [], []
    tables = dev(TABLE)
    for stream, shape, ids in cases:
        out = torch.zeros(shape, dtype=torch.int16, device="cuda").view(torch.bfloat16)
        s, i = dev(stream), dev(np.asarray(ids, dtype=np.int64))
        keep += [s, i]
        outs.append(out)
        jobs.append(S.make_job(out, i, s, int(stream.size), tables))
    assert S.decode_any_batch(jobs) is not None
    torch.cuda.synchronize()
    return [o.view(torch.int16).cpu().numpy().view(np.uint16) for o in outs]


def test_reference_encoder_streams():
    names = ["mode2_narrow", "mode0_palette", "mode1_nibbles", "mode2_ragged"]
    cases = [(ARRAYS[f"{n}_stream"], ARRAYS[f"{n}_ref_cache"].shape, ARRAYS[f"{n}_ids"]) for n in names]
    for name, got in zip(names, decode_all(cases)):
        assert np.array_equal(got, ARRAYS[f"{name}_ref_cache"]), name


def words_for(kind, rng, shape):
    if kind.startswith("mode2"):
        width = int(kind[-1])
        lo = int(rng.integers(0, 128 - (1 << width)))
        high = (rng.integers(0, 2, shape) << 7) | rng.integers(lo, lo + (1 << width), shape)
        low = rng.integers(0, 256, shape)
    elif kind.startswith("mode0"):
        # magnitudes spanning 7 bits, so that mode 2 does not apply
        count = int(kind.split("_")[1])
        rest = np.array([h for h in range(256) if h not in (0x10, 0xF5)])
        highs = np.concatenate([[0x10, 0xF5], rng.choice(rest, size=count - 2, replace=False)])
        high, low = highs[rng.integers(0, count, shape)], rng.integers(0, 256, shape)
    else:  # nibble planes with 2 / 4 / 16 values
        high = rng.integers(0, 256, shape)
        low = (rng.integers(0, 256, shape) & 0x13) | 0x40
    return ((high << 8) | low).astype(np.uint16)


@pytest.mark.parametrize("kind", ["mode2_w1", "mode2_w3", "mode2_w6", "mode0_2", "mode0_9", "mode0_128", "mode1"])
def test_oracle_streams_of_every_width(kind):
    rng = np.random.Generator(np.random.PCG64(zlib.crc32(kind.encode())))
    pool, blocks = 120, 100  # big enough for mode 0's 258-byte header at width 7
    cases, expect = [], []
    for block_words in (1024, 96, 13):  # whole units, a ragged last unit, odd blocks
        cache = words_for(kind, rng, (2, pool, block_words))
        ids = rng.permutation(pool)[:blocks]
        result, stream = oracle.encode_torchop_blocks(cache, ids)
        assert result > 0
        expected_mode = {"mode2": 2, "mode0": 0, "mode1": 1}[kind[:5]]
        assert stream[0] == expected_mode, (kind, block_words, stream[0])
        target = np.zeros_like(cache)
        assert oracle.decode_modes_blocks(stream, target, ids) == 2 * 2 * blocks * block_words
        cases.append((stream, cache.shape, ids))
        expect.append(target)
    for got, want in zip(decode_all(cases), expect):
        assert np.array_equal(got, want)


def test_every_mode_in_one_batch():
    """One call with a stream of each form: 0, 1, 2 (reference encoder), 3
    and 4 (fixed6 / fixed5, oracle), 5 (top16, oracle) and 6 (raw)."""
    rng = np.random.Generator(np.random.PCG64(31))
    cases, want = [], []
    for name in ["mode0_palette", "mode1_nibbles", "mode2_narrow"]:
        cases.append((ARRAYS[f"{name}_stream"], ARRAYS[f"{name}_ref_cache"].shape, ARRAYS[f"{name}_ids"]))
        want.append(ARRAYS[f"{name}_ref_cache"])
    pool, bw = 30, 2048
    for bits in (6, 5):
        highs = np.sort(rng.choice(256, size=20, replace=False))
        cache = ((highs[rng.integers(0, 20, (2, pool, bw))] << 8) | rng.integers(0, 256, (2, pool, bw))).astype(np.uint16)
        ids = rng.permutation(pool)[:9]
        result, stream = oracle.encode_mode_blocks(cache, ids, bits=bits)
        target = np.zeros_like(cache)
        target[:, ids] = cache[:, ids]
        cases.append((stream[:result], cache.shape, ids))
        want.append(target)
    books = np.frombuffer(S._DEFAULT_TOP16_CODEBOOKS[:32], np.uint8).reshape(2, 16)
    n_shape = (2, pool, bw)
    plane = np.zeros(n_shape, dtype=np.int64)
    plane[1] = 1
    exp = books[plane, rng.integers(0, 16, n_shape)].astype(np.int64)
    cache = ((rng.integers(0, 2, n_shape) << 15) | (exp << 7) | rng.integers(0, 128, n_shape)).astype(np.uint16)
    ids = rng.permutation(pool)[:9]
    result, stream = oracle.encode_top16_blocks(cache, ids, TABLE)
    assert stream[0] == 5
    target = np.zeros_like(cache)
    target[:, ids] = cache[:, ids]
    cases.append((stream[:result], cache.shape, ids))
    want.append(target)
    raw = rng.integers(0, 1 << 16, (2, pool, 64), dtype=np.uint16)
    ids = rng.permutation(pool)[:5]
    stream = np.concatenate([[6], raw[:, ids].reshape(-1).view(np.uint8)]).astype(np.uint8)
    target = np.zeros_like(raw)
    target[:, ids] = raw[:, ids]
    cases.append((stream, raw.shape, ids))
    want.append(target)
    for got, expect in zip(decode_all(cases), want):
        assert np.array_equal(got, expect)


def test_malformed_streams_leave_blocks_untouched():
    stream = ARRAYS["mode0_palette_stream"]
    shape, ids = ARRAYS["mode0_palette_ref_cache"].shape, ARRAYS["mode0_palette_ids"]
    bad_width = stream.copy()
    bad_width[1] = 8
    bad_mode = stream.copy()
    bad_mode[0] = 7
    nibble = ARRAYS["mode1_nibbles_stream"].copy()
    nibble[2] = 3  # a nibble-plane width other than 1, 2, 4
    cases = [(stream[:-1], shape, ids), (bad_width, shape, ids), (bad_mode, shape, ids),
             (nibble, ARRAYS["mode1_nibbles_ref_cache"].shape, ARRAYS["mode1_nibbles_ids"])]
    for got in decode_all(cases):
        assert not got.any()


def gpu_torchop(cache, ids):
    """GPU torch-op encode of `ids` of `cache`; (stream bytes, length)."""
    kv = dev(cache.view(np.int16)).view(torch.bfloat16)
    ids_t = dev(np.asarray(ids, dtype=np.int64))
    n = 2 * len(ids) * int(np.prod(cache.shape[2:]))
    buf = torch.zeros(S.torchop_capacity(n), dtype=torch.uint8, device="cuda")
    assert S.encode_torchop_batch([S.make_job(kv, ids_t, buf)]) == 1 + 2 * n
    torch.cuda.synchronize()
    out = buf.cpu().numpy()
    length = S.stream_length(bytes(out[:8]), n)
    return out[:length], length


@pytest.mark.parametrize("name", ["mode2_narrow", "mode0_palette", "mode1_nibbles", "mode2_ragged"])
def test_gpu_torchop_encoder_reproduces_reference_streams(name):
    stream, length = gpu_torchop(ARRAYS[f"{name}_cache"], ARRAYS[f"{name}_src_ids"])
    assert length == ARRAYS[f"{name}_stream"].size
    assert np.array_equal(stream, ARRAYS[f"{name}_stream"])


@pytest.mark.parametrize("kind", ["mode2_w1", "mode2_w3", "mode2_w6", "mode0_2", "mode0_9", "mode0_128", "mode1"])
def test_gpu_torchop_encoder_matches_oracle_and_round_trips(kind):
    rng = np.random.Generator(np.random.PCG64(zlib.crc32(kind.encode()) + 1))
    for block_words in (1024, 96, 13):
        cache = words_for(kind, rng, (2, 120, block_words))
        ids = rng.permutation(120)[:100]
        stream, length = gpu_torchop(cache, ids)
        result, expected = oracle.encode_torchop_blocks(cache, ids)
        assert length == result and np.array_equal(stream, expected), (kind, block_words)
        (got,) = decode_all([(stream, cache.shape, ids)])
        assert np.array_equal(got[:, ids], cache[:, ids])


def test_gpu_torchop_batch_of_ragged_jobs_matches_oracle():
    """Jobs of every form and of sizes that are not whole warps of 16-word
    units (each job's units are padded to whole warps inside the kernel) in
    one batch: every stream equals the oracle's, and no byte between the
    streams changes."""
    rng = np.random.Generator(np.random.PCG64(77))
    specs = [("mode2_w3", 13, 37), ("mode0_9", 96, 5), ("mode1", 7, 61), ("mode0_128", 1024, 3),
             ("mode2_w6", 21, 29), ("raw", 40, 7)]
    jobs, keep, cases, offs = [], [], [], []
    total = 0
    for kind, bw, blocks in specs:
        pool = blocks + 3
        if kind == "raw":
            cache = rng.integers(0, 1 << 16, size=(2, pool, bw), dtype=np.uint16)
        else:
            cache = words_for(kind, rng, (2, pool, bw))
        ids = rng.permutation(pool)[:blocks]
        n = 2 * blocks * bw
        cap = (S.torchop_capacity(n) + 15) // 16 * 16
        cases.append((cache, ids, n))
        offs.append((total, cap))
        total += cap + 64  # a gap after each buffer, checked below
    buf = torch.full((total,), 0xA5, dtype=torch.uint8, device="cuda")
    for (cache, ids, n), (o, cap) in zip(cases, offs):
        kv = dev(cache.view(np.int16)).view(torch.bfloat16)
        ids_t = dev(np.asarray(ids, dtype=np.int64))
        keep += [kv, ids_t]
        jobs.append(S.make_job(kv, ids_t, buf[o:o + cap]))
    assert S.encode_torchop_batch(jobs) == sum(1 + 2 * n for _, _, n in cases)
    torch.cuda.synchronize()
    host = buf.cpu().numpy()
    for (cache, ids, n), (o, cap) in zip(cases, offs):
        result, expected = oracle.encode_torchop_blocks(cache, ids)
        if result == 0:  # the reference sends it raw
            expected = np.concatenate([[6], cache[:, ids].reshape(-1).view(np.uint8)]).astype(np.uint8)
        assert np.array_equal(host[o:o + expected.size], expected)
        assert np.all(host[o + cap:o + cap + 64] == 0xA5)


def test_gpu_torchop_encoder_falls_back_to_raw():
    rng = np.random.Generator(np.random.PCG64(41))
    cache = rng.integers(0, 1 << 16, size=(2, 20, 512), dtype=np.uint16)
    ids = rng.permutation(20)[:11]
    assert oracle.encode_torchop_blocks(cache, ids)[0] == 0  # the reference sends it raw
    stream, length = gpu_torchop(cache, ids)
    assert stream[0] == 6 and length == 1 + 2 * 2 * 11 * 512
    assert np.array_equal(stream[1:].view(np.uint16), cache[:, ids].reshape(-1))
