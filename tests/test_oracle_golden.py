"""Pin the CPU oracle to the reference's own CPU code (golden vectors made by
tests/golden/make_golden.py from the reference source tree)."""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "golden.json").read_text())
ARRAYS = np.load(GOLDEN / "golden.npz")
TABLES = np.frombuffer((GOLDEN / "top16_tables.bin").read_bytes(), dtype=np.uint8).reshape(-1, 544)


@pytest.mark.parametrize("case", META["top16_cases"], ids=lambda c: c["name"])
def test_top16_oracle_stream_and_reference_decoder(case):
    name, n, layer = case["name"], case["n"], case["layer"]
    words = ARRAYS[f"top16_{name}_words"]
    expected_stream = ARRAYS[f"top16_{name}_stream"]
    result, stream = oracle.encode_top16(words, TABLES[layer])
    assert result == oracle.top16_encoded_bytes(n)
    assert np.array_equal(stream, expected_stream)
    assert stream[0] == case["mode"]
    ref_decoded = ARRAYS[f"top16_{name}_ref_decoded"]
    # the oracle decoder agrees with the reference's pure-Python decoder
    blocks = 2
    cache = np.zeros((2, blocks, n // 4), dtype=np.uint16)
    copied = oracle.decode_top16_blocks(stream, cache, [0, 1], TABLES[layer])
    assert copied == 2 * n
    if case["ref_decodes"]:
        assert np.array_equal(cache.reshape(-1), ref_decoded)
        assert np.array_equal(ref_decoded, words)  # lossless
    else:
        # overflow stream: the decoder writes nothing, as the reference's does
        assert not cache.any()


def test_top16_reference_known_answer_payload():
    payload = ARRAYS["kat_payload"]
    words = ARRAYS["kat_words"]
    cache = np.zeros((2, 16, 8), dtype=np.uint16)
    copied = oracle.decode_top16_blocks(payload, cache, list(range(16)), TABLES[0])
    assert copied == 512
    assert np.array_equal(cache.reshape(-1), words)
    # and the oracle encoder reproduces the payload byte for byte
    result, stream = oracle.encode_top16(words, TABLES[0])
    assert result == payload.size
    assert np.array_equal(stream, payload)


@pytest.mark.parametrize("case", META["fixed_cases"], ids=lambda c: c["name"])
def test_fixed_oracle_against_reference_torch_receiver(case):
    name, bits = case["name"], case["bits"]
    words = ARRAYS[f"{name}_words"]
    result, stream = oracle.encode_mode(words, bits=bits)
    assert np.array_equal(stream, ARRAYS[f"{name}_stream"])
    ids = ARRAYS[f"{name}_ids"]
    ref_cache = ARRAYS[f"{name}_ref_cache"]
    # the reference receiver placed the words at the block ids
    packed = ref_cache[:, ids].reshape(-1)
    assert np.array_equal(packed, words)
    if bits == 6:
        cache = np.zeros_like(ref_cache)
        assert oracle.decode_fixed6_blocks(stream, cache, ids) == 2 * words.size
        assert np.array_equal(cache, ref_cache)


def test_top16_tables_match_reference_builder():
    from unchainkv_b200 import splitzip_cuda

    codebooks = (GOLDEN / "top16_codebooks.bin").read_bytes()
    assert splitzip_cuda._TOP16_CODEBOOKS == codebooks
    for layer in range(META["layers"]):
        built = splitzip_cuda.build_top16_tables(codebooks[layer * 32 : (layer + 1) * 32])
        assert built == TABLES[layer].tobytes()


def test_palette_ranking_rule_matches_reference():
    from unchainkv_b200 import splitzip_cuda

    for row in META["rankings"]:
        assert splitzip_cuda.rank_top16(row["histogram"]) == row["top16"]


def test_oracle_gather_equals_index_select_then_encode():
    rng = np.random.Generator(np.random.PCG64(11))
    cache = rng.integers(0, 1 << 16, size=(2, 20, 4, 64), dtype=np.uint16)
    ids = rng.permutation(20)[:7]
    packed = cache[:, ids].reshape(-1)
    result_a, stream_a = oracle.encode_top16(packed, TABLES[3])
    result_b, stream_b = oracle.encode_top16_blocks(cache, ids, TABLES[3])
    assert result_a == result_b > 0
    assert np.array_equal(stream_a, stream_b)
    result_c, stream_c = oracle.encode_mode(packed, bits=6)
    result_d, stream_d = oracle.encode_mode_blocks(cache, ids, bits=6)
    assert result_c == result_d > 0 and np.array_equal(stream_c, stream_d)


def test_oracle_decline_rules_follow_reference():
    words = np.zeros(2, dtype=np.uint16)
    # tiny inputs do not compress (.cu:393, 306)
    assert oracle.encode_top16(words, TABLES[0])[0] == 0
    assert oracle.encode_mode(words)[0] == 0
    n = 4096
    words = np.zeros(n, dtype=np.uint16)
    enc = oracle.top16_encoded_bytes(n)
    need = ((enc + 3) & ~3) + 8
    assert oracle.encode_top16(words, TABLES[0], capacity=need)[0] == enc
    assert oracle.encode_top16(words, TABLES[0], capacity=need - 1)[0] == 0
    fenc = oracle.fixed_encoded_bytes(n)
    fneed = ((fenc + 3) & ~3) + 1032
    assert oracle.encode_mode(words, capacity=fneed)[0] == fenc
    assert oracle.encode_mode(words, capacity=fneed - 1)[0] == 0


def test_multithreaded_oracle_matches_single_thread():
    rng = np.random.Generator(np.random.PCG64(5))
    cache = rng.integers(0, 1 << 16, size=(2, 40, 16, 64), dtype=np.uint16)
    # make exponents mostly in-book so the stream is not all escapes
    book = np.frombuffer(TABLES[2][512:544].tobytes(), dtype=np.uint8)
    exp = book[rng.integers(0, 16, size=cache.shape)].astype(np.uint16)
    rare = rng.random(cache.shape) < 0.004
    exp[rare] = 3
    cache = (cache & 0x807F) | (exp << 7)
    ids = np.ascontiguousarray(rng.permutation(40)[:25], dtype=np.int64)
    single = oracle.encode_top16_blocks(cache, ids, TABLES[2])[1]
    lib = oracle.lib()
    n = 2 * 25 * 1024
    out = np.zeros(2 * n, dtype=np.uint8)
    tables = np.ascontiguousarray(TABLES[2])
    res = lib.orc_encode_top16_blocks_mt(cache.ctypes.data, 40 * 1024, 1024, 1024, ids.ctypes.data,
                                         0, 25, out.ctypes.data, out.size, tables.ctypes.data, 4)
    assert res == single.size
    assert np.array_equal(out[:res], single)


def test_exponent_summary_matches_reference():
    """The calibration trace summary (trace.py:27-58 of the reference)."""
    from unchainkv_b200 import splitzip_cuda

    for row in META["rankings"]:
        assert splitzip_cuda.summarize_symbol_counts(row["histogram"]) == row["summary"]


@pytest.mark.parametrize("case", META["torchop_cases"], ids=lambda c: c["name"])
def test_torchop_modes_match_reference_encoder_and_receiver(case):
    """Modes 2 / 0 / 1: the reference's own torch-op encoder produced the
    stream; the oracle encoder reproduces it byte for byte, and the oracle
    receiver decodes it to the cache the reference receiver wrote."""
    name = case["name"]
    cache = ARRAYS[f"{name}_cache"]
    stream = ARRAYS[f"{name}_stream"]
    result, ours = oracle.encode_torchop_blocks(cache, ARRAYS[f"{name}_src_ids"])
    assert result == stream.size and stream[0] == case["mode"]
    assert np.array_equal(ours, stream)
    ref_cache = ARRAYS[f"{name}_ref_cache"]
    target = np.zeros_like(ref_cache)
    n = 2 * case["blocks"] * int(np.prod(ref_cache.shape[2:]))
    assert oracle.decode_modes_blocks(stream, target, ARRAYS[f"{name}_ids"]) == 2 * n
    assert np.array_equal(target, ref_cache)


def test_fixed5_receiver_matches_reference():
    case = next(c for c in META["fixed_cases"] if c["bits"] == 5)
    name = case["name"]
    ref_cache = ARRAYS[f"{name}_ref_cache"]
    target = np.zeros_like(ref_cache)
    n = 2 * case["blocks"] * case["block_words"]
    assert oracle.decode_modes_blocks(ARRAYS[f"{name}_stream"], target, ARRAYS[f"{name}_ids"]) == 2 * n
    assert np.array_equal(target, ref_cache)


def test_receiver_declines_malformed_mode_streams():
    name = "mode0_palette"
    stream = ARRAYS[f"{name}_stream"].copy()
    target = np.zeros_like(ARRAYS[f"{name}_ref_cache"])
    ids = ARRAYS[f"{name}_ids"]
    assert oracle.decode_modes_blocks(stream[:-1], target, ids) == 0  # short
    bad = stream.copy()
    bad[1] = 8  # width out of range
    assert oracle.decode_modes_blocks(bad, target, ids) == 0
    bad[0] = 7  # no such mode
    assert oracle.decode_modes_blocks(bad, target, ids) == 0
    assert not target.any()
