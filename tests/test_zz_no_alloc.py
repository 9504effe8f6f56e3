"""The top16 encoder that allocates nothing, checked against the standard one.

Some callers cannot allocate device memory while they encode: a serving
engine that gives nearly all of HBM to its paged KV pool (a transient
allocation can fail there), or a path that must not call cudaMalloc /
cudaFree because those can synchronise the device.
kvq_splitzip_bf16_encode_top16_noalloc keeps the escape counts of its
statistics pass in a static device array of the library and writes no byte
past the stream.  The array is shared by all calls, so the test makes several
calls in a row (each finds the previous call's leftovers in the array): in
capacity, then over capacity (a mode-255 stream), then in capacity again.
Each stream is compared byte for byte with kvq_splitzip_bf16_encode_top16
through the C ABI and with the CPU oracle.
This file is collected last on purpose and needs nothing from other tests.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from unchainkv_b200 import splitzip_cuda  # noqa: E402

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

MAX_WORDS = 1 << 27


def make_input(seed, n, layer, escape_rate):
    rng = np.random.Generator(np.random.PCG64(seed))
    books = splitzip_cuda._DEFAULT_TOP16_CODEBOOKS[layer * 32 : layer * 32 + 32]
    book = np.frombuffer(books, dtype=np.uint8).reshape(2, 16)
    plane = (np.arange(n) >= n // 2).astype(np.int64)
    exp = book[plane, rng.integers(0, 16, size=n)].astype(np.int64)
    outside = np.array([v for v in range(256) if v not in set(books)])
    mask = rng.random(n) < escape_rate
    exp[mask] = rng.choice(outside, size=int(mask.sum()))
    words = (rng.integers(0, 2, size=n) << 15) | (exp << 7) | rng.integers(0, 128, size=n)
    tables = np.frombuffer(splitzip_cuda.build_top16_tables(books), dtype=np.uint8).copy()
    return words.astype(np.uint16), tables


def top16_bytes(n):
    return 5 + n + (n + 1) // 2 + 5 * ((n + 199) // 200)


def test_noalloc_encode_matches_standard_entry_point_on_two_calls():
    lib = splitzip_cuda._load()
    assert lib is not None, splitzip_cuda.load_error()
    stream = torch.cuda.current_stream().cuda_stream
    # in capacity, over capacity (2% escapes against 0.5%), in capacity again
    cases = [(11, 3 * 8192 + 77, 1, 0.003), (13, (1 << 20) + 96, 3, 0.02), (12, 1 << 20, 2, 0.0045)]
    for seed, n, layer, rate in cases:
        words, tables = make_input(seed, n, layer, rate)
        src = torch.from_numpy(words.view(np.int16)).cuda()
        tab = torch.from_numpy(tables).cuda()
        encoded = top16_bytes(n)
        # both encoders take a buffer sized by the reference's rule
        tight = ((encoded + 3) & ~3) + 8
        standard = torch.full((tight,), 0xEE, dtype=torch.uint8, device="cuda")
        noalloc = torch.full((tight,), 0x77, dtype=torch.uint8, device="cuda")
        r_std = lib.kvq_splitzip_bf16_encode_top16(src.data_ptr(), standard.data_ptr(), n, standard.numel(),
                                                   tab.data_ptr(), stream)
        r_na = lib.kvq_splitzip_bf16_encode_top16_noalloc(src.data_ptr(), noalloc.data_ptr(), n, noalloc.numel(),
                                                          tab.data_ptr(), stream)
        torch.cuda.synchronize()
        assert r_std == encoded, splitzip_cuda._load().kvq_splitzip_last_error()
        assert r_na == encoded, splitzip_cuda._load().kvq_splitzip_last_error()
        got = noalloc.cpu().numpy()
        assert np.array_equal(got[:encoded], standard.cpu().numpy()[:encoded])
        # the CPU oracle's canonical stream, overflow form included
        res, expected = oracle.encode_top16(words, tables, capacity=tight)
        assert res == encoded and np.array_equal(got[:encoded], expected)
        assert int(got[0]) == (255 if rate > 0.005 else 5)
        # nothing past the stream was touched
        assert (got[encoded:] == 0x77).all()


def test_noalloc_encode_rejects_counts_beyond_its_static_maximum():
    lib = splitzip_cuda._load()
    assert lib is not None, splitzip_cuda.load_error()
    # rejected on the host before any device access, with a clear message
    result = lib.kvq_splitzip_bf16_encode_top16_noalloc(16, 16, MAX_WORDS + 2, 1 << 40, 16, 0)
    assert result == -1
    message = lib.kvq_splitzip_last_error().decode()
    assert "exceeds the static scratch maximum" in message and str(MAX_WORDS) in message
