"""The top16 encoder that allocates nothing, checked against the standard one.

kvq_splitzip_bf16_encode_top16_noalloc serves callers that cannot allocate
device memory or cannot leave spare bytes past the stream in their buffer:
serving engines that give nearly all of HBM to their KV pool, paths that must
not call cudaMalloc / cudaFree (they can synchronise the device), and runtimes
that size stream buffers exactly.  Its scratch is a static device array shared
by all calls, so the test makes two calls in a row (the second finds the first
call's leftovers in the array) and compares both, byte for byte, with
kvq_splitzip_bf16_encode_top16 through the C ABI.
This file is collected last on purpose and needs nothing from other tests.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

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
    cases = [(11, 3 * 8192 + 77, 1, 0.003), (12, 1 << 20, 2, 0.0045)]
    for seed, n, layer, rate in cases:
        words, tables = make_input(seed, n, layer, rate)
        src = torch.from_numpy(words.view(np.int16)).cuda()
        tab = torch.from_numpy(tables).cuda()
        encoded = top16_bytes(n)
        # the standard encoder keeps its scratch past the stream: a roomy buffer
        standard = torch.full((2 * n + 4096,), 0xEE, dtype=torch.uint8, device="cuda")
        # the no-alloc encoder needs only the reference's capacity rule
        tight = ((encoded + 3) & ~3) + 8
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
        assert int(got[0]) == 5
        # nothing past the stream was touched
        assert (got[encoded:] == 0x77).all()
        # the standard encoder declines that tight buffer (it has no room
        # for its scratch); the no-alloc one is what such callers use
        assert lib.kvq_splitzip_bf16_encode_top16(src.data_ptr(), noalloc.data_ptr(), n, noalloc.numel(),
                                                  tab.data_ptr(), stream) == 0


def test_noalloc_encode_rejects_counts_beyond_its_static_maximum():
    lib = splitzip_cuda._load()
    assert lib is not None, splitzip_cuda.load_error()
    # rejected on the host before any device access, with a clear message
    result = lib.kvq_splitzip_bf16_encode_top16_noalloc(16, 16, MAX_WORDS + 2, 1 << 40, 16, 0)
    assert result == -1
    message = lib.kvq_splitzip_last_error().decode()
    assert "exceeds the static scratch maximum" in message and str(MAX_WORDS) in message
