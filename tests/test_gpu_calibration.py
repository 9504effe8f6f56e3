"""GPU calibration: exponent histograms gathered from the paged cache, and
top16 tables ranked on the device, against numpy restatements of the
reference's trace (vllm_connector.py:2871-2904: torch.bincount of
(w >> 7) & 0xFF per plane of the packed layer) and of its codebook ranking
(trace.py:30-33, scripts/extract_llama_top16_codebooks.py:39-40, table
layout splitzip_cuda.py:283-298).  Counts and tables must match exactly."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from unchainkv_b200 import splitzip_cuda as S  # noqa: E402

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]


def dev(a):
    return torch.from_numpy(np.array(a, copy=True, order="C")).cuda()


def packed(cache, ids):
    """The layer's words in the reference's packed order [2, blocks, ...]."""
    return cache[:, ids].reshape(2, -1)


def np_histogram(words2):
    """[2, 256] counts of (w >> 7) & 0xFF per plane (the reference's bincount)."""
    return np.stack([np.bincount((p.astype(np.int64) >> 7) & 0xFF, minlength=256) for p in words2])


def gpu_histograms(cases, repeat=1):
    hists = torch.zeros((len(cases), 2, 256), dtype=torch.int32, device="cuda")
    jobs, keep = [], []
    for i, (cache, ids) in enumerate(cases):
        kv = dev(cache.view(np.int16)).view(torch.bfloat16)
        ids_t = dev(ids)
        keep += [kv, ids_t]  # alive until the launches are done
        jobs.append(S.histogram_job(kv, ids_t, hists[i]))
    for _ in range(repeat):
        assert S.exponent_histogram_batch(jobs) == len(cases)
    torch.cuda.synchronize()
    return hists.cpu().numpy().astype(np.int64)


def test_histograms_of_paged_layers_match_bincount():
    rng = np.random.Generator(np.random.PCG64(21))
    cases = []
    # whole tiles, a ragged last tile, blocks that are not a power of two,
    # a tile that spans the K/V plane boundary, a single tiny block
    for pool, shape, blocks in [(80, (16, 8, 128), 40), (50, (16, 1, 128), 33), (30, (7, 3), 29),
                                (12, (16, 8, 64), 5), (4, (2, 2), 1)]:
        cache = rng.integers(0, 1 << 16, size=(2, pool) + shape, dtype=np.uint16)
        ids = rng.permutation(pool)[:blocks].astype(np.int64)
        cases.append((cache, ids))
    got = gpu_histograms(cases)
    for i, (cache, ids) in enumerate(cases):
        assert np.array_equal(got[i], np_histogram(packed(cache, ids))), i


def test_histograms_accumulate_over_calls():
    rng = np.random.Generator(np.random.PCG64(22))
    cache = rng.integers(0, 1 << 16, size=(2, 20, 16, 8, 128), dtype=np.uint16)
    ids = rng.permutation(20)[:9].astype(np.int64)
    got = gpu_histograms([(cache, ids)], repeat=3)
    assert np.array_equal(got[0], 3 * np_histogram(packed(cache, ids)))


def reference_tables(hist):
    """The layer table from the reference's ranking (>= 16 observed)."""
    books = bytes(S.rank_top16(hist[0]) + S.rank_top16(hist[1]))
    return np.frombuffer(S.build_top16_tables(books), np.uint8)


def test_device_tables_match_the_ranking_rule():
    rng = np.random.Generator(np.random.PCG64(23))
    hists = np.zeros((6, 2, 256), dtype=np.int32)
    for layer in range(6):
        for plane in range(2):
            bins = rng.choice(256, size=int(rng.integers(16, 120)), replace=False)
            hists[layer, plane, bins] = rng.integers(1, 1 << 20, size=bins.size)
            hists[layer, plane, bins[:8]] = 12345  # ties broken by exponent
    tables, observed = S.top16_tables_from_histograms(dev(hists))
    torch.cuda.synchronize()
    tables = tables.cpu().numpy()
    observed = observed.cpu().numpy()
    for layer in range(6):
        assert np.array_equal(tables[layer], reference_tables(hists[layer])), layer
        assert list(observed[layer]) == [int((hists[layer, p] > 0).sum()) for p in range(2)]
    codebooks = S.codebooks_from_tables(torch.from_numpy(tables), torch.from_numpy(observed))
    assert len(codebooks) == 6 * 32


def test_fewer_than_16_observed_exponents():
    hist = np.zeros((1, 2, 256), dtype=np.int32)
    hist[0, 0, [130, 120, 125]] = [5, 9, 5]  # K: 3 observed
    hist[0, 1, np.arange(100, 140)] = 1      # V: 40 observed, all tied
    tables, observed = S.top16_tables_from_histograms(dev(hist))
    torch.cuda.synchronize()
    t = tables.cpu().numpy()[0]
    assert list(observed.cpu().numpy()[0]) == [3, 40]
    # K: the 3 observed by (-count, exponent), then unobserved 0, 1, 2, ...
    assert list(t[512:528]) == [120, 125, 130] + list(range(13))
    assert list(t[528:544]) == list(range(100, 116))
    assert t[120] == 0 and t[125] == 1 and t[130] == 2 and t[0] == 3 and t[200] == 255
    with pytest.raises(ValueError):
        S.codebooks_from_tables(tables, observed)


def test_calibrated_tables_drive_a_lossless_top16_round_trip():
    """histogram -> device tables -> top16 encode of the same blocks: the
    stream equals the CPU oracle's with the same table, and decoding it
    restores every word.  The words use 16 common exponents per plane and 4
    rare ones (0.3% of words, under the 0.5% escape capacity)."""
    rng = np.random.Generator(np.random.PCG64(24))
    pool, blocks = 256, 64
    shape = (2, pool, 16, 8, 128)
    size = int(np.prod(shape))
    common = np.stack([rng.choice(np.arange(100, 140), 16, replace=False) for _ in range(2)])
    rare = np.array([[60, 61, 200, 201], [70, 71, 210, 211]])
    weights = rng.random(16) + 0.2
    plane = np.repeat([0, 1], size // 2)
    exp = common[plane, rng.choice(16, size, p=weights / weights.sum())]
    mask = rng.random(size) < 0.003
    exp[mask] = rare[plane[mask], rng.integers(0, 4, int(mask.sum()))]
    words = (rng.integers(0, 2, size) << 15) | (exp << 7) | rng.integers(0, 128, size)
    cache = words.astype(np.uint16).reshape(shape)
    ids = rng.permutation(pool)[:blocks].astype(np.int64)
    hist = gpu_histograms([(cache, ids)])
    tables, observed = S.top16_tables_from_histograms(dev(hist.astype(np.int32)))
    table = tables[0].contiguous()
    table_np = table.cpu().numpy()
    assert np.array_equal(table_np, reference_tables(hist[0]))
    kv = dev(cache.view(np.int16)).view(torch.bfloat16)
    ids_t = dev(ids)
    n = 2 * blocks * 16 * 8 * 128
    buf = torch.zeros(S.auto_capacity(n), dtype=torch.uint8, device="cuda")
    got = S.encode_top16_batch([S.make_job(kv, ids_t, buf, None, table)])
    result, expected = oracle.encode_top16_blocks(cache, ids, table_np)
    assert got == result
    torch.cuda.synchronize()
    assert np.array_equal(buf[:result].cpu().numpy(), expected[:result])
    out = torch.zeros_like(kv)
    assert S.decode_top16_batch([S.make_job(out, ids_t, buf, result, table)])
    torch.cuda.synchronize()
    back = out.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(back[:, ids], cache[:, ids])
