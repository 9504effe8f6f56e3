"""GPU parity of the batched and device-chosen (auto) codec paths against the
CPU oracle: every job of a batch must produce exactly the stream its single
reference-style call would, and the auto path must end with the stream the
reference's fallback chain (top16 -> fixed6 -> raw mode 6) ends with."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from unchainkv_b200 import splitzip_cuda as S  # noqa: E402

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]


def tables_np(layer):
    return np.frombuffer(S.build_top16_tables(S._DEFAULT_TOP16_CODEBOOKS[layer * 32: layer * 32 + 32]), np.uint8)


def dev(a):
    return torch.from_numpy(np.array(a, copy=True, order="C")).cuda()


def to_u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def book_cache(rng, pool, shape, layer, rate, escape_choices=None):
    books = S._DEFAULT_TOP16_CODEBOOKS[layer * 32: layer * 32 + 32]
    n = 2 * pool * int(np.prod(shape))
    book = np.frombuffer(books, np.uint8).reshape(2, 16)
    plane = (np.arange(n) >= n // 2).astype(np.int64)
    exp = book[plane, rng.integers(0, 16, n)].astype(np.int64)
    outside = np.array([v for v in range(256) if v not in set(books)])
    if escape_choices:
        outside = outside[:escape_choices]
    mask = rng.random(n) < rate
    exp[mask] = rng.choice(outside, int(mask.sum()))
    words = (rng.integers(0, 2, n) << 15) | (exp << 7) | rng.integers(0, 128, n)
    return words.astype(np.uint16).reshape((2, pool) + shape)


def make_case(rng, pool, shape, layer, rate, blocks=None, escape_choices=None):
    cache = book_cache(rng, pool, shape, layer, rate, escape_choices)
    blocks = blocks or pool // 2
    ids = rng.permutation(pool)[:blocks].astype(np.int64)
    return cache, ids, tables_np(layer)


def job_for(kv, ids_t, buf, tables_t, stream_bytes=None):
    return S.make_job(kv, ids_t, buf, stream_bytes, tables_t)


def test_top16_and_fixed6_batches_match_single_calls():
    rng = np.random.Generator(np.random.PCG64(1))
    # blocks of 400 and 512 words: a tile meets more than 32 blocks, so the
    # producer issues its copies in several rounds of 32 runs
    specs = [(40, (16, 8, 128), 0, 0.003), (300, (16, 1, 128), 5, 0.0045), (30, (7, 3), 9, 0.002),
             (64, (16, 8, 128), 31, 0.0), (160, (4, 1, 100), 11, 0.003), (120, (16, 2, 16), 13, 0.004)]
    cases, jobs, bufs, keep = [], [], [], []
    for pool, shape, layer, rate in specs:
        cache, ids, tab = make_case(rng, pool, shape, layer, rate)
        kv = dev(cache.view(np.int16)).view(torch.bfloat16)
        ids_t, tab_t = dev(ids), dev(tab)
        n = 2 * len(ids) * int(np.prod(shape))
        buf = torch.zeros(2 * n + 4096, dtype=torch.uint8, device="cuda")
        jobs.append(job_for(kv, ids_t, buf, tab_t))
        cases.append((cache, ids, tab, n))
        bufs.append(buf)
        keep += [kv, ids_t, tab_t]
    total = S.encode_top16_batch(jobs)
    torch.cuda.synchronize()
    expect = 0
    for (cache, ids, tab, n), buf in zip(cases, bufs):
        res, stream = oracle.encode_top16_blocks(cache, ids, tab)
        expect += res
        assert np.array_equal(buf.cpu().numpy()[:res], stream)
    assert total == expect
    # decode the batch into fresh caches with other block tables
    targets, djobs = [], []
    for (cache, ids, tab, n), buf in zip(cases, bufs):
        ids2 = rng.permutation(cache.shape[1])[: len(ids)].astype(np.int64)
        tgt = torch.zeros(cache.shape, dtype=torch.int16, device="cuda").view(torch.bfloat16)
        ids2_t, tab_t = dev(ids2), dev(tab)
        djobs.append(job_for(tgt, ids2_t, buf, tab_t, S.top16_stream_bytes(n)))
        targets.append((tgt, ids2, cache, ids))
        keep += [ids2_t, tab_t]
    assert S.decode_top16_batch(djobs) == sum(2 * c[3] for c in cases)
    torch.cuda.synchronize()
    for tgt, ids2, cache, ids in targets:
        assert np.array_equal(to_u16(tgt)[:, ids2], cache[:, ids])

    # fixed6 batch
    for buf in bufs:
        buf.zero_()
    total6 = S.encode_bf16_batch(jobs, bits=6)
    torch.cuda.synchronize()
    expect6 = 0
    fixed_ok = []
    for (cache, ids, tab, n), buf in zip(cases, bufs):
        res, stream = oracle.encode_mode_blocks(cache, ids, bits=6)
        expect6 += res
        got = buf.cpu().numpy()
        if stream[0] == 3:
            assert np.array_equal(got[:res], stream)
        else:  # more than 64 high bytes: mode 255 + canonical palette
            assert got[0] == 255 and np.array_equal(got[:65], stream[:65])
        fixed_ok.append(stream[0] == 3)
    assert total6 == expect6
    assert any(fixed_ok)
    keep_jobs = [j for j, ok in zip(djobs, fixed_ok) if ok]
    keep_targets = [t for t, ok in zip(targets, fixed_ok) if ok]
    keep_cases = [c for c, ok in zip(cases, fixed_ok) if ok]
    for j, (cache, ids, tab, n) in zip(keep_jobs, keep_cases):
        j.stream_bytes = S.fixed6_stream_bytes(n)
    for tgt, *_ in keep_targets:
        tgt.zero_()
    assert S.decode_fixed6_batch(keep_jobs) == sum(2 * c[3] for c in keep_cases)
    torch.cuda.synchronize()
    for tgt, ids2, cache, ids in keep_targets:
        assert np.array_equal(to_u16(tgt)[:, ids2], cache[:, ids])


def test_auto_picks_the_reference_chain_result():
    rng = np.random.Generator(np.random.PCG64(2))
    shape = (16, 8, 128)
    kinds = []
    # (a) escapes within capacity -> top16
    kinds.append(("top16",) + make_case(rng, 48, shape, 3, 0.003))
    # (b) escapes over capacity, <= 64 high bytes -> fixed6
    kinds.append(("fixed6",) + make_case(rng, 48, shape, 4, 0.02, escape_choices=3))
    # (c) > 64 distinct high bytes with room for raw -> raw mode 6
    raw_cache = rng.integers(0, 1 << 16, size=(2, 48) + shape, dtype=np.uint16)
    ids = rng.permutation(48)[:24].astype(np.int64)
    kinds.append(("raw", raw_cache, ids, tables_np(0)))
    # (d) same without room for raw -> mode 255
    kinds.append(("overflow", raw_cache, ids, tables_np(0)))
    jobs, bufs, keep = [], [], []
    for kind, cache, ids, tab in kinds:
        kv = dev(cache.view(np.int16)).view(torch.bfloat16)
        ids_t, tab_t = dev(ids), dev(tab)
        n = 2 * len(ids) * int(np.prod(shape))
        cap = S.auto_capacity(n, raw=(kind != "overflow"))
        buf = torch.zeros(cap, dtype=torch.uint8, device="cuda")
        jobs.append(job_for(kv, ids_t, buf, tab_t))
        bufs.append(buf)
        keep += [kv, ids_t, tab_t]
    assert S.encode_auto_batch(jobs)
    torch.cuda.synchronize()
    for (kind, cache, ids, tab), buf in zip(kinds, bufs):
        got = buf.cpu().numpy()
        n = 2 * len(ids) * int(np.prod(shape))
        if kind == "top16":
            res, stream = oracle.encode_top16_blocks(cache, ids, tab)
            assert stream[0] == 5 and np.array_equal(got[:res], stream)
        elif kind == "fixed6":
            assert oracle.encode_top16_blocks(cache, ids, tab)[1][0] == 255
            res, stream = oracle.encode_mode_blocks(cache, ids, bits=6)
            assert stream[0] == 3 and np.array_equal(got[:res], stream)
        elif kind == "raw":
            assert got[0] == 6
            assert np.array_equal(got[1 : 1 + 2 * n].view(np.uint16), cache[:, ids].reshape(-1))
        else:
            res, stream = oracle.encode_mode_blocks(cache, ids, bits=6)
            assert stream[0] == 255 and got[0] == 255
            assert np.array_equal(got[1:65], stream[1:65])
    # decode all four by mode byte; the overflow stream leaves its blocks alone
    targets, djobs = [], []
    for (kind, cache, ids, tab), buf in zip(kinds, bufs):
        ids2 = rng.permutation(48)[: len(ids)].astype(np.int64)
        tgt = torch.full(cache.shape, 7, dtype=torch.int16, device="cuda").view(torch.bfloat16)
        ids2_t, tab_t = dev(ids2), dev(tab)
        djobs.append(job_for(tgt, ids2_t, buf, tab_t))
        targets.append((kind, tgt, ids2, cache, ids))
        keep += [ids2_t, tab_t]
    assert S.decode_auto_batch(djobs)
    torch.cuda.synchronize()
    for kind, tgt, ids2, cache, ids in targets:
        got = to_u16(tgt)
        if kind == "overflow":
            assert (got == 7).all()
        else:
            assert np.array_equal(got[:, ids2], cache[:, ids]), kind


def test_batch_larger_than_one_launch():
    rng = np.random.Generator(np.random.PCG64(3))
    pool, shape = 12, (16, 1, 128)
    jobs, bufs, cases, keep = [], [], [], []
    for i in range(100):
        cache, ids, tab = make_case(rng, pool, shape, i % 32, 0.004, blocks=6)
        kv = dev(cache.view(np.int16)).view(torch.bfloat16)
        ids_t, tab_t = dev(ids), dev(tab)
        n = 2 * 6 * 2048
        buf = torch.zeros(S.auto_capacity(n), dtype=torch.uint8, device="cuda")
        jobs.append(job_for(kv, ids_t, buf, tab_t))
        bufs.append(buf)
        cases.append((cache, ids, tab))
        keep += [kv, ids_t, tab_t]
    assert S.encode_top16_batch(jobs) == sum(S.top16_stream_bytes(2 * 6 * 2048) for _ in range(100))
    torch.cuda.synchronize()
    for (cache, ids, tab), buf in zip(cases, bufs):
        res, stream = oracle.encode_top16_blocks(cache, ids, tab)
        assert np.array_equal(buf.cpu().numpy()[:res], stream)


def test_batch_declines_as_a_whole():
    rng = np.random.Generator(np.random.PCG64(4))
    cache, ids, tab = make_case(rng, 16, (16, 8, 128), 0, 0.003)
    kv = dev(cache.view(np.int16)).view(torch.bfloat16)
    ids_t, tab_t = dev(ids), dev(tab)
    good = torch.full((1 << 20,), 0x5A, dtype=torch.uint8, device="cuda")
    small = torch.full((64,), 0x5A, dtype=torch.uint8, device="cuda")
    jobs = [job_for(kv, ids_t, good, tab_t), job_for(kv, ids_t, small, tab_t)]
    assert S.encode_top16_batch(jobs) is None
    torch.cuda.synchronize()
    assert int(good[0].item()) == 0x5A  # nothing launched


def test_profiler_counts_launches():
    rng = np.random.Generator(np.random.PCG64(5))
    cache, ids, tab = make_case(rng, 32, (16, 8, 128), 1, 0.02)
    kv = dev(cache.view(np.int16)).view(torch.bfloat16)
    ids_t, tab_t = dev(ids), dev(tab)
    n = 2 * len(ids) * 16 * 8 * 128
    bufs = [torch.zeros(S.auto_capacity(n), dtype=torch.uint8, device="cuda") for _ in range(2)]
    jobs = [job_for(kv, ids_t, buf, tab_t) for buf in bufs]
    S.profile_enable(True)
    try:
        for _ in range(3):
            S.encode_auto_batch(jobs)
            S.decode_auto_batch(jobs)
        prof = S.profile_collect()
    finally:
        S.profile_enable(False)
    assert prof["StatsKernel"][1] == 3
    assert prof["EncodeAutoKernel"][1] == 3
    assert prof["DecodeAutoKernel"][1] == 3
    assert prof["ZeroKernel"][1] == 3
    assert all(ms > 0 for ms, _ in prof.values())


def test_auto_round_trip_at_every_stream_alignment():
    """Full tiles coded into stream buffers that start at each byte offset
    0..15: the warp run stores take every funnel shift (and the aligned
    path), in all three modes, for encode and decode."""
    rng = np.random.Generator(np.random.PCG64(7))
    shape = (16, 8, 128)
    pool = 8
    sources = {
        "top16": make_case(rng, pool, shape, 6, 0.003),
        "fixed6": make_case(rng, pool, shape, 7, 0.02, escape_choices=3),
        "raw": (rng.integers(0, 1 << 16, size=(2, pool) + shape, dtype=np.uint16),
                rng.permutation(pool)[:4].astype(np.int64), tables_np(0)),
    }
    n = 2 * 4 * int(np.prod(shape))
    cap = S.auto_capacity(n)
    expected = {}
    for kind, (cache, ids, tab) in sources.items():
        if kind == "top16":
            expected[kind] = oracle.encode_top16_blocks(cache, ids, tab)[1]
        elif kind == "fixed6":
            expected[kind] = oracle.encode_mode_blocks(cache, ids, bits=6)[1]
        else:
            expected[kind] = np.concatenate([[6], cache[:, ids].reshape(-1).view(np.uint8)]).astype(np.uint8)
    big = torch.zeros(48 * (cap + 64), dtype=torch.uint8, device="cuda")
    jobs, views, keep, order = [], [], [], []
    for kind, (cache, ids, tab) in sources.items():
        kv = dev(cache.view(np.int16)).view(torch.bfloat16)
        ids_t, tab_t = dev(ids), dev(tab)
        keep += [kv, ids_t, tab_t]
        for off in range(16):
            start = len(views) * (cap + 64) + off
            view = big[start : start + cap]
            jobs.append(job_for(kv, ids_t, view, tab_t))
            views.append(view)
            order.append((kind, off))
    assert S.encode_auto_batch(jobs)
    torch.cuda.synchronize()
    for (kind, off), view in zip(order, views):
        want = expected[kind]
        got = view.cpu().numpy()[: want.size]
        assert np.array_equal(got, want), (kind, off, int(np.flatnonzero(got != want)[0]))
    targets, djobs = [], []
    for (kind, off), view in zip(order, views):
        cache, ids, tab = sources[kind]
        out = torch.full(cache.shape, 0x1357, dtype=torch.int16, device="cuda").view(torch.bfloat16)
        ids_t, tab_t = dev(ids), dev(tab)
        keep += [ids_t, tab_t]  # the jobs hold raw pointers
        targets.append((kind, off, out))
        djobs.append(job_for(out, ids_t, view, tab_t, stream_bytes=expected[kind].size))
    assert S.decode_auto_batch(djobs)
    torch.cuda.synchronize()
    for kind, off, out in targets:
        cache, ids, _ = sources[kind]
        got = to_u16(out)
        assert np.array_equal(got[:, ids], cache[:, ids]), (kind, off)


def test_mixed_context_batch_like_config3():
    """configs[3] in small: many requests of one layer with log-uniform
    lengths (whole blocks, partial tails holding stale values) in one shared
    pool, values shifted so ~5% of exponents escape the palette.  Every job's
    stream equals the reference chain's result (top16 overflows -> fixed6),
    and the batch round-trips into a second pool."""
    from unchainkv_b200 import workloads as W

    cfg = W.MixedConfig("c3_small", layers=1, model_layers=1, requests=20, min_tokens=16, max_tokens=2048,
                        scale_shift=5.5, kv_heads=2)
    blocks = W.request_blocks(cfg, W.request_lengths(cfg))
    pool = sum(blocks) + 7
    src_ids = W.request_block_tables(pool, blocks, 3000)
    dst_ids = W.request_block_tables(pool, blocks, 3001)
    scales = W.shard_scales(cfg, 0)
    cache = W.draw_tokens(77, scales, pool * cfg.block_tokens, cfg.scale_shift)
    cache = cache.reshape(2, pool, cfg.block_tokens, cfg.kv_heads, cfg.head_dim)
    tab = np.frombuffer(S.build_top16_tables(W.top16_codebooks_from_words(W.draw_tokens(78, scales, 4096))),
                        np.uint8).copy()
    kv = dev(cache.view(np.int16)).view(torch.bfloat16)
    out = torch.zeros_like(kv)
    tab_t = dev(tab)
    keep, jobs, djobs, views, expect = [kv, out, tab_t], [], [], [], []
    caps = [S.auto_capacity(2 * b * cfg.block_words) for b in blocks]
    buf = torch.zeros(sum((c + 15) // 16 * 16 for c in caps), dtype=torch.uint8, device="cuda")
    at = 0
    for b, ids, ids2, cap in zip(blocks, src_ids, dst_ids, caps):
        view = buf[at : at + cap]
        at += (cap + 15) // 16 * 16
        a, d = dev(ids), dev(ids2)
        keep += [a, d]
        jobs.append(job_for(kv, a, view, tab_t))
        res, stream = oracle.encode_top16_blocks(cache, ids, tab)
        if stream[0] == 255:
            res, stream = oracle.encode_mode_blocks(cache, ids, bits=6)
        expect.append(stream[:res])
        djobs.append(job_for(out, d, view, tab_t, stream_bytes=res))
        views.append(view)
    escapes = sum(oracle.escape_count(cache[:, ids].reshape(-1), tab) for ids in src_ids)
    words = sum(2 * b * cfg.block_words for b in blocks)
    assert 0.03 < escapes / words < 0.08
    assert S.encode_auto_batch(jobs)
    torch.cuda.synchronize()
    for i, (view, want) in enumerate(zip(views, expect)):
        assert np.array_equal(view.cpu().numpy()[: want.size], want), i
    assert S.decode_auto_batch(djobs)
    torch.cuda.synchronize()
    got = to_u16(out)
    for ids, ids2 in zip(src_ids, dst_ids):
        assert np.array_equal(got[:, ids2], cache[:, ids])
