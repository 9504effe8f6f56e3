"""Codec-aware decode attention against decompress-then-attend in fp32.

The reference has no attention over compressed KV: its receiver decodes each
stream into the paged cache and runs attention on the bf16 copy
(scripts/bench_codec_attention.py:155-157).  The oracle here is that
pipeline on the CPU: the stream decoded by the CPU oracle, then
softmax(q K^T / sqrt(128)) V accumulated in float64.  Tolerance, from the
benchmark configuration: |out - ref| <= 1e-3 + 2e-2 |ref| (the kernel rounds
P to bf16 for the tensor-core PV product and writes bf16).
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from unchainkv_b200 import splitzip_cuda as S  # noqa: E402
from unchainkv_b200 import workloads as W  # noqa: E402

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

HEADS, DIM, BT = 8, 128, 16
RTOL, ATOL = 2e-2, 1e-3


def bf16_to_f32(words):
    return (words.astype(np.uint32) << 16).view(np.float32)


BOOKS = np.stack([np.arange(116, 132), np.arange(117, 133)]).astype(np.uint8)  # K, V exponents
TABLE = np.frombuffer(S.build_top16_tables(bytes(BOOKS.reshape(-1))), np.uint8)


def top16_words(rng, shape, escape_rate, hot=None):
    """Words whose exponents come from the plane's 16-entry book, except
    escapes at `escape_rate` (half of them large: exponent 136, about 512,
    so that an unpatched escape shows), plus all of `hot` (a boolean mask)."""
    plane = np.zeros(shape, np.int64)
    plane[1] = 1
    exp = BOOKS[plane, rng.integers(0, 16, shape)].astype(np.int64)
    esc = rng.random(shape) < escape_rate
    if hot is not None:
        esc |= hot
    exp[esc] = np.where(rng.random(int(esc.sum())) < 0.5, 110, 136)
    return ((rng.integers(0, 2, shape) << 15) | (exp << 7) | rng.integers(0, 128, shape)).astype(np.uint16)


def request(seed, ctx, layer, mode):
    """Words [2, blocks*16, 8, 128] of one request (config[0] distribution,
    stale values in the unused tail of the last block; for top16, exponents
    from a 16-entry book per plane with 0.3% escapes) and its stream."""
    blocks = -(-ctx // BT)
    if mode == 5:
        rng = np.random.Generator(np.random.PCG64(seed))
        words = top16_words(rng, (2, blocks * BT, HEADS, DIM), 0.003)
        res, stream = oracle.encode_top16(words.reshape(-1), TABLE)
        assert stream[0] == 5
        return words, stream[:res]
    words = W.draw_tokens(seed, W.channel_scales(layer), blocks * BT)
    if mode == 3:
        res, stream = oracle.encode_mode(words.reshape(-1), bits=6)
        assert stream[0] == 3
        stream = stream[:res]
    else:
        stream = np.concatenate([[6], words.reshape(-1).view(np.uint8)]).astype(np.uint8)
    return words, stream


def reference(q, words, ctx, group):
    """float64 softmax(q K^T / sqrt(128)) V over the first ctx tokens."""
    k = bf16_to_f32(words[0, :ctx]).astype(np.float64)  # [ctx, 8, 128]
    v = bf16_to_f32(words[1, :ctx]).astype(np.float64)
    qf = bf16_to_f32(q).astype(np.float64).reshape(HEADS, group, DIM)
    out = np.empty((HEADS, group, DIM))
    for h in range(HEADS):
        s = qf[h] @ k[:, h, :].T / np.sqrt(DIM)  # [group, ctx]
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[h] = p @ v[:, h, :]
    return out.reshape(HEADS * group, DIM)


def place(stream, aligned):
    """Upload a stream at an address 15 mod 16 (fixed6 and raw planes on
    16-byte boundaries), at 11 mod 16 (aligned=11: top16 planes on them), or
    at a 16-byte aligned one (planes past them)."""
    if aligned is True:
        buf = S.attention_stream_buffer(stream.size, "cuda")
        buf.copy_(torch.from_numpy(stream.copy()))
        return buf
    if aligned:
        raw = torch.empty(stream.size + 32, dtype=torch.uint8, device="cuda")
        start = (aligned - raw.data_ptr()) % 16
        buf = raw[start:start + stream.size]
        buf.copy_(torch.from_numpy(stream.copy()))
        return buf
    return torch.from_numpy(stream.copy()).cuda()


def run(ctxs, modes, group=4, seed=0, aligned=False, reqs=None):
    rng = np.random.Generator(np.random.PCG64(seed))
    if reqs is None:
        reqs = [request(seed * 1000 + i, c, i % 4, m) for i, (c, m) in enumerate(zip(ctxs, modes))]
    q = W.bf16_bits(rng.standard_normal((len(ctxs), HEADS * group, DIM)).astype(np.float32))
    q_t = torch.from_numpy(q.view(np.int16)).cuda().view(torch.bfloat16)
    out = torch.full_like(q_t, float("nan"))
    streams = [place(s, aligned) for _, s in reqs]
    table = torch.from_numpy(TABLE.copy()).cuda()
    tables = [table if m == 5 else None for m in modes] if 5 in modes else None
    assert S.attention_decode(q_t, streams, ctxs, out, tables=tables) == len(ctxs)
    torch.cuda.synchronize()
    got = bf16_to_f32(out.view(torch.int16).cpu().numpy().view(np.uint16))
    for i, ((words, _), ctx) in enumerate(zip(reqs, ctxs)):
        ref = reference(q[i], words, ctx, group)
        err = np.abs(got[i] - ref)
        assert np.all(err <= ATOL + RTOL * np.abs(ref)), (i, ctx, float(err.max()))


def test_fixed6_streams_ragged_contexts():
    # single token, partial and whole blocks, several items per request
    run([1, 15, 16, 17, 333, 2048], [3] * 6)


def test_raw_and_fixed6_streams_in_one_batch():
    run([100, 1000, 64, 7], [6, 3, 6, 3], seed=1)


@pytest.mark.parametrize("modes", [[3, 3, 3], [6, 3, 6]])
def test_streams_placed_on_plane_boundaries(modes):
    """Streams at addresses 15 mod 16 take the plain 16-byte load path."""
    run([17, 513, 4096], modes, seed=5, aligned=True)


def test_group_sizes():
    run([300, 40], [3, 3], group=1, seed=2)
    run([300, 40], [3, 3], group=8, seed=3)
    run([300, 40], [5, 5], group=1, seed=10)
    run([300, 40], [5, 5], group=8, seed=11, aligned=11)


def test_batch_of_config4():
    """configs[4] at full size: 32 requests, contexts log-uniform in
    [1024, 8192] (the benchmark's seeded contexts), fixed6 streams of the
    configs[0] distribution, 32 q heads over 8 kv heads."""
    ctxs = W.attention_contexts(W.CONFIGS["c4"])
    assert len(ctxs) == 32 and min(ctxs) >= 1024 and max(ctxs) <= 8192
    run(ctxs, [3] * 32, seed=4)
    run(ctxs, [5] * 32, seed=12)


@pytest.mark.parametrize("aligned", [False, True, 11])
def test_top16_streams(aligned):
    """top16 streams (mode 5, with the layer's table): body and nibbles
    decoded into the fragments from the books; the escapes, read from the
    sorted entries, corrected in S^T (K) and in the partials (V)."""
    run([1, 37, 16, 300, 1029], [5] * 5, seed=6, aligned=aligned)


def test_top16_fixed6_and_raw_streams_in_one_batch():
    run([200, 75, 1000, 33], [5, 3, 6, 5], seed=7)
    run([64, 64], [3, 3], seed=8, reqs=[request(8000, 64, 0, 3), request(8001, 64, 1, 3)])


@pytest.mark.parametrize("plane", [0, 1])
def test_top16_stage_with_more_escapes_than_it_holds(plane):
    """A block plane with about 6000 escapes in a stream still within
    capacity.  K plane: runs of one token and head span many 32-entry chunks
    of the escape warp's sums.  V plane: more escapes than one batch of the
    correction kernel holds (4096 at group 4), so the item takes two."""
    ctx = 64 * BT
    rng = np.random.Generator(np.random.PCG64(9 + plane))
    shape = (2, ctx, HEADS, DIM)
    hot = np.zeros(shape, bool)
    hot[plane, 3 * BT:4 * BT] = rng.random((BT, HEADS, DIM)) < 0.37  # block 3 of the plane
    words = top16_words(rng, shape, 0.0005, hot=hot)
    res, stream = oracle.encode_top16(words.reshape(-1), TABLE)
    assert stream[0] == 5 and int(hot.sum()) > 5088
    run([ctx], [5], seed=9, reqs=[(words, stream[:res])])


def test_declines_bad_shapes():
    q = torch.zeros((1, 32, 128), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros_like(q)
    s = torch.zeros(100, dtype=torch.uint8, device="cuda")
    assert S.attention_decode(q, [s], [0], out) is None  # empty context
    assert S.attention_decode(q[:, :30], [s], [5], out[:, :30]) is None  # heads not a multiple of 8
    assert S.attention_decode(q.float(), [s], [5], out) is None
