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


def request(seed, ctx, layer, mode):
    """Words [2, blocks*16, 8, 128] of one request (config[0] distribution,
    stale values in the unused tail of the last block) and its stream."""
    blocks = -(-ctx // BT)
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
    """Upload a stream at an address 15 mod 16 (planes on 16-byte
    boundaries) or at a 16-byte aligned one (planes 1 byte past them)."""
    if aligned:
        buf = S.attention_stream_buffer(stream.size, "cuda")
        buf.copy_(torch.from_numpy(stream.copy()))
        return buf
    return torch.from_numpy(stream.copy()).cuda()


def run(ctxs, modes, group=4, seed=0, aligned=False):
    rng = np.random.Generator(np.random.PCG64(seed))
    reqs = [request(seed * 1000 + i, c, i % 4, m) for i, (c, m) in enumerate(zip(ctxs, modes))]
    q = W.bf16_bits(rng.standard_normal((len(ctxs), HEADS * group, DIM)).astype(np.float32))
    q_t = torch.from_numpy(q.view(np.int16)).cuda().view(torch.bfloat16)
    out = torch.full_like(q_t, float("nan"))
    streams = [place(s, aligned) for _, s in reqs]
    assert S.attention_decode(q_t, streams, ctxs, out) == len(ctxs)
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


def test_batch_like_config4():
    """configs[4] in small: 8 requests, contexts log-uniform in [1024, 8192]."""
    rng = np.random.Generator(np.random.PCG64(4))
    ctxs = [int(x) for x in np.exp(rng.uniform(np.log(1024), np.log(8192), size=8))]
    run(ctxs, [3] * 8, seed=4)


def test_declines_bad_shapes():
    q = torch.zeros((1, 32, 128), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros_like(q)
    s = torch.zeros(100, dtype=torch.uint8, device="cuda")
    assert S.attention_decode(q, [s], [0], out) is None  # empty context
    assert S.attention_decode(q[:, :30], [s], [5], out[:, :30]) is None  # heads not a multiple of 8
    assert S.attention_decode(q.float(), [s], [5], out) is None
