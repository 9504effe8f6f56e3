"""Codec writeback (the reference's _try_splitzip_writeback,
vllm_connector.py:3460-3563, segments :3720-3738): after an encode, each
layer's stream is copied over its own blocks, K-plane run then V-plane run;
reading the segments back in order gives the stream, which decodes to the
original words.  Fragmented, non-adjacent and aliasing cases decline."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from unchainkv_b200 import splitzip_cuda as S  # noqa: E402
from unchainkv_b200 import workloads as W  # noqa: E402

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]


def test_streams_written_over_their_blocks_read_back_and_decode():
    layers, pool, blocks, start = 3, 40, 12, 7
    kv = torch.empty((layers, 2, pool, 16, 8, 128), dtype=torch.bfloat16, device="cuda")
    for l in range(layers):
        words = W.draw_tokens(2000 + l, W.channel_scales(l), pool * 16).reshape(2, pool, 16, 8, 128)
        kv[l].copy_(torch.from_numpy(words.view(np.int16)).view(torch.bfloat16))
    original = kv.clone()
    n = 2 * blocks * 16 * 8 * 128
    cap = (S.auto_capacity(n) + 15) // 16 * 16
    buf = torch.zeros(layers * cap, dtype=torch.uint8, device="cuda")
    tables = torch.from_numpy(np.frombuffer(S.build_top16_tables(S._DEFAULT_TOP16_CODEBOOKS[:32]),
                                            np.uint8).copy()).cuda()
    enc = [S.make_job(kv[l], None, buf[l * cap:(l + 1) * cap], cap, tables, start, blocks) for l in range(layers)]
    assert S.encode_auto_batch(enc)
    torch.cuda.synchronize()
    heads = buf.view(layers, cap)[:, :8].cpu().numpy()
    lengths = [S.stream_length(bytes(h), n) for h in heads]
    streams = [buf[l * cap:l * cap + lengths[l]].clone() for l in range(layers)]
    jobs = [S.writeback_job(kv[l], buf[l * cap:(l + 1) * cap], lengths[l], start, blocks) for l in range(layers)]
    assert S.writeback_batch(jobs) == sum(lengths)
    torch.cuda.synchronize()
    for l in range(layers):
        segments = S.writeback_segments(kv[l], start, blocks)
        staged = torch.cat(segments)[:lengths[l]]
        assert torch.equal(staged, streams[l])
        # blocks outside the run are untouched
        assert torch.equal(kv[l][:, :start], original[l][:, :start])
        assert torch.equal(kv[l][:, start + blocks:], original[l][:, start + blocks:])
        # the staged bytes decode to the original words
        out = torch.zeros_like(kv[l])
        assert S.decode_any_batch([S.make_job(out, None, staged.clone(), lengths[l], tables, start, blocks)])
        torch.cuda.synchronize()
        assert torch.equal(out[:, start:start + blocks].view(torch.int16),
                           original[l][:, start:start + blocks].view(torch.int16))


def test_writeback_declines_like_the_reference():
    kv = torch.zeros((2, 20, 16, 1, 128), dtype=torch.bfloat16, device="cuda")
    buf = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    ids = torch.arange(3, 8, device="cuda")
    fragmented = S.make_job(kv, ids, buf, 1024)
    assert S.writeback_batch([fragmented]) is None
    too_long = S.writeback_job(kv, buf, 2 * 2 * 2 * 16 * 128 + 1, 3, 2)
    assert S.writeback_batch([too_long]) is None
    inside = kv[0, 3:5].reshape(-1).view(torch.uint8)
    aliasing = S.writeback_job(kv, inside, 64, 3, 2)
    assert S.writeback_batch([aliasing]) is None
    strided = torch.zeros((2, 20, 32, 1, 128), dtype=torch.bfloat16, device="cuda")[:, :, :16]
    assert S.writeback_batch([S.writeback_job(strided, buf, 64, 3, 2)]) is None
