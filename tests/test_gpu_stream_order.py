"""Stream order across overlapped launches.

The codec kernels are launched so that each may be scheduled while the
previous kernel of its stream finishes; each waits for that kernel before it
touches global memory.  Here batches run back to back on one stream with no
host synchronisation in between and reuse the same stream buffer: encode A,
decode A, encode B into the same buffer, decode B, and so on.  If any kernel
read or wrote global memory before its predecessor completed, a decode would
see the next encode's bytes (or a stats pass the previous encode's scratch)
and a cache would differ from its source.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from unchainkv_b200 import splitzip_cuda as S  # noqa: E402

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

BOOKS = S._DEFAULT_TOP16_CODEBOOKS


def dev(a):
    return torch.from_numpy(np.array(a, copy=True, order="C")).cuda()


def book_cache(rng, pool, shape, layer, rate):
    """A paged cache [2, pool, *shape] of words whose exponents come from the
    layer's top16 books, with a fraction `rate` of other exponents."""
    book = np.frombuffer(BOOKS[layer * 32:layer * 32 + 32], np.uint8).reshape(2, 16).astype(np.int64)
    full = (2, pool) + shape
    plane = np.zeros(full, dtype=np.int64)
    plane[1] = 1
    exp = book[plane, rng.integers(0, 16, full)]
    esc = rng.random(full) < rate
    exp[esc] = rng.integers(1, 255, int(esc.sum()))
    return ((rng.integers(0, 2, full) << 15) | (exp << 7) | rng.integers(0, 128, full)).astype(np.uint16)


@pytest.mark.parametrize("rate", [0.003, 0.02])
def test_back_to_back_batches_reusing_one_buffer(rate):
    rng = np.random.Generator(np.random.PCG64(int(rate * 1e4) + 5))
    shape, pool, blocks, layers = (16, 8, 128), 24, 16, 3
    n = 2 * blocks * int(np.prod(shape))
    tables = [dev(np.frombuffer(S.build_top16_tables(BOOKS[l * 32:l * 32 + 32]), np.uint8)) for l in range(layers)]
    cap = (S.auto_capacity(n) + 15) // 16 * 16
    buf = torch.zeros(layers * cap, dtype=torch.uint8, device="cuda")  # one buffer, every round
    rounds = []
    keep = []
    for r in range(6):
        caches = [book_cache(rng, pool, shape, l, rate) for l in range(layers)]
        ids = rng.permutation(pool)[:blocks].astype(np.int64)
        ids2 = rng.permutation(pool)[:blocks].astype(np.int64)
        kv = [dev(c.view(np.int16)).view(torch.bfloat16) for c in caches]
        out = [torch.zeros_like(k) for k in kv]
        ids_t, ids2_t = dev(ids), dev(ids2)
        keep += kv + out + [ids_t, ids2_t]
        enc = [S.make_job(kv[l], ids_t, buf[l * cap:(l + 1) * cap], cap, tables[l]) for l in range(layers)]
        dec = [S.make_job(out[l], ids2_t, buf[l * cap:(l + 1) * cap], cap, tables[l]) for l in range(layers)]
        rounds.append((caches, ids, ids2, out, enc, dec))
    torch.cuda.synchronize()
    # every round on the current stream, no host synchronisation in between
    for caches, ids, ids2, out, enc, dec in rounds:
        assert S.encode_auto_batch(enc)
        assert S.decode_auto_batch(dec)
    torch.cuda.synchronize()
    for caches, ids, ids2, out, enc, dec in rounds:
        for l in range(layers):
            got = out[l].view(torch.int16).cpu().numpy().view(np.uint16)
            assert np.array_equal(got[:, ids2], caches[l][:, ids])
    # and the last round's streams are the oracle's
    caches, ids = rounds[-1][0], rounds[-1][1]
    host = buf.cpu().numpy()
    for l in range(layers):
        expected = oracle.encode_auto_blocks(caches[l], ids, tables[l].cpu().numpy())
        assert np.array_equal(host[l * cap:l * cap + expected.size], expected)
