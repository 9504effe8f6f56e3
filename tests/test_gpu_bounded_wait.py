"""Device-side waits run out, report, and leave the GPU usable.

Every mbarrier wait of the codec kernels is bounded (the reference spins
without a limit, native/unchain_kv/kvq_splitzip_cuda.cu:51-55).  Here a
test-only build of the fixed6 encode's statistics pass has a limit of 4
tries per wait, and its producer leaves one stage's full barrier an arrival
short (kvq_splitzip_test_encode_mode_skip_arrival): the consumers' wait for
that stage runs out.  Nothing faults and nothing waits without a limit:
the kernels return, kvq_splitzip_device_errors() counts the miss, the
stream carries a mode-255 header (no receiver decodes it), the count
resets, and the next ordinary encode gives the oracle's stream.
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


def words_with_palette(n, distinct=40, seed=0):
    rng = np.random.Generator(np.random.PCG64(seed))
    highs = np.sort(rng.choice(256, size=distinct, replace=False)).astype(np.uint16)
    return ((highs[rng.integers(0, distinct, size=n)] << 8) | rng.integers(0, 256, size=n)).astype(np.uint16)


@pytest.mark.parametrize("skip_tile", [0, 2])
def test_wait_that_runs_out_is_counted_and_marks_the_stream(skip_tile):
    lib = S._load()
    assert lib is not None, S.load_error()
    stream = torch.cuda.current_stream().cuda_stream
    n = 5 * 8192 + 100
    words = words_with_palette(n, seed=skip_tile)
    src = torch.from_numpy(words.view(np.int16)).cuda()
    cap = 2 * n
    dst = torch.zeros(cap, dtype=torch.uint8, device="cuda")
    exp_res, expected = oracle.encode_mode(words, bits=6, capacity=cap)
    assert expected[0] == 3

    S.device_errors_reset()
    assert S.device_errors() == 0
    res = lib.kvq_splitzip_test_encode_mode_skip_arrival(src.data_ptr(), dst.data_ptr(), n, cap, stream, 6,
                                                         skip_tile)
    torch.cuda.synchronize()  # the kernels returned
    assert res == exp_res
    assert S.device_errors() >= 1
    got = dst.cpu().numpy()
    assert got[0] == 255  # reported in band: the receiver declines this stream

    # the count resets, and the context is usable: an ordinary encode matches
    S.device_errors_reset()
    assert S.device_errors() == 0
    dst.zero_()
    assert lib.kvq_splitzip_bf16_encode_mode(src.data_ptr(), dst.data_ptr(), n, cap, stream, 6) == exp_res
    torch.cuda.synchronize()
    assert np.array_equal(dst.cpu().numpy()[:exp_res], expected)
    assert S.device_errors() == 0


def test_skip_beyond_the_last_tile_changes_nothing():
    """With the skipped tile past the input, the test build runs like the
    product one: no wait runs out and the stream is the oracle's."""
    lib = S._load()
    stream = torch.cuda.current_stream().cuda_stream
    n = 3 * 8192 + 7
    words = words_with_palette(n, seed=9)
    src = torch.from_numpy(words.view(np.int16)).cuda()
    cap = 2 * n
    dst = torch.zeros(cap, dtype=torch.uint8, device="cuda")
    exp_res, expected = oracle.encode_mode(words, bits=6, capacity=cap)
    S.device_errors_reset()
    res = lib.kvq_splitzip_test_encode_mode_skip_arrival(src.data_ptr(), dst.data_ptr(), n, cap, stream, 6,
                                                         1 << 30)
    torch.cuda.synchronize()
    assert res == exp_res
    assert np.array_equal(dst.cpu().numpy()[:exp_res], expected)
    assert S.device_errors() == 0
