"""The reference's own Python wrapper and its own tests, run on this library.

The drop-in claim at the Python boundary: the reference's ctypes wrapper
(src/unchain_kv/splitzip_cuda.py, installed unchanged into baseline/_ref by
oracle/build.py) loads this repository's library through
UNCHAIN_KV_SPLITZIP_LIB, exactly as a reference deployment would, and
* the reference's wrapper tests (tests/test_splitzip_cuda.py, its GPU round
  trips at :92-185 included) pass unchanged against it;
* the per-layer call pattern of the reference's codec benchmark
  (scripts/bench_codec_matrix.py:104-188: gather the blocks, encode_top16,
  fixed6 when top16 overflows, decode into a paged cache) gives the oracle's
  streams and a bit-exact cache, with escapes exactly at the top16 capacity
  (every 200th word, :108-111) and above it.
Skipped when the reference package was not installed (no checkout at build
time).
"""

import importlib
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from unchainkv_b200 import splitzip_cuda as S  # noqa: E402
from unchainkv_b200 import workloads as W  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
REF_TESTS = REF / "reference_tests" / "test_splitzip_cuda.py"

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
    pytest.mark.skipif(not (REF / "unchain_kv" / "splitzip_cuda.py").exists(),
                       reason="reference package not installed in baseline/_ref"),
]


def reference_wrapper():
    """The reference's unchain_kv.splitzip_cuda, bound to this library."""
    os.environ["UNCHAIN_KV_SPLITZIP_LIB"] = str(S.library_path())
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    module = importlib.import_module("unchain_kv.splitzip_cuda")
    assert module.available(), module.load_error()
    assert Path(module._LIB._name).resolve() == S.library_path().resolve()
    return module


def test_reference_wrapper_tests_pass_unchanged_against_this_library():
    env = dict(os.environ, PYTHONPATH=str(REF), UNCHAIN_KV_SPLITZIP_LIB=str(S.library_path()))
    proc = subprocess.run([sys.executable, "-m", "pytest", "-q", "-rs", "-p", "no:cacheprovider", str(REF_TESTS)],
                          cwd=str(REF), env=env, capture_output=True, text=True, timeout=600)
    out = proc.stdout + proc.stderr
    assert proc.returncode == 0, out[-4000:]
    assert "skipped" not in out, out[-2000:]  # its GPU round trips ran
    assert "6 passed" in out, out[-2000:]


def matrix_layer_words(books: bytes, blocks: int, block_words: int, every: int) -> np.ndarray:
    """[2, blocks, block_words] words in the codec benchmark's top16 pattern:
    each plane one in-book exponent with a fixed mantissa, and one escaped
    exponent on every `every`-th word (every 200th: escapes == capacity)."""
    words = np.empty((2, blocks, block_words), dtype=np.uint16)
    words[0] = (books[0] << 7) | 0x15
    words[1] = (books[16] << 7) | 0x2A
    escape = next(v for v in range(1, 255) if v not in books)
    words.reshape(-1)[::every] = (escape << 7) | 0x33
    return words


@pytest.mark.parametrize("every", [200, 150])
def test_reference_call_pattern_through_reference_wrapper(every):
    ref = reference_wrapper()
    device = torch.device("cuda", 0)
    blocks, block_words, layers = 64, 16 * 8 * 128, 3
    pool = 2 * blocks
    ids = W.block_table(pool, blocks, 3000)
    ids2 = W.block_table(pool, blocks, 3001)
    ids_t = torch.as_tensor(ids, device=device)
    cache = torch.zeros((2, pool, block_words), dtype=torch.bfloat16, device=device)
    target = torch.zeros_like(cache)
    pack = torch.empty((2, blocks, block_words), dtype=torch.bfloat16, device=device)
    raw_bytes = pack.numel() * 2
    encoded = torch.empty(raw_bytes + 1, dtype=torch.uint8, device=device)
    for layer in range(layers):
        books = ref._TOP16_CODEBOOKS[layer * 32:(layer + 1) * 32]
        words = matrix_layer_words(books, blocks, block_words, every)
        cache.index_copy_(1, ids_t, torch.from_numpy(words.view(np.int16)).to(device).view(torch.bfloat16))
        torch.index_select(cache, 1, ids_t, out=pack)
        res = ref.encode_top16(pack, encoded, layer)
        torch.cuda.synchronize()
        tables = np.frombuffer(S.build_top16_tables(books), dtype=np.uint8)
        exp_res, exp_stream = oracle.encode_top16(words.reshape(-1), tables, capacity=raw_bytes + 1)
        assert res == exp_res
        got = encoded[:res].cpu().numpy()
        assert np.array_equal(got, exp_stream)
        target.zero_()
        if got[0] == 5:
            assert every == 200  # escapes exactly at capacity still fit
            copied = ref.decode_top16(encoded[:res], target, [int(i) for i in ids2], raw_bytes, layer)
        else:
            # the connector's fallback: top16 overflowed, re-encode as fixed6
            assert every < 200 and got[0] == 255
            res6 = ref.encode_bf16(pack, encoded, bits=6)
            torch.cuda.synchronize()
            e6, s6 = oracle.encode_mode(words.reshape(-1), bits=6, capacity=raw_bytes + 1)
            assert res6 == e6 and np.array_equal(encoded[:res6].cpu().numpy(), s6)
            copied = ref.decode_fixed6(encoded[:res6], target, [int(i) for i in ids2], raw_bytes)
        torch.cuda.synchronize()
        assert copied == raw_bytes
        got_cache = target.view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(got_cache[:, ids2], words)
