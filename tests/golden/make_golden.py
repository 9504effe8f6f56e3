#!/usr/bin/env python3
"""Generate the golden vectors that pin the CPU oracle to the reference.

Run from the repository root, in a checkout where the reference tree is
available (its location is ``UNCHAIN_KV_REFERENCE_ROOT``, or the default
``REFERENCE`` below)::

    python tests/golden/make_golden.py

Every expected output below is produced by the REFERENCE's own CPU code,
imported from its source tree:

* ``unchain_kv.splitzip_cuda._TOP16_CODEBOOKS`` / ``_top16_tables``
  (src/unchain_kv/splitzip_cuda.py:11-31, 283-298) -> ``top16_tables.bin``;
* ``unchain_kv.vllm_connector._decode_splitzip_top16_payload``
  (src/unchain_kv/vllm_connector.py:176-220), the pure-Python top16 decoder
  -> decoded words of oracle-encoded streams and of the hand-built payload of
  tests/test_vllm_connector.py:333-371;
* ``UnchainKVConnector._copy_splitzip_bf16_native_blocks`` with the native
  decoder off (src/unchain_kv/vllm_connector.py:5098-5313), the torch mode-3
  (fixed6) and mode-4 (fixed5) receivers -> decoded caches of oracle-encoded
  fixed streams;
* ``UnchainKVConnector._splitzip_bf16_native_blocks`` on CPU tensors, the
  torch-op encoder (src/unchain_kv/vllm_connector.py:3204-3366), and the
  torch receiver -> mode 2 / 0 / 1 streams and their decoded caches;
* ``unchain_kv.trace.summarize_symbol_counts`` (src/unchain_kv/trace.py:27-58),
  the palette ranking rule -> top-16 exponent lists of seeded histograms and
  the whole summary the calibration trace records for them.

The streams themselves come from the CPU oracle (oracle/splitzip_oracle.c);
storing them pins the oracle's canonical bytes against regressions, while the
reference decoders pin their meaning.  The fixtures are small (a few tens of
KB) and committed; the GPU box never needs the reference tree.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
# the reference checkout: UNCHAIN_KV_REFERENCE_ROOT, else one named
# `reference` beside this repository
REFERENCE = Path(os.environ.get("UNCHAIN_KV_REFERENCE_ROOT") or REPO.parent / "reference")
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REFERENCE / "src"))
os.environ["UNCHAIN_KV_SPLITZIP_NATIVE_DECODE"] = "0"

import torch  # noqa: E402

from oracle import oracle  # noqa: E402
import unchain_kv.splitzip_cuda as ref_splitzip  # noqa: E402
import unchain_kv.vllm_connector as ref_connector  # noqa: E402
from unchain_kv.trace import summarize_symbol_counts  # noqa: E402


def ref_tables(layer: int) -> bytes:
    return bytes(ref_splitzip._top16_tables(layer, "cpu", torch).tolist())


def words_from_books(rng, n, books, escape_every=None, escape_exp=None, escape_rate=0.0):
    """Seeded words whose exponents come from the plane's codebook, with
    selected escapes (exponents outside the book)."""
    index = np.arange(n)
    plane = (index >= n // 2).astype(np.int64)
    book = np.frombuffer(books, dtype=np.uint8).reshape(2, 16)
    exp = book[plane, rng.integers(0, 16, size=n)].astype(np.int64)
    outside = np.array([v for v in range(256) if v not in set(books)], dtype=np.int64)
    if escape_every:
        exp[::escape_every] = escape_exp if escape_exp is not None else outside[0]
    if escape_rate:
        mask = rng.random(n) < escape_rate
        exp[mask] = rng.choice(outside, size=int(mask.sum()))
    sign = rng.integers(0, 2, size=n)
    mant = rng.integers(0, 128, size=n)
    return ((sign << 15) | (exp << 7) | mant).astype(np.uint16)


def make_connector():
    config = SimpleNamespace(kv_transfer_config=SimpleNamespace(kv_role="kv_consumer"))
    return ref_connector.UnchainKVConnector(config, "worker")


def main() -> None:
    out = {}
    rng = np.random.Generator(np.random.PCG64(7))

    # ---- interface tables -------------------------------------------------
    codebooks = bytes(ref_splitzip._TOP16_CODEBOOKS)
    layers = len(codebooks) // 32
    (HERE / "top16_codebooks.bin").write_bytes(codebooks)
    tables = b"".join(ref_tables(layer) for layer in range(layers))
    (HERE / "top16_tables.bin").write_bytes(tables)
    out["layers"] = layers

    # ---- top16: oracle streams decoded by the reference CPU decoder -------
    top16_cases = []
    arrays = {}
    specs = [
        # name, n, layer, escape_every, escape_rate
        ("small_one_escape", 256, 0, None, 0.0),
        ("at_capacity", 2 * 3 * 2048, 5, 200, 0.0),
        ("random_escapes", 2 * 2 * 4096, 17, None, 0.003),
        ("odd_blocks", 2 * 7 * 130, 31, None, 0.004),
        ("overflow", 2 * 4 * 1024, 9, None, 0.02),
    ]
    for name, n, layer, every, rate in specs:
        books = codebooks[layer * 32 : (layer + 1) * 32]
        words = words_from_books(rng, n, books, escape_every=every, escape_rate=rate)
        if name == "small_one_escape":
            words[3] = (words[3] & 0x807F) | (100 << 7)
        table = np.frombuffer(ref_tables(layer), dtype=np.uint8)
        result, stream = oracle.encode_top16(words, table)
        assert result == oracle.top16_encoded_bytes(n), (name, result)
        decoded = ref_connector._decode_splitzip_top16_payload(bytes(stream), 2 * n, books)
        arrays[f"top16_{name}_words"] = words
        arrays[f"top16_{name}_stream"] = stream
        if decoded is None:
            assert stream[0] == 255, name
            arrays[f"top16_{name}_ref_decoded"] = np.zeros(0, dtype=np.uint16)
        else:
            arrays[f"top16_{name}_ref_decoded"] = np.frombuffer(decoded, dtype=np.uint16)
        top16_cases.append({"name": name, "n": n, "layer": layer,
                            "mode": int(stream[0]), "ref_decodes": decoded is not None})
    out["top16_cases"] = top16_cases

    # ---- the reference's hand-built top16 payload (KAT) -------------------
    # Construction described at tests/test_vllm_connector.py:333-371: 256 words,
    # layer-0 codebooks, code = index % 16, sign = index % 2, mantissa =
    # index % 128, one escape at position 3 with exponent 100.
    count = 256
    books = codebooks[:32]
    words = []
    body = bytearray(count)
    codes = bytearray((count + 1) // 2)
    for index in range(count):
        plane = index >= count // 2
        code = index % 16
        exponent = books[plane * 16 + code]
        if index == 3:
            exponent, code = 100, 0
        word = ((index % 2) << 15) | (exponent << 7) | (index % 128)
        words.append(word)
        body[index] = (word & 0x7F) | ((word >> 8) & 0x80)
        codes[index // 2] |= code << ((index % 2) * 4)
    capacity = (count + 199) // 200
    payload = bytearray(5 + count + len(codes) + capacity * 5)
    payload[0] = 5
    payload[1:5] = (1).to_bytes(4, "little")
    payload[5 : 5 + count] = body
    payload[5 + count : 5 + count + len(codes)] = codes
    entry = 5 + count + len(codes)
    payload[entry : entry + 4] = (3).to_bytes(4, "little")
    payload[entry + 4] = 100
    decoded = ref_connector._decode_splitzip_top16_payload(bytes(payload), count * 2, books)
    assert decoded == b"".join(w.to_bytes(2, "little") for w in words)
    arrays["kat_payload"] = np.frombuffer(bytes(payload), dtype=np.uint8)
    arrays["kat_words"] = np.array(words, dtype=np.uint16)

    # ---- fixed6 / fixed5: oracle streams through the torch receiver -------
    connector = make_connector()
    fixed_cases = []
    for name, bits, blocks, block_words, distinct in (
        ("fixed6_scatter", 6, 12, 256, 40),
        ("fixed6_ragged", 6, 5, 31, 64),
        ("fixed5_scatter", 5, 8, 128, 30),
    ):
        n = 2 * blocks * block_words
        highs = np.sort(rng.choice(256, size=distinct, replace=False)).astype(np.uint16)
        words = ((highs[rng.integers(0, distinct, size=n)] << 8)
                 | rng.integers(0, 256, size=n)).astype(np.uint16)
        result, stream = oracle.encode_mode(words, bits=bits)
        assert result == oracle.fixed_encoded_bytes(n, bits) and stream[0] == (3 if bits == 6 else 4)
        pool = blocks * 3
        ids = [int(v) for v in rng.permutation(pool)[:blocks]]
        target = torch.zeros((2, pool, block_words), dtype=torch.bfloat16)
        restored, copied = connector._copy_splitzip_bf16_native_blocks(
            target, ids, [bytes(stream)],
            {"raw_bytes": 2 * n, "encoded_bytes": int(result)})
        assert (restored, copied) == (blocks, 2 * n), (name, restored, copied)
        cache = target.view(torch.int16).numpy().view(np.uint16).copy()
        arrays[f"{name}_words"] = words
        arrays[f"{name}_stream"] = stream
        arrays[f"{name}_ids"] = np.array(ids, dtype=np.int64)
        arrays[f"{name}_ref_cache"] = cache
        fixed_cases.append({"name": name, "bits": bits, "blocks": blocks,
                            "block_words": block_words, "pool": pool})
    out["fixed_cases"] = fixed_cases

    # ---- torch-op modes 2 / 0 / 1: the reference's own encoder and receiver
    # (src/unchain_kv/vllm_connector.py:3204-3366, 5168-5278) on CPU tensors
    torchop_cases = []
    saved = {name: os.environ.get(name) for name in ("UNCHAIN_KV_CODEC", "UNCHAIN_KV_CODEC_GPU_SLOTS")}
    os.environ["UNCHAIN_KV_CODEC"] = "splitzip_bf16"
    os.environ["UNCHAIN_KV_CODEC_GPU_SLOTS"] = "1"
    for name, pool, block_words, blocks in (
        ("mode2_narrow", 12, 512, 7),
        ("mode0_palette", 10, 1024, 6),
        ("mode1_nibbles", 9, 768, 5),
        ("mode2_ragged", 6, 37, 5),
    ):
        shape = (2, pool, block_words)
        if name.startswith("mode2"):
            high = (rng.integers(0, 2, shape) << 7) | rng.integers(58, 64 + 3 * (name == "mode2_ragged"), shape)
            low = rng.integers(0, 256, shape)
        elif name == "mode0_palette":
            highs = rng.choice(256, size=45, replace=False)
            high, low = highs[rng.integers(0, 45, shape)], rng.integers(0, 256, shape)
        else:
            high, low = rng.integers(0, 256, shape), (rng.integers(0, 256, shape) & 0x31) | 0x04
        cache = ((high << 8) | low).astype(np.uint16)
        # the reference gathers a contiguous run of blocks on the CPU (a
        # scattered list needs its GPU pack pool); its receiver scatters into
        # a permuted list
        start = int(rng.integers(0, pool - blocks + 1))
        src_ids = list(range(start, start + blocks))
        ids = [int(v) for v in rng.permutation(pool)[:blocks]]
        connector = ref_connector.UnchainKVConnector(
            SimpleNamespace(kv_transfer_config=SimpleNamespace(kv_role="kv_producer")), "worker")
        kv = torch.from_numpy(cache.view(np.int16).copy()).view(torch.bfloat16)
        encoded = connector._splitzip_bf16_native_blocks(kv, src_ids)
        assert encoded is not None, name
        data, _, raw_bytes, encoded_bytes, _ = encoded
        stream = np.frombuffer(bytes(data), dtype=np.uint8)[:encoded_bytes].copy()
        target = torch.zeros_like(kv)
        restored, copied = make_connector()._copy_splitzip_bf16_native_blocks(
            target, ids, [bytes(stream)], {"raw_bytes": raw_bytes, "encoded_bytes": encoded_bytes})
        assert (restored, copied) == (blocks, raw_bytes), (name, restored, copied)
        arrays[f"{name}_cache"] = cache
        arrays[f"{name}_src_ids"] = np.array(src_ids, dtype=np.int64)
        arrays[f"{name}_ids"] = np.array(ids, dtype=np.int64)
        arrays[f"{name}_stream"] = stream
        arrays[f"{name}_ref_cache"] = target.view(torch.int16).numpy().view(np.uint16).copy()
        torchop_cases.append({"name": name, "mode": int(stream[0]), "blocks": blocks})
    for key, value in saved.items():
        if value is None:
            os.environ.pop(key, None)
        else:
            os.environ[key] = value
    out["torchop_cases"] = torchop_cases

    # ---- palette ranking rule ---------------------------------------------
    rankings = []
    for seed in range(4):
        local = np.random.Generator(np.random.PCG64(100 + seed))
        hist = np.zeros(256, dtype=np.int64)
        hist[local.choice(256, size=40, replace=False)] = local.integers(1, 50, size=40)
        hist[local.choice(256, size=6, replace=False)] = 17  # ties
        summary = summarize_symbol_counts(hist.tolist())
        rankings.append({"histogram": hist.tolist(), "top16": summary["top16_exponents"], "summary": summary})
    out["rankings"] = rankings

    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    total = sum(p.stat().st_size for p in HERE.iterdir() if p.is_file())
    print(f"wrote golden fixtures ({total} bytes)")


if __name__ == "__main__":
    main()
