"""Seeded synthetic KV caches and palettes for the benchmark configurations.

No public dataset or checkpoint is involved: the configs specify a value
distribution, and this module draws it.

* Every (plane, kv_head, head_dim) channel has a scale s_c drawn
  log-uniform in [0.01, 4].  2% of channels are outliers with s_c x 50.
* A value is N(0, 1) * s_c in fp32, rounded to nearest-even bf16.
* The top16 palette of a layer is the 16 most frequent exponents of a
  seeded 4096-token calibration draw, one palette per plane.  Ties are
  broken by exponent value, and code = rank: the rule of the reference's
  trace.py:30-33 and scripts/extract_llama_top16_codebooks.py:39-40.
* Seeds: calibration 1000+layer, data 2000+layer, block tables 3000+k,
  request lengths 4000.  Shard s of a multi-GPU run (one process per GPU)
  adds 100000*s to the data seeds and holds kv heads
  [s*kv_heads, (s+1)*kv_heads) mod model_kv_heads of the model's channel
  scales: under TP=8 each GPU codes its own head of every layer.

Host (numpy, exact) and device (torch CUDA generator) drawers are provided.
The device drawer is for benchmark-sized caches and is seeded but not
bit-identical to the numpy one.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

KV_HEADS = 8
HEAD_DIM = 128
BLOCK_TOKENS = 16


@dataclass(frozen=True)
class CodecConfig:
    name: str
    layers: int
    tokens: int
    kv_heads: int = KV_HEADS
    head_dim: int = HEAD_DIM
    block_tokens: int = BLOCK_TOKENS
    pool_factor: int = 2  # pool blocks = pool_factor * blocks used
    model_kv_heads: int = KV_HEADS  # kv heads of the whole model (TP shards hold kv_heads of them)

    @property
    def blocks(self) -> int:
        return self.tokens // self.block_tokens

    @property
    def block_words(self) -> int:
        return self.block_tokens * self.kv_heads * self.head_dim

    @property
    def words_per_layer(self) -> int:
        return 2 * self.blocks * self.block_words

    @property
    def raw_bytes(self) -> int:
        return 2 * self.words_per_layer * self.layers


# BASELINE.json configs[0..2] (configs[3] and [4] have their own builders).
CONFIG0 = CodecConfig("c0_single_layer_roundtrip", layers=1, tokens=1024, pool_factor=4)
CONFIG1 = CodecConfig("c1_llama3_8b_prefill_4096", layers=32, tokens=4096)
CONFIG2 = CodecConfig("c2_llama3_70b_tp8_shard_32768", layers=80, tokens=32768, kv_heads=1)


@dataclass(frozen=True)
class MixedConfig:
    """many requests per layer with log-uniform
    lengths (most final blocks partial, the unused slots holding stale values
    of the same distribution), values drawn with their scale multiplied by
    `scale_shift` against an unshifted calibration so that about 5% of the
    exponents fall outside the palette.  `layers` of the model's
    `model_layers` are coded per step (device memory cap)."""

    name: str
    layers: int
    model_layers: int
    requests: int
    min_tokens: int
    max_tokens: int
    scale_shift: float
    kv_heads: int = KV_HEADS
    head_dim: int = HEAD_DIM
    block_tokens: int = BLOCK_TOKENS
    pool_factor: float = 1.25
    model_kv_heads: int = KV_HEADS

    @property
    def block_words(self) -> int:
        return self.block_tokens * self.kv_heads * self.head_dim


CONFIG3 = MixedConfig("c3_mixed_context_64req_escape5", layers=8, model_layers=32, requests=64,
                      min_tokens=256, max_tokens=32768, scale_shift=5.5)
CONFIGS = {"c0": CONFIG0, "c1": CONFIG1, "c2": CONFIG2, "c3": CONFIG3}


@dataclass(frozen=True)
class AttentionConfig:
    """decode attention of `requests` queries (32 q
    heads over 8 kv heads, head dim 128) over K/V held as fixed6 streams of
    16-token paged blocks drawn from the configs[0] distribution, contexts
    log-uniform in [min_tokens, max_tokens] (seed 4004)."""

    name: str
    requests: int = 32
    min_tokens: int = 1024
    max_tokens: int = 8192
    group: int = 4
    kv_heads: int = KV_HEADS
    head_dim: int = HEAD_DIM
    block_tokens: int = BLOCK_TOKENS
    model_kv_heads: int = KV_HEADS
    layers: int = 1

    @property
    def block_words(self) -> int:
        return self.block_tokens * self.kv_heads * self.head_dim


CONFIG4 = AttentionConfig("c4_codec_decode_attention_32req")
CONFIGS["c4"] = CONFIG4


def attention_contexts(cfg: AttentionConfig) -> list[int]:
    rng = np.random.Generator(np.random.PCG64(4004))
    lo, hi = np.log(cfg.min_tokens), np.log(cfg.max_tokens)
    return [int(x) for x in np.floor(np.exp(rng.uniform(lo, hi, size=cfg.requests)))]


def request_lengths(cfg: MixedConfig) -> np.ndarray:
    """Seeded log-uniform request lengths in tokens (seed 4000)."""
    rng = np.random.Generator(np.random.PCG64(4000))
    lo, hi = np.log(cfg.min_tokens), np.log(cfg.max_tokens)
    return np.floor(np.exp(rng.uniform(lo, hi, size=cfg.requests))).astype(np.int64)


def request_blocks(cfg: MixedConfig, lengths) -> list[int]:
    """Whole blocks per request (a partial last block is sent whole, as the
    reference does)."""
    return [int(-(-int(t) // cfg.block_tokens)) for t in lengths]


def request_block_tables(pool_blocks: int, blocks: list[int], seed: int) -> list[np.ndarray]:
    """Disjoint block tables: a seeded permutation of the pool split among
    the requests in order."""
    perm = np.random.Generator(np.random.PCG64(seed)).permutation(pool_blocks).astype(np.int64)
    out, at = [], 0
    for b in blocks:
        out.append(perm[at : at + b].copy())
        at += b
    if at > pool_blocks:
        raise ValueError("pool smaller than the requests' blocks")
    return out


def channel_scales(layer: int, kv_heads: int = KV_HEADS, head_dim: int = HEAD_DIM,
                   outlier_factor: float = 50.0) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(1000 + layer))
    scales = np.exp(rng.uniform(np.log(0.01), np.log(4.0), size=(2, kv_heads, head_dim)))
    outliers = rng.random((2, kv_heads, head_dim)) < 0.02
    scales[outliers] *= outlier_factor
    return scales.astype(np.float32)


def shard_heads(cfg: CodecConfig, shard: int) -> tuple[int, int]:
    """Model kv heads [h0, h1) held by shard `shard` (one process per GPU)."""
    h0 = (shard * cfg.kv_heads) % cfg.model_kv_heads
    return h0, h0 + cfg.kv_heads


def shard_scales(cfg: CodecConfig, layer: int, shard: int = 0) -> np.ndarray:
    """Channel scales [2, kv_heads, head_dim] of a shard's heads of `layer`."""
    h0, h1 = shard_heads(cfg, shard)
    return channel_scales(layer, cfg.model_kv_heads, cfg.head_dim)[:, h0:h1]


def max_over_ranks(value: float) -> float:
    """Max of `value` over the ranks of the default process group (the
    benchmark's timing rule); the value itself when not distributed.  Works
    with the gloo (CPU) and nccl (current CUDA device) backends."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def bf16_bits(values: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    rounded = bits + np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))
    return (rounded >> np.uint32(16)).astype(np.uint16)


def draw_tokens(seed: int, scales: np.ndarray, tokens: int, scale_shift: float = 1.0) -> np.ndarray:
    """[2, tokens, kv_heads, head_dim] bf16 bit patterns (uint16)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    kvh, hd = scales.shape[1:]
    values = rng.standard_normal((2, tokens, kvh, hd), dtype=np.float32)
    values *= (scales * np.float32(scale_shift))[:, None, :, :]
    return bf16_bits(values)


def top16_codebooks_from_words(words: np.ndarray) -> bytes:
    """32 codebook bytes (K then V) from [2, ...] bf16 words."""
    from .splitzip_cuda import rank_top16

    books = bytearray()
    for plane in range(2):
        exps = (words[plane].reshape(-1) >> 7) & 0xFF
        hist = np.bincount(exps, minlength=256)
        top = rank_top16(hist)
        if len(top) < 16:  # pad with unused exponents so the table is complete
            top += [e for e in range(256) if e not in top][: 16 - len(top)]
        books.extend(top)
    return bytes(books)


def layer_codebooks(layer: int, kv_heads: int = KV_HEADS, head_dim: int = HEAD_DIM) -> bytes:
    scales = channel_scales(layer, kv_heads, head_dim)
    calibration = draw_tokens(1000 + layer + 100000, scales, 4096)
    return top16_codebooks_from_words(calibration)


def shard_codebooks(cfg: CodecConfig, layer: int, shard: int = 0) -> bytes:
    """Host-calibrated codebooks of a shard's heads of `layer`."""
    calibration = draw_tokens(1000 + layer + 100000 + 1000000 * shard, shard_scales(cfg, layer, shard), 4096)
    return top16_codebooks_from_words(calibration)


def block_table(pool_blocks: int, blocks: int, seed: int) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.permutation(pool_blocks)[:blocks].astype(np.int64)


def paged_cache_host(cfg: CodecConfig, layer: int, ids: np.ndarray, scale_shift: float = 1.0,
                     fill_seed: int | None = None, shard: int = 0) -> np.ndarray:
    """A [2, pool, block_tokens, kv_heads, head_dim] uint16 cache whose blocks
    `ids` hold one request's tokens (in block-table order) and whose other
    blocks hold independent draws of the same distribution."""
    pool = cfg.blocks * cfg.pool_factor
    scales = shard_scales(cfg, layer, shard)
    cache = draw_tokens(fill_seed if fill_seed is not None else 5000 + layer + 100000 * shard, scales,
                        pool * cfg.block_tokens, scale_shift)
    cache = cache.reshape(2, pool, cfg.block_tokens, cfg.kv_heads, cfg.head_dim)
    request = draw_tokens(2000 + layer + 100000 * shard, scales, cfg.tokens, scale_shift)
    cache[:, ids] = request.reshape(2, cfg.blocks, cfg.block_tokens, cfg.kv_heads, cfg.head_dim)
    return cache


# ------------------------------------------------------------------ device


def draw_tokens_device(seed: int, scales, tokens: int, device, scale_shift: float = 1.0):
    """Device analogue of draw_tokens: returns a bf16 tensor [2, tokens, kvh, hd]."""
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    sc = torch.as_tensor(np.asarray(scales) * scale_shift, device=device, dtype=torch.float32)
    kvh, hd = sc.shape[1:]
    values = torch.randn((2, tokens, kvh, hd), generator=gen, device=device, dtype=torch.float32)
    values.mul_(sc[:, None])
    return values.to(torch.bfloat16)


def codebooks_device(words_bf16) -> bytes:
    """Codebooks from a device bf16 tensor [2, ...] (histograms on the GPU)."""
    import torch

    from .splitzip_cuda import rank_top16

    books = bytearray()
    for plane in range(2):
        w = words_bf16[plane].reshape(-1).view(torch.int16).to(torch.int32) & 0xFFFF
        hist = torch.bincount((w >> 7) & 0xFF, minlength=256).cpu().tolist()
        top = rank_top16(hist)
        if len(top) < 16:
            top += [e for e in range(256) if e not in top][: 16 - len(top)]
        books.extend(top)
    return bytes(books)


def fill_layer_device(cache_layer, cfg: CodecConfig, layer: int, ids, scale_shift: float = 1.0, shard: int = 0):
    """Fill a device cache layer [2, pool, bt, kvh, hd] (bf16) in place:
    request tokens at `ids`, independent draws elsewhere.  Returns the
    layer's calibrated codebooks (32 bytes)."""
    import torch

    device = cache_layer.device
    pool = cache_layer.shape[1]
    scales = shard_scales(cfg, layer, shard)
    filler = draw_tokens_device(5000 + layer + 100000 * shard, scales, pool * cfg.block_tokens, device, scale_shift)
    cache_layer.copy_(filler.view(2, pool, cfg.block_tokens, cfg.kv_heads, cfg.head_dim))
    request = draw_tokens_device(2000 + layer + 100000 * shard, scales, cfg.tokens, device, scale_shift)
    ids_t = torch.as_tensor(ids, device=device, dtype=torch.int64)
    cache_layer.index_copy_(1, ids_t, request.view(2, cfg.blocks, cfg.block_tokens, cfg.kv_heads, cfg.head_dim))
    calibration = draw_tokens_device(1000 + layer + 100000 + 1000000 * shard, scales, 4096, device)
    return codebooks_device(calibration)


def fill_pool_device(cache_layer, cfg: MixedConfig, layer: int, shard: int = 0):
    """Fill a whole device pool layer [2, pool, bt, kvh, hd] (bf16) with the
    shifted distribution (every request's blocks, partial tails included,
    hold draws of it).  Returns the codebooks of an unshifted calibration."""
    device = cache_layer.device
    pool = cache_layer.shape[1]
    scales = shard_scales(cfg, layer, shard)
    values = draw_tokens_device(2000 + layer + 100000 * shard, scales, pool * cfg.block_tokens, device,
                                cfg.scale_shift)
    cache_layer.copy_(values.view(2, pool, cfg.block_tokens, cfg.kv_heads, cfg.head_dim))
    calibration = draw_tokens_device(1000 + layer + 100000 + 1000000 * shard, scales, 4096, device)
    return codebooks_device(calibration)


def mixed_sample_host(cfg: MixedConfig, layer: int, requests: int, shard: int = 0):
    """Host (numpy) sample of configs[3] for the CPU baseline: the first
    `requests` requests of `layer` in a pool that holds just their blocks.
    Returns (cache, block tables, codebooks)."""
    blocks = request_blocks(cfg, request_lengths(cfg)[:requests])
    pool = sum(blocks)
    tables = request_block_tables(pool, blocks, 3000)
    scales = shard_scales(cfg, layer, shard)
    cache = draw_tokens(2000 + layer + 100000 * shard, scales, pool * cfg.block_tokens, cfg.scale_shift)
    cache = cache.reshape(2, pool, cfg.block_tokens, cfg.kv_heads, cfg.head_dim)
    calibration = draw_tokens(1000 + layer + 100000 + 1000000 * shard, scales, 4096)
    return cache, tables, top16_codebooks_from_words(calibration)
