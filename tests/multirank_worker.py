"""One rank of the two-rank CPU (gloo) check of the multi-GPU path's host
logic; started by tests/test_multirank_gloo.py through torchrun.

Each rank codes its own shard of a TP-sharded model (its own kv head of the
70B-like config, one layer, a few blocks) with the CPU oracle: top16, then the
reference's fallback to fixed6 when the escapes overflow, then a decode back
into a paged cache.  It reports its heads, stream mode and checksum, whether
the round trip was exact, and the max-over-ranks value of (rank + 1), to
the JSON file named by argv[1] with the rank appended."""

from __future__ import annotations

import dataclasses
import datetime
import hashlib
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main() -> None:
    out = Path(sys.argv[1])
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import oracle
        from unchainkv_b200 import splitzip_cuda as S
        from unchainkv_b200 import workloads as w

        cfg = dataclasses.replace(w.CONFIGS["c2"], layers=1, tokens=256)
        pool = cfg.blocks * cfg.pool_factor
        ids = w.block_table(pool, cfg.blocks, 3000)
        cache = w.paged_cache_host(cfg, 0, ids, shard=rank)
        tables = np.frombuffer(S.build_top16_tables(w.shard_codebooks(cfg, 0, rank)), np.uint8).copy()
        res, stream = oracle.encode_top16_blocks(cache, ids, tables)
        target = np.zeros_like(cache)
        if stream[0] == 5:
            oracle.decode_top16_blocks(stream[:res], target, ids, tables)
        else:
            res, stream = oracle.encode_mode_blocks(cache, ids, bits=6)
            oracle.decode_fixed6_blocks(stream[:res], target, ids)
        exact = bool(np.array_equal(target[:, ids], cache[:, ids]))
        result = {
            "rank": rank,
            "world": world,
            "heads": list(w.shard_heads(cfg, rank)),
            "mode": int(stream[0]),
            "stream_sha": hashlib.sha256(stream[:res].tobytes()).hexdigest(),
            "exact": exact,
            "max": w.max_over_ranks(float(rank + 1)),
        }
        dist.barrier()
        Path(f"{out}.{rank}").write_text(json.dumps(result))
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
