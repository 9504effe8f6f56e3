"""The multi-GPU path's host logic on two gloo ranks (CPU): every rank codes
its own shard, the shards are disjoint, no data crosses ranks, and the
timing rule (max over ranks) holds.  The GPU data path has no collective, so
this covers everything a rank shares with the others."""

import json
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parents[1]


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_code_their_own_shards(tmp_path):
    out = tmp_path / "rank"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           str(ROOT / "tests" / "multirank_worker.py"), str(out)]
    proc = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-3000:]
    results = [json.loads(Path(f"{out}.{r}").read_text()) for r in range(2)]
    assert [r["heads"] for r in results] == [[0, 1], [1, 2]]
    assert all(r["exact"] for r in results)
    assert all(r["mode"] in (3, 5) for r in results)
    assert results[0]["stream_sha"] != results[1]["stream_sha"]
    assert all(r["max"] == 2.0 for r in results)


def test_transport_tokens_keep_the_order_on_two_gloo_ranks(tmp_path):
    """The stream transport's ready / free token exchange (the ordering the
    GPU transport relies on), on two gloo ranks."""
    out = tmp_path / "tok"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           str(ROOT / "tests" / "transport_worker.py"), str(out), "gloo", "6"]
    proc = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-3000:]
    results = [json.loads(Path(f"{out}.{r}").read_text()) for r in range(2)]
    assert all(r["ok"] for r in results), results
