"""GPU-to-GPU stream transport on two GPUs: rank 0 encodes layers (auto
codec) into its transport buffers, rank 1 decodes them straight from rank
0's HBM over NVLink into its own paged cache, two steps in flight, and checks
every step bit for bit (tests/transport_worker.py).  Skipped on a box with
fewer than two GPUs."""

import json
import socket
import subprocess
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parents[1]

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs"),
]


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_streams_decode_on_arrival_over_nvlink(tmp_path):
    out = tmp_path / "tr"
    cmd = ["timeout", "-k", "30", "280", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           str(ROOT / "tests" / "transport_worker.py"), str(out), "nccl", "5"]
    proc = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-3000:]
    results = [json.loads(Path(f"{out}.{r}").read_text()) for r in range(2)]
    assert all(r["ok"] for r in results), results
    assert all(r["errors"] == 0 for r in results)
