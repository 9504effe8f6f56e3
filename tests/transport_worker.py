"""One rank of a transport check, started through torchrun by
tests/test_multirank_gloo.py (CPU, gloo: the token order alone) and
tests/test_gpu_transport.py (GPUs, NCCL: streams over NVLink).

argv: output path, backend ("gloo" or "nccl"), steps.  Rank 0 sends to rank
1.  On gloo the ranks check that every ready token carries the sender's step
and every free token the receiver's.  On NCCL rank 0 encodes configs[0]-
sized layers (auto codec) into the transport's buffers and rank 1 decodes
them straight from rank 0's memory into its own cache, two slots in flight;
rank 1 checks every step bit for bit.  Each rank writes a JSON report to
<output>.<rank>."""

from __future__ import annotations

import datetime
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def gloo_tokens(steps: int, rank: int) -> dict:
    from unchainkv_b200.transport import TokenSchedule

    t = TokenSchedule(0, 1, rank)
    seen = []
    for k in range(steps):
        t.step(k)
        seen.append(t.received_step() if rank == 1 else (t.freed_step() if k > 0 else -1))
    t.finish()
    final = t.freed_step() if rank == 0 else -1
    if rank == 1:
        ok = seen == list(range(steps))
    else:
        ok = seen == [-1] + list(range(steps - 1)) and final == steps - 1
    return {"ok": ok, "seen": seen, "final": final}


def nccl_streams(steps: int, rank: int) -> dict:
    import numpy as np

    from unchainkv_b200 import splitzip_cuda as S
    from unchainkv_b200 import workloads as W
    from unchainkv_b200.transport import StreamTransport, peer_job

    device = torch.device("cuda", rank)
    layers, pool, blocks = 3, 96, 64
    n = 2 * blocks * 16 * 8 * 128
    cap = (S.auto_capacity(n) + 15) // 16 * 16
    tr = StreamTransport(layers * cap, sender=0, receiver=1)
    tables = torch.from_numpy(np.frombuffer(S.build_top16_tables(S._DEFAULT_TOP16_CODEBOOKS[:32]),
                                            np.uint8).copy()).to(device)
    src_ids = torch.as_tensor(W.block_table(pool, blocks, 3000), device=device)
    dst_ids = torch.as_tensor(W.block_table(pool, blocks, 3001), device=device)

    def layer_words(k, l):
        return W.draw_tokens(2000 + 7 * k + l, W.channel_scales(l), pool * 16).reshape(2, pool, 16, 8, 128)

    ok = True
    keep = []
    if rank == 0:
        kv = torch.empty((layers, 2, pool, 16, 8, 128), dtype=torch.bfloat16, device=device)
        for k in range(steps):
            base = tr.buffer(k)
            for l in range(layers):
                kv[l].copy_(torch.from_numpy(layer_words(k, l).view(np.int16)).view(torch.bfloat16))
            jobs = [peer_job(kv[l], src_ids, base + l * cap, cap, tables) for l in range(layers)]
            keep.append(jobs)
            if S.encode_auto_batch(jobs) is None:
                ok = False
            # the next step's inputs overwrite kv: wait for this encode first
            torch.cuda.current_stream().synchronize()
            tr.step(k)
    else:
        out = torch.zeros((layers, 2, pool, 16, 8, 128), dtype=torch.bfloat16, device=device)
        for k in range(steps):
            tr.step(k)
            base = tr.buffer(k)
            jobs = [peer_job(out[l], dst_ids, base + l * cap, cap, tables) for l in range(layers)]
            if S.decode_auto_batch(jobs) is None:
                ok = False
            torch.cuda.current_stream().synchronize()
            for l in range(layers):
                want = torch.from_numpy(layer_words(k, l).view(np.int16)).to(device)[:, src_ids.cpu()]
                if not torch.equal(out[l][:, dst_ids].view(torch.int16), want):
                    ok = False
    tr.finish()
    tr.close()
    return {"ok": ok, "errors": S.device_errors()}


def main() -> None:
    out, backend, steps = Path(sys.argv[1]), sys.argv[2], int(sys.argv[3])
    rank = int(os.environ["RANK"])
    if backend == "nccl":
        torch.cuda.set_device(rank)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
    else:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        report = gloo_tokens(steps, rank) if backend == "gloo" else nccl_streams(steps, rank)
    finally:
        dist.destroy_process_group()
    Path(f"{out}.{rank}").write_text(json.dumps(report))


if __name__ == "__main__":
    main()
