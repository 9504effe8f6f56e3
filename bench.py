#!/usr/bin/env python3
"""Benchmark of the B200 splitzip KV codec (encode + decode round trip).

Metric: codec GB/s of raw bf16 KV per GPU (encode, decode)
and % of HBM peak; ratio.

Headline workload (default, configs[1]): Llama-3-8B full prefill KV, 32
layers, one 4096-token prompt, 8 kv heads x 128, bf16, paged blocks of 16
tokens with a scattered block table, per-layer palettes.  The request's
tokens are the seeded numpy draw of the config's distribution (per-channel
scale log-uniform [0.01, 4], 2% outlier channels x50), the same bytes the
reference arm encodes on the host; the other pool blocks hold device draws.
One step = fused gather + encode of all 32 layers (device-chosen codec:
top16, else fixed6, else raw -- the reference's fallback chain) + decode +
scatter of all 32 streams into a second paged cache with another block
table.  Inputs (512 MiB raw per step) are larger than L2.  After the timed
loop every stream is compared byte for byte with the CPU oracle's.

The timed region is the driver's K-step loop, repeated R times (each
repeat bracketed by a barrier and a synchronize, max over ranks) until at
least --min-timed-ms of device time is covered; ms_per_step is the median
of the R per-step figures.

The default line also carries blocks for the other paths, each timed the
same way: `top16` (in-capacity top16 data, escapes exactly at the
capacity), `attention` (configs[4] decode attention over fixed6 and top16
streams), `tp8_shard` (configs[2]: rank r codes kv head r of the 70B TP=8
shard, 80 layers), `reference_api` (the reference's own Python wrapper and
per-layer call pattern driving this library) and, at N >= 2, `transfer`
(GPU -> GPU over NVLink, decode on arrival).

`value` = raw KV bytes per step / device time per step, summed over ranks
(whole job); `e2e` = the same through the public batch API with the stream
copied device->pinned host->device inside the timed region (the reference's
producer/consumer path, scripts/bench_codec_matrix.py:159-188).

--impl reference times the reference's CPU path (the CPU oracle's
multi-threaded restatement of the codec: top16 attempt -> fixed6 fallback ->
decode) on a bounded sample of the same bytes, with the same config keys.

Rank 0 writes exactly one JSON line to stdout; everything else (NCCL's INFO
lines included) goes to stderr.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

METRIC = "codec GB/s of raw bf16 KV per GPU (encode, decode) and % HBM peak; ratio"
REF_PACKAGE = ROOT / "baseline" / "_ref"
ATTN_TOP16_BOOKS = bytes(range(117, 133)) + bytes(range(118, 134))  # K, V exponents of the top16 attention streams


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--workload", choices=("c1", "c2", "c3", "c4", "top16", "calib", "modes", "writeback", "transfer"),
                   default="c1",
                   help="c1: configs[1] (default, with the other paths as blocks of its line); c2: configs[2] "
                        "per-GPU TP shard; c3: configs[3] mixed batch; c4: configs[4] decode attention over "
                        "compressed KV; top16: in-capacity top16 data; calib: GPU calibration over the configs[1] "
                        "cache; modes: receiver decode of the torch-op forms; writeback; transfer (N >= 2)")
    p.add_argument("--min-timed-ms", type=float, default=1000.0,
                   help="repeat the K-step loop until this much device time is timed (headline)")
    p.add_argument("--block-timed-ms", type=float, default=300.0, help="the same for each block of the line")
    p.add_argument("--no-blocks", action="store_true", help="c1 line without the other paths' blocks")
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--cpu-layers", type=int, default=2, help="layers in the CPU baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--skip-e2e", action="store_true")
    p.add_argument("--attn-streams", choices=("fixed6", "top16"), default="fixed6",
                   help="c4: the stream form attended (top16: book-drawn exponents with 0.3%% escapes, since "
                        "the configs[0] distribution overflows top16)")
    p.add_argument("--layers", type=int, default=None,
                   help="override the layer count (small ncu captures only; the bench line uses the config's)")
    return p.parse_args(argv)


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class JsonOut:
    """stdout carries exactly one JSON line.  Everything else the process
    prints, at the Python or the C level (NCCL's INFO lines, vLLM's logger,
    which the reference's connector imports), goes to stderr."""

    def __init__(self):
        sys.stdout.flush()
        self.fd = os.dup(1)
        os.dup2(2, 1)

    def emit(self, line: dict):
        os.write(self.fd, (json.dumps(line) + "\n").encode())


def host_threads() -> int:
    """Host threads this process may use (torchrun sets OMP_NUM_THREADS=1 for
    its ranks; the CPU legs pass their thread count explicitly instead)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def rounded(x, k=3):
    return None if x is None else round(float(x), k)


# ----------------------------------------------------------------- clocks


class ClockSampler:
    """SM clocks and clock-event reasons of the benchmark's GPUs, sampled every
    10 ms during the timed region through NVML (read-only queries); falls back
    to `nvidia-smi -lms 100` where NVML cannot be loaded."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices, period_s: float = 0.01):
        self.gpus = list(gpu_indices)
        self.period = period_s
        self.rows = []  # (sm_mhz, util_pct, set of reasons)
        self.max_mhz = None
        self.stop_flag = threading.Event()
        self.thread = None
        self.proc = None

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            handles = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in self.gpus]
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handles[0], pynvml.NVML_CLOCK_SM))
            masks = [(name, getattr(pynvml, const)) for name, const in self.REASONS]
        except Exception:  # no NVML: nvidia-smi
            self._start_smi()
            return self

        def poll():
            while not self.stop_flag.is_set():
                for h in handles:
                    try:
                        sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                        util = float(pynvml.nvmlDeviceGetUtilizationRates(h).gpu)
                        bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    except Exception:
                        continue
                    self.rows.append((sm, util, {name for name, m in masks if bits & m}))
                time.sleep(self.period)

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()
        return self

    def _start_smi(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        names = [name for name, _ in self.REASONS]

        def read():
            for line in self.proc.stdout:
                r = [x.strip() for x in line.split(",")]
                if len(r) < 10 or not r[0].isdigit() or int(r[0]) not in self.gpus:
                    continue
                try:
                    sm, util = float(r[1]), float(r[4])
                    self.max_mhz = float(r[2])
                except ValueError:
                    continue
                self.rows.append((sm, util, {n for n, v in zip(names, r[6:10]) if v.lower() == "active"}))

        self.thread = threading.Thread(target=read, daemon=True)
        self.thread.start()

    def stop(self):
        self.stop_flag.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        return self

    def summary(self):
        loaded = [r for r in self.rows if r[1] >= 30] or self.rows
        if not loaded:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"], "samples": 0}
        reasons = set()
        for r in loaded:
            reasons |= r[2]
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(loaded)}


# ------------------------------------------------------------- process


class Ctx:
    """One benchmark process (one GPU): rank, device, launch stream, the
    process group (NCCL, N > 1), timing helpers and the JSON output.

    stdout carries rank 0's one JSON line; everything else goes to stderr
    (JsonOut), NCCL's INFO lines included (they name the communicator's rank
    count)."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist

        self.out = JsonOut()
        self.args = args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.device = torch.device("cuda", self.local)
        self.dist = dist
        if self.world > 1:
            import datetime

            # NCCL's INFO lines (on stderr, see JsonOut) name each
            # communicator's rank count; a quieter level set by the image is
            # raised to INFO
            if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
                os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.device)
        from unchainkv_b200 import splitzip_cuda as S

        if not S.available():
            raise RuntimeError(f"splitzip library missing: {S.load_error()}")
        self.S = S
        self.lib = S._load()
        self.stream = torch.cuda.current_stream(self.device)
        self.sp = self.stream.cuda_stream
        self.torch = torch

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, value: float) -> float:
        from unchainkv_b200 import workloads as W

        return W.max_over_ranks(value)

    def sum(self, value: float) -> float:
        if self.world == 1:
            return value
        t = self.torch.tensor([value], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(t)
        return float(t.item())

    def timed(self, fn, steps: int) -> float:
        """Device ms of `steps` calls of fn on the launch stream, bracketed by
        a barrier and a synchronize, max over ranks."""
        torch = self.torch
        self.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(self.stream)
        for _ in range(steps):
            fn()
        end.record(self.stream)
        end.synchronize()
        ms = start.elapsed_time(end)
        self.barrier()
        return self.max(ms)

    def timed_repeats(self, fn, steps: int, warmup: int, min_ms: float):
        """W untimed calls, then the K-step loop R times until min_ms of device
        time is covered (R from the first loop's max-over-ranks time, so
        every rank runs the same R).  Returns (median ms per step, R, total
        timed ms)."""
        for _ in range(warmup):
            fn()
        first = self.timed(fn, steps)
        repeats = max(1, min(100000, math.ceil(min_ms / max(first, 1e-3))))
        per = [first / steps]
        for _ in range(repeats - 1):
            per.append(self.timed(fn, steps) / steps)
        return statistics.median(per), repeats, sum(per) * steps

    def timed_local(self, fn, steps: int, warmup: int, min_ms: float):
        """timed_repeats for work that one rank runs alone: no barrier and no
        collective."""
        torch = self.torch
        for _ in range(warmup):
            fn()
        per = []
        while not per or (sum(per) * steps < min_ms and len(per) < 100000):
            torch.cuda.synchronize()
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(self.stream)
            for _ in range(steps):
                fn()
            end.record(self.stream)
            end.synchronize()
            per.append(start.elapsed_time(end) / steps)
        return statistics.median(per), len(per), sum(per) * steps

    def profile(self, fn, steps: int):
        """Per-kernel device ms and launches of `steps` calls of fn (CUDA
        events around every launch of this library, on its launch stream)."""
        S = self.S
        S.profile_enable(True)
        for _ in range(steps):
            fn()
        prof = S.profile_collect()
        S.profile_enable(False)
        return prof

    def sampler(self):
        return ClockSampler(range(self.world)).start() if self.rank == 0 else None

    def emit(self, line: dict):
        if self.rank == 0:
            self.out.emit(line)

    def close(self):
        if self.world > 1 and self.dist.is_initialized():
            self.dist.barrier()
            self.dist.destroy_process_group()


def kernel_table(prof, alg: dict, prof_steps: int):
    """{kernel: launches, ms per launch, algorithmic bytes per launch, GB/s}
    from a profiler pass; alg holds algorithmic bytes per step."""
    kernels = {}
    for name, (ms, nl) in prof.items():
        per = ms / nl
        per_launch = alg[name] * prof_steps / nl if name in alg else None
        kernels[name] = {"launches": nl, "ms_per_launch": round(per, 5), "alg_bytes_per_launch": per_launch,
                         "gbs": round(per_launch / (per * 1e-3) / 1e9, 1) if per_launch else None}
    return kernels


def ncu_traffic(workload: str, kernel: str):
    """Per-launch DRAM bytes (read + write) of `kernel` on `workload` from the
    ncu launch list summarised in profiles/dram_traffic.txt, or None."""
    path = ROOT / "profiles" / "dram_traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) == 3 and not line.startswith("#") and parts[0] == workload and parts[1] == kernel:
            return int(parts[2])
    return None


def roofline_of(kernels: dict, kernel: str, workload: str):
    peak, peak_kind = peaks()
    dom = kernels[kernel]
    traffic = ncu_traffic(workload, kernel)
    return {"bound": "hbm", "kernel": kernel, "achieved": dom["gbs"], "peak": peak, "unit": "GB/s",
            "frac": round(dom["gbs"] / peak, 4) if dom["gbs"] else None, "peak_kind": peak_kind,
            "traffic": traffic,
            "traffic_source": "profiles/dram_traffic.txt (ncu dram__bytes_read.sum + dram__bytes_write.sum per "
                              "launch of the same workload)" if traffic else None,
            "alg_bytes_per_launch": dom["alg_bytes_per_launch"]}


# ------------------------------------------------------------- host data


def host_request_words(cfg, layers, shard: int, threads: int = 16):
    """The request tokens of every layer as the reference arm draws them
    (workloads.draw_tokens, numpy PCG64 seeds 2000 + layer + 100000 shard),
    [2, blocks, block_tokens, kv_heads, head_dim] uint16, and the layer's
    host-calibrated codebooks (32 bytes).  Drawn on host threads."""
    from unchainkv_b200 import workloads as W

    shape = (2, cfg.blocks, cfg.block_tokens, cfg.kv_heads, cfg.head_dim)

    def one(layer):
        scales = W.shard_scales(cfg, layer, shard)
        words = W.draw_tokens(2000 + layer + 100000 * shard, scales, cfg.tokens).reshape(shape)
        return words, W.shard_codebooks(cfg, layer, shard)

    with ThreadPoolExecutor(max(1, min(threads, os.cpu_count() or 1))) as ex:
        out = list(ex.map(one, layers))
    return [w for w, _ in out], [b for _, b in out]


def build_plan(ctx, cfg, L, shard=None):
    """Device caches, per-layer tables and the encode/decode jobs of one step.
    c1/c2: one request per layer, its tokens the host draw (host_words);
    c3: many requests per layer sharing the layer's paged pool, device
    draw.  Streams of all jobs sit in one transfer buffer at 16-byte aligned
    offsets."""
    import torch

    from unchainkv_b200 import splitzip_cuda as S
    from unchainkv_b200 import workloads as W

    device = ctx.device
    shard = ctx.rank if shard is None else shard
    mixed = isinstance(cfg, W.MixedConfig)
    if mixed:
        blocks = W.request_blocks(cfg, W.request_lengths(cfg))
        pool = int(sum(blocks) * cfg.pool_factor)
        src_ids = W.request_block_tables(pool, blocks, 3000)
        dst_ids = W.request_block_tables(pool, blocks, 3001)
    else:
        blocks = [cfg.blocks]
        pool = cfg.blocks * cfg.pool_factor
        src_ids = [W.block_table(pool, cfg.blocks, 3000)]
        dst_ids = [W.block_table(pool, cfg.blocks, 3001)]
    shape = (L, 2, pool, cfg.block_tokens, cfg.kv_heads, cfg.head_dim)
    src = torch.empty(shape, dtype=torch.bfloat16, device=device)
    dst = torch.zeros(shape, dtype=torch.bfloat16, device=device)
    src_t = [torch.as_tensor(x, device=device) for x in src_ids]
    dst_t = [torch.as_tensor(x, device=device) for x in dst_ids]
    host_words = None
    if mixed:
        books = b"".join(W.fill_pool_device(src[l], cfg, l, shard=shard) for l in range(L))
    else:
        host_words, book_list = host_request_words(cfg, range(L), shard)
        books = b"".join(book_list)
        for l in range(L):
            # the other pool blocks: independent device draws of the distribution
            filler = W.draw_tokens_device(5000 + l + 100000 * shard, W.shard_scales(cfg, l, shard),
                                          pool * cfg.block_tokens, device)
            src[l].copy_(filler.view(src[l].shape))
            req = torch.from_numpy(host_words[l].view(np.int16)).to(device).view(torch.bfloat16)
            src[l].index_copy_(1, src_t[0], req)
        del filler
    tables = torch.tensor(
        np.frombuffer(b"".join(S.build_top16_tables(books[l * 32:(l + 1) * 32]) for l in range(L)), np.uint8)
        .reshape(L, 544).copy(), device=device)
    jobs = []  # (layer, request, n, offset, capacity)
    offset = 0
    for l in range(L):
        for r, nb in enumerate(blocks):
            n = 2 * nb * cfg.block_words
            cap = (S.auto_capacity(n) + 15) // 16 * 16
            jobs.append((l, r, n, offset, cap))
            offset += cap
    streams = torch.zeros(offset, dtype=torch.uint8, device=device)
    enc = S.job_array([S.make_job(src[l], src_t[r], streams[o:o + c], c, tables[l]) for l, r, n, o, c in jobs])
    dec = S.job_array([S.make_job(dst[l], dst_t[r], streams[o:o + c], c, tables[l]) for l, r, n, o, c in jobs])
    return {"src": src, "dst": dst, "tables": tables, "jobs": jobs, "streams": streams, "enc": enc,
            "dec": dec, "src_t": src_t, "dst_t": dst_t, "src_ids": src_ids, "pool": pool, "blocks": blocks,
            "host_words": host_words, "raw_bytes": 2 * sum(n for _, _, n, _, _ in jobs), "shard": shard}


def check_round_trip(P, what):
    import torch

    for l in range(P["src"].shape[0]):
        for s_ids, d_ids in zip(P["src_t"], P["dst_t"]):
            if not torch.equal(P["dst"][l][:, d_ids].view(torch.int16), P["src"][l][:, s_ids].view(torch.int16)):
                raise RuntimeError(f"{what}: layer {l} round trip differs")


def stream_census(ctx, P):
    """Mode byte, stream length and top16 escape count of every job."""
    import torch

    S = ctx.S
    jobs = P["jobs"]
    offsets = torch.tensor([o for _, _, _, o, _ in jobs], device=ctx.device)
    modes = P["streams"][offsets].cpu().tolist()
    sizes = [S.stream_bytes(m, n) for m, (_, _, n, _, _) in zip(modes, jobs)]
    escapes = words = 0
    for l in range(P["src"].shape[0]):
        t = P["tables"][l]
        for s_ids in P["src_t"]:
            w = P["src"][l][:, s_ids].reshape(2, -1).view(torch.int16).to(torch.int32) & 0xFFFF
            e = (w >> 7) & 0xFF
            escapes += int((t[:256][e[0].long()] == 255).sum() + (t[256:512][e[1].long()] == 255).sum())
            words += w.numel()
    return modes, sizes, escapes, words


def oracle_parity(ctx, P, sizes, max_jobs=None):
    """Every (or the first max_jobs) job's timed stream against the CPU
    oracle's stream of the same words, byte for byte.  c1/c2: the oracle
    reads the host draw both arms use; c3: the request's words copied back
    from the device cache."""
    from oracle import oracle

    jobs = P["jobs"]
    pick = range(len(jobs)) if max_jobs is None else range(min(max_jobs, len(jobs)))
    host_streams = P["streams"].cpu().numpy()
    tables = P["tables"].cpu().numpy()
    checked = 0
    t0 = time.perf_counter()
    for i in pick:
        l, r, n, o, c = jobs[i]
        if P["host_words"] is not None:
            words = P["host_words"][l]
            ids = np.arange(words.shape[1], dtype=np.int64)
        else:
            import torch

            words = P["src"][l][:, P["src_t"][r]].view(torch.int16).cpu().numpy().view(np.uint16)
            ids = np.arange(words.shape[1], dtype=np.int64)
        expected = oracle.encode_auto_blocks(words, ids, tables[l], threads=host_threads())
        got = host_streams[o:o + len(expected)]
        if sizes[i] != len(expected) or not np.array_equal(got, expected):
            bad = np.flatnonzero(got != expected)[:4].tolist() if got.size == expected.size else "length"
            raise RuntimeError(f"job {i} (layer {l}, request {r}): GPU stream differs from the oracle at {bad}")
        checked += 1
    return {"jobs_checked": checked, "jobs": len(jobs), "bytes_equal": True,
            "bytes_checked": int(sum(sizes[i] for i in pick)),
            "checker": "CPU oracle (C restatement of kvq_splitzip_cuda.cu + the connector's fallback chain), "
                       + ("on the host draw the reference arm encodes" if P["host_words"] is not None
                          else "on the words copied back from the device cache"),
            "check_s": round(time.perf_counter() - t0, 2)}


# ------------------------------------------------------------ codec runs


def codec_run(ctx, cfg, L, min_ms, *, parity_jobs=None, e2e=True, cpu=True, clocks=True, workload="c1"):
    """Auto encode + decode round trip of a codec config on this rank's
    shard.  Returns the line's fields (value = whole-job GB/s)."""
    import torch

    S, lib, args = ctx.S, ctx.lib, ctx.args
    P = build_plan(ctx, cfg, L)
    jobs, streams, enc, dec = P["jobs"], P["streams"], P["enc"], P["dec"]
    J = len(jobs)
    sp = ctx.sp
    raw_bytes = P["raw_bytes"]

    def encode():
        if lib.kvq_splitzip_bf16_encode_auto_batch(enc, J, sp) <= 0:
            raise RuntimeError("encode declined: " + lib.kvq_splitzip_last_error().decode())

    def decode():
        if lib.kvq_splitzip_bf16_decode_auto_batch(dec, J, sp) <= 0:
            raise RuntimeError("decode declined: " + lib.kvq_splitzip_last_error().decode())

    def step():
        encode()
        decode()

    step()
    torch.cuda.synchronize()
    check_round_trip(P, "first step")
    modes, sizes, escapes, words = stream_census(ctx, P)
    encoded_total = sum(s for s in sizes if s)

    sampler = ctx.sampler() if clocks else None
    ms_step, repeats, timed_ms = ctx.timed_repeats(step, args.steps, args.warmup, min_ms)
    if sampler:
        sampler.stop()
    ms_enc, _, _ = ctx.timed_repeats(encode, args.steps, 1, min_ms / 4)
    ms_dec, _, _ = ctx.timed_repeats(decode, args.steps, 1, min_ms / 4)
    torch.cuda.synchronize()
    check_round_trip(P, "timed steps")
    parity = oracle_parity(ctx, P, sizes, parity_jobs)
    prof_steps = max(1, min(args.steps, 100))
    prof = ctx.profile(step, prof_steps)

    e2e_line = None
    if e2e and not args.skip_e2e:
        e2e_line = codec_e2e(ctx, P, encode)

    peak, peak_kind = peaks()
    alg_step = {"StatsKernel": raw_bytes, "EncodeAutoKernel": raw_bytes + encoded_total,
                "DecodeAutoKernel": encoded_total + raw_bytes, "ZeroKernel": 64 * J}
    kernels = kernel_table(prof, alg_step, prof_steps)
    dominant = max(prof.items(), key=lambda kv: kv[1][0])[0]
    launches_per_step = sum(nl for _, nl in prof.values()) / prof_steps
    alg_round_trip = sum(alg_step[k] for k in ("StatsKernel", "EncodeAutoKernel", "DecodeAutoKernel"))
    alg_encode = raw_bytes + encoded_total  # one read of the raw KV, the streams written
    enc_gbs = raw_bytes / (ms_enc * 1e-3) / 1e9
    dec_gbs = raw_bytes / (ms_dec * 1e-3) / 1e9
    cpu_line = None
    if cpu and not args.no_cpu_baseline and ctx.world == 1:  # rank 0 at N=1 only
        cpu_line = cpu_baseline(cfg, max(1, args.cpu_layers), shard=P["shard"])
    out = {
        "value": round(ctx.world * raw_bytes / (ms_step * 1e-3) / 1e9, 3),
        "ms_per_step": round(ms_step, 5),
        "repeats": repeats,
        "timed_ms": round(timed_ms, 1),
        "encode_gbs_per_gpu": round(enc_gbs, 2),
        "decode_gbs_per_gpu": round(dec_gbs, 2),
        "encode_hbm_frac": round(alg_encode / (ms_enc * 1e-3) / 1e9 / peak, 4),
        "decode_hbm_frac": round(alg_encode / (ms_dec * 1e-3) / 1e9 / peak, 4),
        "hbm_frac_round_trip": round(alg_round_trip / (ms_step * 1e-3) / 1e9 / peak, 4),
        "ratio": round(raw_bytes / encoded_total, 4),
        "escape_rate": round(escapes / words, 5),
        "modes": {str(m): modes.count(m) for m in sorted(set(modes))},
        "parity": parity,
        "roofline": roofline_of(kernels, dominant, workload),
        "kernels": kernels,
        "gpu_launches": int(round(launches_per_step * args.steps * repeats)),
        "clocks": sampler.summary() if sampler else None,
        "cpu_baseline": cpu_line,
        "e2e": e2e_line,
        "_plan": {"jobs": J, "pool": P["pool"], "blocks": P["blocks"], "raw_bytes": raw_bytes,
                  "encoded": encoded_total, "layers": L},
    }
    del P
    torch.cuda.empty_cache()
    return out


def codec_e2e(ctx, P, encode):
    """The same round trip through the public batch API with host buffers:
    encode -> mode bytes -> exact D2H into pinned host -> H2D into receive
    buffers -> decode, the copies inside the timed region.

    Steps run as a two-slot pipeline, as a sender and a receiver would: step
    i+1's encode and its mode-byte read run while step i's copies are on the
    wire, and every step still copies its own streams down and up (the
    copies of a step are exact: each job's stream length from its mode
    byte).  Slot s has its own device streams, pinned host buffer and
    receive buffer; events keep a slot from being reused before its last
    reader is done.  The encodes run on the launch stream, the decodes on a
    second stream; the timed region (events on the launch stream, barrier
    and synchronize on both sides, max over ranks) ends after the last
    decode."""
    import torch

    S, lib, args = ctx.S, ctx.lib, ctx.args
    jobs = P["jobs"]
    J = len(jobs)
    offsets = torch.tensor([o for _, _, _, o, _ in jobs], device=ctx.device)
    streams = [P["streams"], torch.zeros_like(P["streams"])]
    encs = [P["enc"], S.job_array([S.make_job(P["src"][l], P["src_t"][r], streams[1][o:o + c], c, P["tables"][l])
                                   for l, r, n, o, c in jobs])]
    recv = [torch.zeros_like(P["streams"]) for _ in range(2)]
    host = [torch.empty(P["streams"].numel(), dtype=torch.uint8, pin_memory=True) for _ in range(2)]
    mode_host = torch.empty((J,), dtype=torch.uint8, pin_memory=True)
    decs = [S.job_array([S.make_job(P["dst"][l], P["dst_t"][r], recv[k][o:o + c], c, P["tables"][l])
                         for l, r, n, o, c in jobs]) for k in range(2)]
    d2h = torch.cuda.Stream(ctx.device)
    h2d = torch.cuda.Stream(ctx.device)
    dec = torch.cuda.Stream(ctx.device)
    stream = ctx.stream
    moved = {}
    state = {"step": 0, "d2h_done": [None, None], "h2d_done": [None, None], "decoded": [None, None]}

    def e2e_step():
        k = state["step"] & 1
        state["step"] += 1
        # the slot's streams are free once the D2H of its previous step is done
        if state["d2h_done"][k] is not None:
            stream.wait_event(state["d2h_done"][k])
        if lib.kvq_splitzip_bf16_encode_auto_batch(encs[k], J, ctx.sp) <= 0:
            raise RuntimeError("encode declined: " + lib.kvq_splitzip_last_error().decode())
        mode_host.copy_(streams[k][offsets], non_blocking=True)
        encoded = torch.cuda.Event()
        encoded.record(stream)
        encoded.synchronize()  # the host needs the modes for exact lengths
        lengths = [S.stream_bytes(int(m), n) for m, (_, _, n, _, _) in zip(mode_host.tolist(), jobs)]
        if any(x is None for x in lengths):
            raise RuntimeError("a job produced no stream (mode 255)")
        d2h.wait_event(encoded)
        if state["h2d_done"][k] is not None:
            d2h.wait_event(state["h2d_done"][k])  # the host slot's last H2D read it
        if state["decoded"][k] is not None:
            h2d.wait_event(state["decoded"][k])  # the receive slot's last decode read it
        last = None
        for (l, r, n, o, c), size in zip(jobs, lengths):
            with torch.cuda.stream(d2h):
                host[k][o:o + size].copy_(streams[k][o:o + size], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(d2h)
            h2d.wait_event(ev)
            with torch.cuda.stream(h2d):
                recv[k][o:o + size].copy_(host[k][o:o + size], non_blocking=True)
                last = torch.cuda.Event()
                last.record(h2d)
        state["d2h_done"][k] = ev
        state["h2d_done"][k] = last
        dec.wait_event(last)
        if lib.kvq_splitzip_bf16_decode_auto_batch(decs[k], J, dec.cuda_stream) <= 0:
            raise RuntimeError("decode declined: " + lib.kvq_splitzip_last_error().decode())
        decoded = torch.cuda.Event()
        decoded.record(dec)
        state["decoded"][k] = decoded
        state["last_decoded"] = decoded
        moved["d2h"] = sum(lengths) + J
        moved["h2d"] = sum(lengths)

    def e2e_timed(steps):
        ctx.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            e2e_step()
        stream.wait_event(state["last_decoded"])
        end.record(stream)
        end.synchronize()
        ms = start.elapsed_time(end)
        ctx.barrier()
        return ctx.max(ms)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_ms = e2e_timed(args.e2e_steps) / args.e2e_steps
    wall_ms = (time.perf_counter() - t0) * 1e3 / args.e2e_steps
    check_round_trip(P, "e2e")
    return {"value": round(ctx.world * P["raw_bytes"] / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
            "h2d_bytes_per_step": moved["h2d"], "d2h_bytes_per_step": moved["d2h"],
            "ms_per_step": round(e2e_ms, 4), "wall_ms_per_step": round(wall_ms, 4),
            "path": "encode_auto_batch -> D2H pinned -> H2D -> decode_auto_batch, two steps in flight"}


def codec_config(cfg, plan, world):
    from unchainkv_b200 import workloads as W

    if isinstance(cfg, W.MixedConfig):
        shape_cfg = {"requests": cfg.requests, "tokens_per_layer": int(sum(plan["blocks"]) * cfg.block_tokens),
                     "request_tokens": [cfg.min_tokens, cfg.max_tokens], "scale_shift": cfg.scale_shift,
                     "model_layers": cfg.model_layers}
    else:
        shape_cfg = {"tokens": cfg.tokens}
    return {"workload": cfg.name, "layers": plan["layers"], **shape_cfg, "kv_heads": cfg.kv_heads,
            "head_dim": cfg.head_dim, "block_tokens": cfg.block_tokens, "pool_blocks": plan["pool"],
            "jobs_per_step": plan["jobs"], "raw_bytes_per_step": plan["raw_bytes"],
            "encoded_bytes_per_step": plan["encoded"],
            "policy": "device-chosen codec per job (top16 -> fixed6 -> raw)",
            "l2": f"inputs larger than L2 (raw KV per step {plan['raw_bytes'] / 2**20:.0f} MiB, L2 126 MB)",
            "parallelism": f"independent per-GPU shards x{world} (no collective)"}


def codec_line(ctx, cfg, r, data):
    plan = r.pop("_plan")
    line = {"metric": METRIC, "value": r.pop("value"), "unit": "GB/s", "n_gpus": ctx.world,
            "steps": ctx.args.steps, "warmup": ctx.args.warmup, "ms_per_step": r.pop("ms_per_step"),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u16", "data": data,
            "config": codec_config(cfg, plan, ctx.world)}
    line.update(r)
    return line


# ------------------------------------------------------------ top16 block


def top16_layer_words(ctx, cfg, layer: int, books: bytes, every: int = 200):
    """[2, blocks, bt, kvh, hd] words of one in-capacity top16 layer (device):
    random signs and mantissas, exponents uniform over the plane's 16-entry
    book, and an escaped exponent on exactly every `every`-th word -- the
    escape pattern of the reference's codec benchmark
    (scripts/bench_codec_matrix.py:108-111), so escapes == capacity."""
    import torch

    shape = (2, cfg.blocks, cfg.block_tokens, cfg.kv_heads, cfg.head_dim)
    gen = torch.Generator(device=ctx.device)
    gen.manual_seed(8000 + layer + 100000 * ctx.rank)
    book = torch.tensor(list(books), dtype=torch.int32, device=ctx.device).view(2, 16)
    code = torch.randint(0, 16, shape, generator=gen, device=ctx.device)
    exp = torch.stack([book[p][code[p]] for p in range(2)])
    flat = exp.view(-1)
    escape = next(v for v in range(1, 255) if v not in books)
    flat[::every] = escape
    sign = torch.randint(0, 2, shape, generator=gen, device=ctx.device, dtype=torch.int32)
    mant = torch.randint(0, 128, shape, generator=gen, device=ctx.device, dtype=torch.int32)
    return ((sign << 15) | (exp << 7) | mant).to(torch.int16).view(torch.bfloat16)


def top16_run(ctx, min_ms, L=None):
    """configs[1]-shaped layers of in-capacity top16 data: the reference-ABI
    top16 encode (fused gather, stream buffers of exactly the reference's
    capacity) + top16 decode, and the device-chosen auto codec on the same
    data.  Sampled streams checked against the oracle."""
    import torch

    from oracle import oracle
    from unchainkv_b200 import workloads as W

    S, lib, args = ctx.S, ctx.lib, ctx.args
    cfg = W.CONFIGS["c1"]
    L = L or args.layers or cfg.layers
    pool = cfg.blocks * cfg.pool_factor
    ids = W.block_table(pool, cfg.blocks, 3000)
    ids2 = W.block_table(pool, cfg.blocks, 3001)
    ids_t, ids2_t = torch.as_tensor(ids, device=ctx.device), torch.as_tensor(ids2, device=ctx.device)
    shape = (2, pool, cfg.block_tokens, cfg.kv_heads, cfg.head_dim)
    src = torch.zeros((L,) + shape, dtype=torch.bfloat16, device=ctx.device)
    dst = torch.zeros_like(src)
    books = [W.shard_codebooks(cfg, l, ctx.rank) for l in range(L)]
    for l in range(L):
        src[l].index_copy_(1, ids_t, top16_layer_words(ctx, cfg, l, books[l]))
    tables = torch.tensor(np.frombuffer(b"".join(S.build_top16_tables(b) for b in books), np.uint8)
                          .reshape(L, 544).copy(), device=ctx.device)
    n = cfg.words_per_layer
    tight = S.top16_capacity(n)
    cap_t = (tight + 15) // 16 * 16
    cap_a = (S.auto_capacity(n) + 15) // 16 * 16
    bufs_t = torch.zeros(L * cap_t, dtype=torch.uint8, device=ctx.device)
    bufs_a = torch.zeros(L * cap_a, dtype=torch.uint8, device=ctx.device)
    enc_t = S.job_array([S.make_job(src[l], ids_t, bufs_t[l * cap_t:l * cap_t + tight], tight, tables[l])
                         for l in range(L)])
    size = S.top16_stream_bytes(n)
    dec_t = S.job_array([S.make_job(dst[l], ids2_t, bufs_t[l * cap_t:l * cap_t + size], size, tables[l])
                         for l in range(L)])
    enc_a = S.job_array([S.make_job(src[l], ids_t, bufs_a[l * cap_a:(l + 1) * cap_a], cap_a, tables[l])
                         for l in range(L)])
    dec_a = S.job_array([S.make_job(dst[l], ids2_t, bufs_a[l * cap_a:(l + 1) * cap_a], cap_a, tables[l])
                         for l in range(L)])
    sp = ctx.sp

    def call(name, jobs):
        if getattr(lib, name)(jobs, L, sp) <= 0:
            raise RuntimeError(f"{name} declined: " + lib.kvq_splitzip_last_error().decode())

    fns = {"encode_top16": lambda: call("kvq_splitzip_bf16_encode_top16_batch", enc_t),
           "decode_top16": lambda: call("kvq_splitzip_bf16_decode_top16_batch", dec_t),
           "encode_auto": lambda: call("kvq_splitzip_bf16_encode_auto_batch", enc_a),
           "decode_auto": lambda: call("kvq_splitzip_bf16_decode_auto_batch", dec_a)}
    raw = 2 * n * L
    out = {"data": "configs[1] shape, exponents uniform over each layer's book, one escape on every 200th word "
                   "(escapes == capacity, scripts/bench_codec_matrix.py:108-111), random signs and mantissas",
           "layers": L, "raw_bytes_per_step": raw, "stream_bytes_per_step": size * L,
           "ratio": round(raw / (size * L), 4), "capacity_bytes": tight}
    peak, _ = peaks()
    sampler = ctx.sampler()
    for path, (e, d) in {"reference_abi": ("encode_top16", "decode_top16"),
                         "auto": ("encode_auto", "decode_auto")}.items():
        fns[e]()
        fns[d]()
        torch.cuda.synchronize()
        bufs = bufs_t if path == "reference_abi" else bufs_a
        cap = cap_t if path == "reference_abi" else cap_a
        heads = bufs.view(L, cap)[:, 0].cpu().tolist()
        if any(h != 5 for h in heads):
            raise RuntimeError(f"top16 block ({path}): modes {sorted(set(heads))}, expected 5")
        for l in range(L):
            if not torch.equal(dst[l][:, ids2_t].view(torch.int16), src[l][:, ids_t].view(torch.int16)):
                raise RuntimeError(f"top16 block ({path}): layer {l} round trip differs")
        for l in (0, L - 1):  # streams against the oracle
            words = src[l][:, ids_t].view(torch.int16).cpu().numpy().view(np.uint16)
            exp_res, exp = oracle.encode_top16_blocks(words, np.arange(cfg.blocks), tables[l].cpu().numpy(),
                                                      capacity=tight)
            got = bufs[l * cap:l * cap + size].cpu().numpy()
            if exp_res != size or not np.array_equal(got, exp):
                raise RuntimeError(f"top16 block ({path}): layer {l} stream differs from the oracle")
        ms_e, rep_e, _ = ctx.timed_repeats(fns[e], args.steps, args.warmup, min_ms / 2)
        ms_d, rep_d, _ = ctx.timed_repeats(fns[d], args.steps, args.warmup, min_ms / 2)
        prof_steps = max(1, min(args.steps, 50))
        prof = ctx.profile(lambda: (fns[e](), fns[d]()), prof_steps)
        alg = {"Top16StatsKernel": raw, "EncodeTop16Kernel": raw + size * L,
               "Top16ScanKernel": 52 * L * ((n + S.TILE_WORDS - 1) // S.TILE_WORDS),  # 32-byte records read, 20 bytes written
               "StatsKernel": raw, "EncodeAutoKernel": raw + size * L,
               "DecodeTop16Kernel": size * L + raw, "DecodeAutoKernel": size * L + raw,
               "EscapePatchKernel": 8 * L * (n // 200)}
        kernels = kernel_table(prof, alg, prof_steps)
        for k in kernels.values():
            if k["gbs"]:
                k["hbm_frac"] = round(k["gbs"] / peak, 4)
        alg_enc = raw + size * L
        out[path] = {"encode_gbs_per_gpu": round(raw / (ms_e * 1e-3) / 1e9, 2),
                     "decode_gbs_per_gpu": round(raw / (ms_d * 1e-3) / 1e9, 2),
                     "encode_hbm_frac": round(alg_enc / (ms_e * 1e-3) / 1e9 / peak, 4),
                     "decode_hbm_frac": round(alg_enc / (ms_d * 1e-3) / 1e9 / peak, 4),
                     "ms_encode": round(ms_e, 5), "ms_decode": round(ms_d, 5), "repeats": [rep_e, rep_d],
                     "kernels": kernels,
                     "parity": {"jobs_checked": 2, "bytes_equal": True, "modes": {"5": L}}}
    if sampler:
        sampler.stop()
        out["clocks"] = sampler.summary()
    del src, dst, bufs_t, bufs_a
    torch.cuda.empty_cache()
    return out


# --------------------------------------------------------- attention


def attention_top16_stream(cfg, blocks, r, shard, table, device):
    """A top16 stream of one request's K/V: exponents drawn from the plane's
    16-entry book, 0.3% escapes (exponents 105 and 135), random signs and
    mantissas; encoded by the library, placed so that its planes sit on
    16-byte boundaries."""
    import torch

    from unchainkv_b200 import splitzip_cuda as S

    gen = torch.Generator(device=device)
    gen.manual_seed(7000 + r + 100000 * shard)
    shape = (2, blocks, cfg.block_tokens, cfg.kv_heads, cfg.head_dim)
    books = torch.tensor(list(ATTN_TOP16_BOOKS), dtype=torch.int32, device=device).view(2, 1, 1, 1, 1, 16)
    code = torch.randint(0, 16, shape + (1,), generator=gen, device=device)
    exp = torch.gather(books.expand(shape + (16,)), -1, code).squeeze(-1)
    esc = torch.rand(shape, generator=gen, device=device) < 0.003
    big = torch.rand(shape, generator=gen, device=device) < 0.5
    exp = torch.where(esc, torch.where(big, 135, 105), exp)
    sign = torch.randint(0, 2, shape, generator=gen, device=device, dtype=torch.int32)
    mant = torch.randint(0, 128, shape, generator=gen, device=device, dtype=torch.int32)
    words = ((sign << 15) | (exp << 7) | mant).to(torch.int16).view(torch.bfloat16).contiguous()
    n = words.numel()
    buf = torch.zeros(S.top16_capacity(n) + 16, dtype=torch.uint8, device=device)
    if not S.encode_top16_batch([S.make_job(words, None, buf, None, table, block_start=0, block_count=blocks)]):
        raise RuntimeError("top16 encode declined: " + S._load().kvq_splitzip_last_error().decode())
    torch.cuda.synchronize()
    if int(buf[0].item()) != 5:
        raise RuntimeError("the top16 attention data did not give a top16 stream")
    size = S.stream_bytes(5, n)
    raw = torch.empty(size + 32, dtype=torch.uint8, device=device)
    start = (11 - raw.data_ptr()) % 16  # body and nibble planes on 16-byte boundaries
    stream = raw[start:start + size]
    stream.copy_(buf[:size])
    return stream


def attention_inputs(cfg, device, shard, codec="fixed6"):
    """per request a stream of its one-layer K/V placed on a
    plane boundary, contexts, a bf16 N(0,1) query batch and the per-request
    tables (None for fixed6).  fixed6: device draw of the configs[0]
    distribution, encoded by the library; top16: see
    attention_top16_stream."""
    import torch

    from unchainkv_b200 import splitzip_cuda as S
    from unchainkv_b200 import workloads as W

    ctxs = W.attention_contexts(cfg)
    zero_tables = torch.zeros(544, dtype=torch.uint8, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(4005 + shard)
    q = torch.randn((cfg.requests, cfg.kv_heads * cfg.group, cfg.head_dim), generator=gen, device=device)
    if codec == "top16":
        table = torch.frombuffer(bytearray(S.build_top16_tables(ATTN_TOP16_BOOKS)), dtype=torch.uint8).to(device)
        streams = [attention_top16_stream(cfg, -(-ctx // cfg.block_tokens), r, shard, table, device)
                   for r, ctx in enumerate(ctxs)]
        return ctxs, streams, q.to(torch.bfloat16), [table] * len(ctxs)
    streams = []
    for r, ctx in enumerate(ctxs):
        blocks = -(-ctx // cfg.block_tokens)
        scales = W.channel_scales(r % 32, cfg.kv_heads, cfg.head_dim)
        kv = W.draw_tokens_device(2000 + r + 100000 * shard, scales, blocks * cfg.block_tokens, device)
        kv = kv.view(2, blocks, cfg.block_tokens, cfg.kv_heads, cfg.head_dim).contiguous()
        n = kv.numel()
        buf = torch.zeros(S.auto_capacity(n), dtype=torch.uint8, device=device)
        job = S.make_job(kv, None, buf, None, zero_tables, block_start=0, block_count=blocks)
        if not S.encode_bf16_batch([job], 6):
            raise RuntimeError("fixed6 encode declined: " + S._load().kvq_splitzip_last_error().decode())
        torch.cuda.synchronize()
        if int(buf[0].item()) != 3:
            raise RuntimeError("configs[4] data did not give a fixed6 stream")
        size = S.stream_bytes(3, n)
        stream = S.attention_stream_buffer(size, device)
        stream.copy_(buf[:size])
        streams.append(stream)
    return ctxs, streams, q.to(torch.bfloat16), None


def attention_errors(cfg, ctxs, streams, q, out, tables=None):
    """Every request against fp32 attention over its stream decoded by the
    codec (decompress then attend, the reference's path,
    scripts/bench_codec_attention.py:150-157).  Raises above 2e-2 relative /
    1e-3 absolute; returns the largest absolute and relative errors."""
    import torch

    from unchainkv_b200 import splitzip_cuda as S

    worst_abs = worst_ratio = 0.0
    for r in range(len(ctxs)):
        blocks = -(-ctxs[r] // cfg.block_tokens)
        kv = torch.zeros((2, blocks, cfg.block_tokens, cfg.kv_heads, cfg.head_dim), dtype=torch.bfloat16,
                         device=q.device)
        table = tables[r] if tables is not None else torch.zeros(544, dtype=torch.uint8, device=q.device)
        job = S.make_job(kv, None, streams[r], streams[r].numel(), table, block_start=0, block_count=blocks)
        if not S.decode_auto_batch([job]):
            raise RuntimeError("reference decode declined")
        k = kv[0].reshape(-1, cfg.kv_heads, cfg.head_dim)[: ctxs[r]].float()
        v = kv[1].reshape(-1, cfg.kv_heads, cfg.head_dim)[: ctxs[r]].float()
        qf = q[r].float().view(cfg.kv_heads, cfg.group, cfg.head_dim)
        s = torch.einsum("hgd,thd->hgt", qf, k) / cfg.head_dim ** 0.5
        ref = torch.einsum("hgt,thd->hgd", torch.softmax(s, dim=-1), v).reshape(-1, cfg.head_dim)
        diff = (out[r].float() - ref).abs()
        allowed = 1e-3 + 2e-2 * ref.abs()
        bad = diff > allowed
        if bool(bad.any()):
            raise RuntimeError(f"request {r}: attention differs from fp32 decompress-then-attend at "
                               f"{int(bad.sum())} values")
        worst_abs = max(worst_abs, float(diff.max()))
        worst_ratio = max(worst_ratio, float((diff / allowed).max()))
    return worst_abs, worst_ratio


def attention_cpu_gbs(cfg, requests: int = 2, repeats: int = 3):
    """Decompress-then-attend on host cores: the CPU oracle decodes each
    request's fixed6 stream, numpy attends in fp32.  Returns (GB/s of raw KV
    attended, threads, sample)."""
    from oracle import oracle
    from unchainkv_b200 import workloads as W

    ctxs = W.attention_contexts(cfg)[:requests]
    jobs = []
    for r, ctx in enumerate(ctxs):
        blocks = -(-ctx // cfg.block_tokens)
        words = W.draw_tokens(2000 + r, W.channel_scales(r % 32, cfg.kv_heads, cfg.head_dim), blocks * cfg.block_tokens)
        res, stream = oracle.encode_mode(words.reshape(-1), bits=6)
        jobs.append((ctx, blocks, stream[:res]))
    rng = np.random.Generator(np.random.PCG64(4005))
    q = rng.standard_normal((requests, cfg.kv_heads, cfg.group, cfg.head_dim)).astype(np.float32)

    threads = host_threads()
    lib = oracle.lib()

    def run():
        for r, (ctx, blocks, stream) in enumerate(jobs):
            cache = np.zeros((2, blocks, cfg.block_tokens, cfg.kv_heads, cfg.head_dim), np.uint16)
            bw = cfg.block_tokens * cfg.kv_heads * cfg.head_dim
            ids = np.arange(blocks, dtype=np.int64)
            lib.orc_decode_fixed6_blocks_mt(stream.ctypes.data, stream.size, cache.ctypes.data, 2 * blocks * bw,
                                            blocks, bw, blocks * bw, bw, 0, ids.ctypes.data, threads)
            kv = (cache.astype(np.uint32) << 16).view(np.float32).reshape(2, -1, cfg.kv_heads, cfg.head_dim)[:, :ctx]
            s = np.einsum("hgd,thd->hgt", q[r], kv[0]) / np.sqrt(cfg.head_dim)
            s -= s.max(axis=-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=-1, keepdims=True)
            np.einsum("hgt,thd->hgd", p, kv[1])

    run()
    times = []
    for _ in range(repeats):
        t = time.perf_counter()
        run()
        times.append(time.perf_counter() - t)
    raw = sum(4 * ctx * cfg.kv_heads * cfg.head_dim for ctx, _, _ in jobs)
    return (raw / statistics.median(times) / 1e9, threads,
            f"first {requests} of {cfg.requests} requests (oracle decode on {threads} threads, numpy attention)")


def attention_run(ctx, codec, min_ms, e2e=True, cpu=True, clocks=True):
    """configs[4] decode attention over `codec` streams.  Returns the line's
    fields."""
    import torch

    from unchainkv_b200 import workloads as W

    S, lib, args = ctx.S, ctx.lib, ctx.args
    cfg = W.CONFIGS["c4"]
    ctxs, streams, q, tables = attention_inputs(cfg, ctx.device, ctx.rank, codec)
    out = torch.empty_like(q)
    reqs = S.attention_requests(q, streams, ctxs, out, tables)
    ws = torch.empty(lib.kvq_splitzip_attention_workspace_bytes(reqs, len(ctxs), cfg.group), dtype=torch.uint8,
                     device=ctx.device)

    def step():
        if S.attention_decode(q, streams, ctxs, out, workspace=ws, tables=tables) != len(ctxs):
            raise RuntimeError("attention declined: " + lib.kvq_splitzip_last_error().decode())

    step()
    torch.cuda.synchronize()
    worst_abs, worst_ratio = attention_errors(cfg, ctxs, streams, q, out, tables)
    sampler = ctx.sampler() if clocks else None
    ms_step, repeats, timed_ms = ctx.timed_repeats(step, args.steps, args.warmup, min_ms)
    if sampler:
        sampler.stop()
    prof_steps = max(1, min(args.steps, 100))
    prof = ctx.profile(step, prof_steps)
    raw = sum(4 * c * cfg.kv_heads * cfg.head_dim for c in ctxs)
    stream_bytes = sum(x.numel() for x in streams)
    qo = 2 * q.numel() * 2
    kernels = kernel_table(prof, {"AttnKernel": stream_bytes + qo}, prof_steps)
    e2e_line = None
    if e2e and not args.skip_e2e:
        q_host = q.cpu().pin_memory()
        out_host = torch.empty_like(q_host).pin_memory()

        def e2e_step():
            q.copy_(q_host, non_blocking=True)
            step()
            out_host.copy_(out, non_blocking=True)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        e2e_ms = ctx.timed(e2e_step, args.e2e_steps) / args.e2e_steps
        e2e_line = {"value": round(ctx.world * raw / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": q.numel() * 2, "d2h_bytes_per_step": out.numel() * 2,
                    "ms_per_step": round(e2e_ms, 4), "path": "pinned q -> attention_decode -> pinned out"}
    cpu_line = None
    if cpu and not args.no_cpu_baseline and ctx.world == 1:
        gbs, threads, sample = attention_cpu_gbs(cfg)
        cpu_line = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                    "sample": sample + ", oracle fixed6 decode then numpy fp32 attention", "cpu": cpu_model()}
    roof = roofline_of(kernels, "AttnKernel", "c4" if codec == "fixed6" else "c4_top16")
    return {
        "value": round(ctx.world * raw / (ms_step * 1e-3) / 1e9, 3),
        "ms_per_step": round(ms_step, 5), "repeats": repeats, "timed_ms": round(timed_ms, 1),
        "max_abs_err_vs_fp32": worst_abs, "max_err_over_tolerance": round(worst_ratio, 4),
        "tolerance": "|out - ref| <= 1e-3 + 2e-2 |ref| vs fp32 decompress-then-attend, every request",
        "roofline": roof, "kernels": kernels,
        "gpu_launches": int(round(sum(nl for _, nl in prof.values()) / prof_steps * args.steps * repeats)),
        "clocks": sampler.summary() if sampler else None, "cpu_baseline": cpu_line, "e2e": e2e_line,
        "_cfg": {"workload": cfg.name, "streams": codec, "requests": cfg.requests,
                 "q_heads": cfg.kv_heads * cfg.group, "kv_heads": cfg.kv_heads, "head_dim": cfg.head_dim,
                 "block_tokens": cfg.block_tokens, "context_tokens": [cfg.min_tokens, cfg.max_tokens],
                 "tokens_per_step": sum(ctxs), "stream_bytes_per_step": stream_bytes, "raw_kv_bytes_per_step": raw,
                 "l2": "compressed KV per step larger than L2",
                 "parallelism": f"independent per-GPU batches x{ctx.world} (no collective)"},
    }


# ------------------------------------------------- reference wrapper block


def reference_api_run(ctx, min_ms, L=32):
    """The reference's own Python wrapper (unchain_kv.splitzip_cuda, installed
    unchanged in baseline/_ref) driving this library through
    UNCHAIN_KV_SPLITZIP_LIB, in the per-layer call pattern of the
    reference's codec benchmark (scripts/bench_codec_matrix.py:104-188):
    gather the layer's blocks with index_select, encode_top16, copy the
    stream to pinned host and back, decode_top16 into the paged cache.  On
    configs[1]-shaped in-capacity top16 layers; device-only time (pack +
    encode + decode) and with the host copies, next to this library's own
    batched fused path on the same data."""
    import importlib

    import torch

    from unchainkv_b200 import workloads as W

    if not (REF_PACKAGE / "unchain_kv" / "splitzip_cuda.py").exists():
        return {"unavailable": "reference package not installed in baseline/_ref"}
    os.environ["UNCHAIN_KV_SPLITZIP_LIB"] = str(ctx.S.library_path())
    if str(REF_PACKAGE) not in sys.path:
        sys.path.insert(0, str(REF_PACKAGE))
    ref = importlib.import_module("unchain_kv.splitzip_cuda")
    if not ref.available():
        return {"unavailable": f"reference wrapper does not load this library: {ref.load_error()}"}
    args = ctx.args
    cfg = W.CONFIGS["c1"]
    layers = min(L, len(ref._TOP16_CODEBOOKS) // 32)
    pool = cfg.blocks * cfg.pool_factor
    ids = W.block_table(pool, cfg.blocks, 3000)
    ids_list = [int(i) for i in ids]
    ids_t = torch.as_tensor(ids, device=ctx.device)
    bw = cfg.block_words
    cache = torch.zeros((layers, 2, pool, bw), dtype=torch.bfloat16, device=ctx.device)
    target = torch.zeros((2, pool, bw), dtype=torch.bfloat16, device=ctx.device)
    pack = torch.empty((2, cfg.blocks, bw), dtype=torch.bfloat16, device=ctx.device)
    raw_bytes = pack.numel() * 2
    encoded = torch.empty(raw_bytes + 1, dtype=torch.uint8, device=ctx.device)
    received = torch.empty_like(encoded)
    host = torch.empty(raw_bytes + 1, dtype=torch.uint8, pin_memory=True)
    for l in range(layers):
        books = ref._TOP16_CODEBOOKS[l * 32:(l + 1) * 32]
        cache[l].index_copy_(1, ids_t, top16_layer_words(ctx, cfg, l, books).view(2, cfg.blocks, bw))
    size = ctx.S.top16_stream_bytes(2 * cfg.blocks * bw)

    def device_step():
        for l in range(layers):
            torch.index_select(cache[l], 1, ids_t, out=pack)
            res = ref.encode_top16(pack, encoded, l)
            if res != size:
                raise RuntimeError(f"reference wrapper encode_top16 returned {res}")
            if ref.decode_top16(encoded[:size], target, ids_list, raw_bytes, l) != raw_bytes:
                raise RuntimeError("reference wrapper decode_top16 declined")

    def host_step():
        for l in range(layers):
            torch.index_select(cache[l], 1, ids_t, out=pack)
            if ref.encode_top16(pack, encoded, l) != size:
                raise RuntimeError("reference wrapper encode_top16 declined")
            host[:size].copy_(encoded[:size], non_blocking=True)
            received[:size].copy_(host[:size], non_blocking=True)
            if ref.decode_top16(received[:size], target, ids_list, raw_bytes, l) != raw_bytes:
                raise RuntimeError("reference wrapper decode_top16 declined")

    device_step()
    torch.cuda.synchronize()
    if int(encoded[0].item()) != 5 or not torch.equal(target[:, ids_t].view(torch.int16),
                                                      cache[layers - 1][:, ids_t].view(torch.int16)):
        raise RuntimeError("reference wrapper round trip differs")
    steps = max(1, args.steps // 10)
    ms_dev, rep_dev, _ = ctx.timed_local(device_step, steps, 2, min_ms / 2)
    ms_host, rep_host, _ = ctx.timed_local(host_step, steps, 2, min_ms / 2)
    prof = ctx.profile(device_step, 2)
    raw = raw_bytes * layers
    return {"path": "reference unchain_kv.splitzip_cuda (unchanged) -> this library; per layer: index_select pack "
                    "-> encode_top16 -> [D2H pinned -> H2D] -> decode_top16",
            "layers": layers, "raw_bytes_per_step": raw,
            "device_gbs_per_gpu": round(raw / (ms_dev * 1e-3) / 1e9, 2),
            "with_host_copies_gbs_per_gpu": round(raw / (ms_host * 1e-3) / 1e9, 2),
            "ms_per_step": [round(ms_dev, 4), round(ms_host, 4)], "repeats": [rep_dev, rep_host],
            "launches_per_layer": round(sum(nl for _, nl in prof.values()) / (2 * layers), 2),
            "kernels": {k: {"launches": nl, "ms_per_launch": round(ms / nl, 5)} for k, (ms, nl) in prof.items()}}


# ----------------------------------------------------------- transfer


def transfer_run(ctx, min_ms):
    """Prefill -> decode KV transfer (N >= 2, even): rank 2p encodes
    configs[1] (auto codec, all 32 layers) into its stream buffers; rank 2p +
    1 decodes them straight from rank 2p's HBM over NVLink into its own paged
    cache (unchainkv_b200.transport).  Two steps are in flight.  Also times
    the same bytes of raw KV sent over NCCL between the pair.  Every rank
    returns; rank 0's dict is the block."""
    import torch

    from unchainkv_b200 import workloads as W
    from unchainkv_b200.transport import StreamTransport, peer_job

    S, lib, args, dist = ctx.S, ctx.lib, ctx.args, ctx.dist
    world, rank = ctx.world, ctx.rank
    cfg = W.CONFIGS["c1"]
    L = args.layers or cfg.layers
    pair = rank // 2
    sender, receiver = 2 * pair, 2 * pair + 1
    P = build_plan(ctx, cfg, L, shard=pair)  # both ranks of a pair hold the same source words
    jobs, raw = P["jobs"], P["raw_bytes"]
    capacity = int(P["streams"].numel())
    transports = [StreamTransport(capacity, sender=2 * q, receiver=2 * q + 1) for q in range(world // 2)]
    tr = transports[pair]
    role = tr.role
    J = len(jobs)
    slots = []
    for s in range(tr.slots):
        base = tr.buffer(s)
        kv = P["src"] if role == "sender" else P["dst"]
        idx = P["src_t"] if role == "sender" else P["dst_t"]
        slots.append(S.job_array([peer_job(kv[l], idx[r], base + o, c, P["tables"][l]) for l, r, n, o, c in jobs]))
    sp = ctx.sp
    k_step = [0]

    def step():
        k = k_step[0]
        if role == "sender":
            if lib.kvq_splitzip_bf16_encode_auto_batch(slots[k % tr.slots], J, sp) <= 0:
                raise RuntimeError("encode declined: " + lib.kvq_splitzip_last_error().decode())
            tr.step(k)
        else:
            tr.step(k)
            if lib.kvq_splitzip_bf16_decode_auto_batch(slots[k % tr.slots], J, sp) <= 0:
                raise RuntimeError("decode declined: " + lib.kvq_splitzip_last_error().decode())
        k_step[0] = k + 1

    step()
    torch.cuda.synchronize()
    ok = torch.ones(1, device=ctx.device)
    if role == "receiver":
        try:
            check_round_trip(P, "transferred step")
        except RuntimeError:
            ok.zero_()
    stream_total = 0.0
    if role == "sender":
        if lib.kvq_splitzip_bf16_encode_auto_batch(P["enc"], J, sp) <= 0:
            raise RuntimeError("encode declined")
        torch.cuda.synchronize()
        _, sizes, _, _ = stream_census(ctx, P)
        stream_total = float(sum(s or 0 for s in sizes))
    ms_step, repeats, _ = ctx.timed_repeats(step, args.steps, args.warmup, min_ms)
    torch.cuda.synchronize()
    if role == "receiver":
        try:
            check_round_trip(P, "transferred timed steps")
        except RuntimeError:
            ok.zero_()
    prof = ctx.profile(step, max(1, min(args.steps, 50)))
    torch.cuda.synchronize()
    for t in transports:
        t.finish()
    raw_buf = torch.empty(raw, dtype=torch.uint8, device=ctx.device)

    def raw_step():
        if role == "sender":
            dist.send(raw_buf, receiver)
        else:
            dist.recv(raw_buf, sender)

    raw_steps = max(3, min(args.steps, 20))
    ms_raw = ctx.timed(raw_step, raw_steps) / raw_steps
    dec = prof.get("DecodeAutoKernel", (0.0, 1))
    enc = prof.get("EncodeAutoKernel", (0.0, 1))
    per = torch.tensor([dec[0] / max(dec[1], 1), enc[0] / max(enc[1], 1), stream_total], device=ctx.device)
    dist.all_reduce(per, op=dist.ReduceOp.MAX)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    for t in transports:
        t.close()
    del P, slots
    torch.cuda.empty_cache()
    nvlink_peak = 770.0  # measured peer copy per direction on this pool's B200s (GB/s)
    dec_ms, enc_ms, stream_total = float(per[0]), float(per[1]), float(per[2])
    pairs = world // 2
    return {"metric": "KV transfer GB/s of raw bf16 KV delivered (encode on the sender GPU, decode on arrival over "
                      "NVLink on the receiver GPU)",
            "value": round(pairs * raw / (ms_step * 1e-3) / 1e9, 3), "unit": "GB/s",
            "ms_per_step": round(ms_step, 5), "repeats": repeats, "pairs": pairs, "layers": L,
            "raw_bytes_per_step": raw, "stream_bytes_per_step": int(stream_total),
            "ratio": round(raw / stream_total, 4) if stream_total else None, "slots_in_flight": tr.slots,
            "bit_exact": bool(ok.item() == 1),
            "raw_kv_over_nccl_gbs": round(pairs * raw / (ms_raw * 1e-3) / 1e9, 3),
            "roofline": {"bound": "nvlink", "kernel": "DecodeAutoKernel (receiver, reading the sender's streams)",
                         "achieved": round(stream_total / (dec_ms * 1e-3) / 1e9, 1) if dec_ms else None,
                         "peak": nvlink_peak, "unit": "GB/s",
                         "frac": round(stream_total / (dec_ms * 1e-3) / 1e9 / nvlink_peak, 4) if dec_ms else None,
                         "peak_kind": "measured peer copy (pool reference)"},
            "kernels": {"DecodeAutoKernel": {"ms_per_launch": round(dec_ms, 5)},
                        "EncodeAutoKernel": {"ms_per_launch": round(enc_ms, 5)}},
            "parallelism": f"{pairs} sender -> receiver pair(s), ordered by NCCL tokens"}


# ---------------------------------------------------------- CPU baseline


def cpu_jobs(cfg, layers: int, shard: int = 0):
    """Host sample of a workload for the CPU legs: (cache, src ids, dst ids,
    544-byte tables) per call.  c1/c2: the first `layers` layers of the
    request, the same host draw the GPU arm encodes; c3: the first
    `4*layers` requests of layer 0."""
    from unchainkv_b200 import splitzip_cuda, workloads

    def table(books):
        return np.frombuffer(splitzip_cuda.build_top16_tables(books), dtype=np.uint8).copy()

    if isinstance(cfg, workloads.MixedConfig):
        cache, tabs, books = workloads.mixed_sample_host(cfg, 0, 4 * layers, shard=shard)
        pool = cache.shape[1]
        tabs2 = workloads.request_block_tables(pool, [len(t) for t in tabs], 3001)
        t544 = table(books)
        return [(cache, np.ascontiguousarray(a), np.ascontiguousarray(b), t544) for a, b in zip(tabs, tabs2)]
    words, books = host_request_words(cfg, range(layers), shard)
    ids = np.arange(cfg.blocks, dtype=np.int64)
    ids2 = np.ascontiguousarray(workloads.block_table(cfg.blocks * cfg.pool_factor, cfg.blocks, 3001))
    return [(w, ids, ids2, table(b)) for w, b in zip(words, books)]


def cpu_pipeline_gbs(cfg, layers: int, repeats: int = 3, shard: int = 0):
    """The reference path on host cores: top16 attempt -> (overflow) fixed6
    encode -> decode into a second cache, per call, all host threads.
    Returns (GB/s of raw KV, threads, escape rate, mode histogram, sample)."""
    from oracle import oracle
    from unchainkv_b200 import workloads

    lib = oracle.lib()
    threads = host_threads()
    jobs = cpu_jobs(cfg, layers, shard)
    bw = cfg.block_words
    largest = max(2 * len(ids) * bw for _, ids, _, _ in jobs)
    out = np.zeros(2 * largest + 4096, dtype=np.uint8)
    pool = max(int(max(ids2.max() for _, _, ids2, _ in jobs)) + 1, jobs[0][0].shape[1])
    target = np.zeros((2, pool) + jobs[0][0].shape[2:], dtype=np.uint16)
    modes = {}
    escapes = 0

    def run(cache, ids, ids2, tables):
        blocks = len(ids)
        n = 2 * blocks * bw
        ps = cache.shape[1] * bw
        pt = target.shape[1] * bw
        res = lib.orc_encode_top16_blocks_mt(cache.ctypes.data, ps, bw, bw, ids.ctypes.data, 0, blocks,
                                             out.ctypes.data, out.size, tables.ctypes.data, threads)
        mode = int(out[0])
        if mode == 255:
            res = lib.orc_encode_mode_blocks_mt(cache.ctypes.data, ps, bw, bw, ids.ctypes.data, 0, blocks,
                                                out.ctypes.data, out.size, 6, threads)
            mode = int(out[0])
            lib.orc_decode_fixed6_blocks_mt(out.ctypes.data, res, target.ctypes.data, n, blocks, bw, pt, bw,
                                            0, ids2.ctypes.data, threads)
        else:
            lib.orc_decode_top16_blocks_mt(out.ctypes.data, res, target.ctypes.data, n, blocks, bw, pt, bw,
                                           0, ids2.ctypes.data, tables.ctypes.data, threads)
        return mode

    words = 0
    for cache, ids, ids2, tables in jobs:  # warm-up + mode census
        mode = run(cache, ids, ids2, tables)
        modes[mode] = modes.get(mode, 0) + 1
        escapes += oracle.escape_count(cache[:, ids].reshape(-1), tables)
        words += 2 * len(ids) * bw
    times = []
    for _ in range(repeats):
        t = time.perf_counter()
        for job in jobs:
            run(*job)
        times.append(time.perf_counter() - t)
    sec = statistics.median(times)
    if isinstance(cfg, workloads.MixedConfig):
        sample = f"first {len(jobs)} of {cfg.requests} requests of one layer, host numpy draw of the same distribution"
    else:
        sample = f"{len(jobs)} of {cfg.layers} layers: the host draw the GPU arm encodes"
    return 2 * words / sec / 1e9, threads, escapes / words, modes, sample


def connector_cpu_gbs(cfg, shard: int = 0, chunk_blocks: int = 16):
    """The reference connector's own CPU codec (vllm_connector.py:3204-3343
    torch-op encoder, :5098-5313 receiver) on CPU tensors, with
    torch.set_num_threads(nproc): one layer of the same host draw, encoded
    and decoded back `chunk_blocks` blocks per call.  The connector takes
    that path only below 1 MiB per call (vllm_connector.py:3042-3060: a
    larger layer goes to its GPU codec buffer, and a CPU tensor is sent
    raw), so the layer is coded in 512 KiB calls.  None when the reference
    package is not installed."""
    if not (REF_PACKAGE / "unchain_kv" / "vllm_connector.py").exists():
        return None
    import importlib
    from types import SimpleNamespace

    import torch

    if str(REF_PACKAGE) not in sys.path:
        sys.path.insert(0, str(REF_PACKAGE))
    saved = {k: os.environ.get(k) for k in ("UNCHAIN_KV_CODEC", "UNCHAIN_KV_CODEC_GPU_SLOTS")}
    os.environ["UNCHAIN_KV_CODEC"] = "splitzip_bf16"
    os.environ["UNCHAIN_KV_CODEC_GPU_SLOTS"] = "1"
    threads = os.cpu_count() or 1
    old_threads = torch.get_num_threads()
    try:
        connector_mod = importlib.import_module("unchain_kv.vllm_connector")
        torch.set_num_threads(threads)
        words, _ = host_request_words(cfg, [0], shard)
        kv = torch.from_numpy(words[0].reshape(2, cfg.blocks, -1).view(np.int16).copy()).view(torch.bfloat16)
        producer = connector_mod.UnchainKVConnector(
            SimpleNamespace(kv_transfer_config=SimpleNamespace(kv_role="kv_producer")), "worker")
        consumer = connector_mod.UnchainKVConnector(
            SimpleNamespace(kv_transfer_config=SimpleNamespace(kv_role="kv_consumer")), "worker")
        target = torch.zeros_like(kv)
        chunks = [list(range(b, min(b + chunk_blocks, cfg.blocks))) for b in range(0, cfg.blocks, chunk_blocks)]

        def run():
            modes, raw = set(), 0
            for ids in chunks:
                encoded = producer._splitzip_bf16_native_blocks(kv, ids)
                if encoded is None:
                    raise RuntimeError("reference connector declined the CPU encode")
                data, _, raw_bytes, enc_bytes, _ = encoded
                payload = bytes(data)[:enc_bytes]
                restored, copied = consumer._copy_splitzip_bf16_native_blocks(
                    target, ids, [payload], {"raw_bytes": raw_bytes, "encoded_bytes": enc_bytes})
                if copied != raw_bytes:
                    raise RuntimeError("reference connector receiver declined")
                # the payload left: its codec buffer is free again, as after a send
                producer._release_pending_codec_buffers()
                modes.add(payload[0])
                raw += raw_bytes
            return sorted(modes), raw

        modes, raw = run()
        t = time.perf_counter()
        run()
        sec = time.perf_counter() - t
        if not torch.equal(target.view(torch.int16), kv.view(torch.int16)):
            raise RuntimeError("reference connector CPU round trip differs")
        return {"value": round(raw / sec / 1e9, 4), "unit": "GB/s", "cores": threads,
                "kind": "reference (connector CPU codec)",
                "sample": f"1 of {cfg.layers} layers of the host draw in {len(chunks)} calls of {chunk_blocks} "
                          f"blocks; torch-op encode (modes {modes}) + receiver decode",
                "cpu": cpu_model()}
    except Exception as exc:  # the reference's code path itself failed here
        return {"unavailable": f"reference connector CPU codec: {type(exc).__name__}: {exc}"}
    finally:
        torch.set_num_threads(old_threads)
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def python_decoder_gbs():
    """The reference's pure-Python top16 decoder (vllm_connector.py:176-220)
    on one in-capacity top16 stream of 2^18 words (single thread); None when
    the reference package is not installed."""
    if not (REF_PACKAGE / "unchain_kv" / "vllm_connector.py").exists():
        return None
    import importlib

    from oracle import oracle
    from unchainkv_b200 import splitzip_cuda as S

    if str(REF_PACKAGE) not in sys.path:
        sys.path.insert(0, str(REF_PACKAGE))
    try:
        mod = importlib.import_module("unchain_kv.vllm_connector")
        n = 1 << 18
        books = S._DEFAULT_TOP16_CODEBOOKS[:32]
        rng = np.random.Generator(np.random.PCG64(4200))
        book = np.frombuffer(books, dtype=np.uint8).reshape(2, 16)
        exp = book[(np.arange(n) >= n // 2).astype(np.int64), rng.integers(0, 16, size=n)].astype(np.int64)
        exp[::200] = next(v for v in range(1, 255) if v not in books)
        words = ((rng.integers(0, 2, size=n) << 15) | (exp << 7) | rng.integers(0, 128, size=n)).astype(np.uint16)
        tables = np.frombuffer(S.build_top16_tables(books), dtype=np.uint8)
        res, stream = oracle.encode_top16(words, tables)
        payload = bytes(stream[:res])
        t = time.perf_counter()
        out = mod._decode_splitzip_top16_payload(payload, 2 * n, books)
        sec = time.perf_counter() - t
        if out != words.tobytes():
            raise RuntimeError("reference pure-Python decoder output differs")
        return {"value": round(2 * n / sec / 1e9, 6), "unit": "GB/s", "cores": 1,
                "kind": "reference (pure-Python top16 decoder)",
                "sample": f"one in-capacity top16 stream of {n} words (escapes == capacity), decode only",
                "cpu": cpu_model()}
    except Exception as exc:
        return {"unavailable": f"reference pure-Python decoder: {type(exc).__name__}: {exc}"}


def cpu_baseline(cfg, layers: int, shard: int = 0, repeats: int = 3, others: bool = True):
    from unchainkv_b200 import workloads

    gbs, threads, esc, modes, sample = cpu_pipeline_gbs(cfg, layers, repeats, shard)
    line = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample,
            "cpu": cpu_model(), "escape_rate": round(esc, 5), "modes": {str(k): v for k, v in modes.items()}}
    if others and not isinstance(cfg, workloads.MixedConfig):
        line["others"] = [x for x in (connector_cpu_gbs(cfg, shard), python_decoder_gbs()) if x is not None]
    return line


def reference_arm(args):
    """`--impl reference`: the reference's CPU codec path (restated by the
    oracle), rank 0 only, bounded sample per step, with the GPU arm's config
    keys."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from unchainkv_b200 import workloads

    out = JsonOut()
    if args.workload in ("calib", "modes", "writeback", "transfer", "top16"):
        out.emit({"impl": "reference", "unavailable": "auxiliary workload; its line reports the CPU "
                  "restatement as cpu_baseline"})
        return
    cfg = workloads.CONFIGS[args.workload]
    common = {"impl": "reference", "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
              "higher_is_better": True, "scaling": "weak", "vs_baseline": None}
    if args.workload == "c4":
        gbs, threads, sample = attention_cpu_gbs(cfg, repeats=max(1, args.steps))
        out.emit({
            **common, "metric": "decode attention over compressed KV: GB/s of raw bf16 KV attended per GPU",
            "value": round(gbs, 3), "dtype": "fp32",
            "data": "synthetic (seeded numpy draw of the configs[0] distribution)",
            "config": {"workload": cfg.name, "streams": "fixed6", "requests": cfg.requests,
                       "q_heads": cfg.kv_heads * cfg.group, "kv_heads": cfg.kv_heads, "head_dim": cfg.head_dim,
                       "block_tokens": cfg.block_tokens, "context_tokens": [cfg.min_tokens, cfg.max_tokens],
                       "pipeline": "oracle fixed6 decode -> numpy fp32 attention"},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample + " per step", "cpu": cpu_model()},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        })
        return
    layers = max(1, args.cpu_layers)
    cpu = cpu_baseline(cfg, layers, repeats=max(1, args.steps), others=args.workload == "c1")
    cpu["sample"] += " per step"
    if isinstance(cfg, workloads.MixedConfig):
        blocks = workloads.request_blocks(cfg, workloads.request_lengths(cfg))
        shape_cfg = {"requests": cfg.requests, "tokens_per_layer": int(sum(blocks) * cfg.block_tokens),
                     "request_tokens": [cfg.min_tokens, cfg.max_tokens], "scale_shift": cfg.scale_shift,
                     "model_layers": cfg.model_layers}
        pool = int(sum(blocks) * cfg.pool_factor)
        jobs = cfg.layers * cfg.requests
        raw = 2 * cfg.layers * sum(2 * b * cfg.block_words for b in blocks)
    else:
        shape_cfg = {"tokens": cfg.tokens}
        pool = cfg.blocks * cfg.pool_factor
        jobs = cfg.layers
        raw = cfg.raw_bytes
    out.emit({
        **common, "metric": METRIC, "value": cpu["value"], "dtype": "u16",
        "data": "synthetic (seeded numpy draw of the config distribution; the same bytes the GPU arm encodes)",
        "config": {"workload": cfg.name, "layers": cfg.layers, **shape_cfg, "kv_heads": cfg.kv_heads,
                   "head_dim": cfg.head_dim, "block_tokens": cfg.block_tokens, "pool_blocks": pool,
                   "jobs_per_step": jobs, "raw_bytes_per_step": raw,
                   "policy": "top16 attempt -> fixed6 fallback -> decode (host threads)",
                   "parallelism": "host threads of one process (rank 0)"},
        "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


# ------------------------------------------------------------ auxiliary


def modes_layer_words(layer: int, shape, rng):
    """Host words of a `modes` layer: the configs[1] draw (sign/magnitude,
    mode 2), 40 high bytes with magnitudes spanning 7 bits (palette, mode
    0), or random high bytes over 2-value low nibbles (nibble planes, mode
    1), by layer % 3."""
    from unchainkv_b200 import workloads as W

    kind = layer % 3
    if kind == 0:
        tokens = shape[1] * shape[2] // (W.KV_HEADS * W.HEAD_DIM)
        words = W.draw_tokens(2000 + layer, W.channel_scales(layer), tokens)
        return np.ascontiguousarray(words.reshape(shape))
    if kind == 1:
        rest = np.array([h for h in range(256) if h not in (0x10, 0xF5)])
        highs = np.concatenate([[0x10, 0xF5], rng.choice(rest, size=38, replace=False)])
        high, low = highs[rng.integers(0, 40, shape)], rng.integers(0, 256, shape)
    else:
        high, low = rng.integers(0, 256, shape), (rng.integers(0, 256, shape) & 0x11) | 0x40
    return ((high << 8) | low).astype(np.uint16)


def aux_run(ctx):
    """--workload calib: GPU calibration (exponent histograms gathered from
    the configs[1] paged cache + device-ranked top16 tables of all 32
    layers).  --workload modes: the receiver's torch-op forms (modes 2, 0, 1)
    decoded into the paged cache, 12 configs[1]-shaped layers.
    --workload writeback: the configs[1] streams copied over their blocks."""
    import torch

    from unchainkv_b200 import workloads as W

    S, args, device, rank = ctx.S, ctx.args, ctx.device, ctx.rank
    cfg = W.CONFIGS["c1"]

    if args.workload == "calib":
        L = args.layers or cfg.layers
        P = build_plan(ctx, cfg, L)
        src, ids = P["src"], P["src_t"][0]
        hist = torch.zeros((L, 2, 256), dtype=torch.int32, device=device)
        tables = torch.empty((L, 544), dtype=torch.uint8, device=device)
        observed = torch.empty((L, 2), dtype=torch.int32, device=device)
        jobs = S.job_array([S.histogram_job(src[l], ids, hist[l]) for l in range(L)])
        raw = P["raw_bytes"]

        def step():
            hist.zero_()
            if S.exponent_histogram_batch(jobs) != L:
                raise RuntimeError("histograms declined")
            S.top16_tables_from_histograms(hist, tables, observed)

        step()
        torch.cuda.synchronize()
        for l in range(L):  # the reference's bincount and ranking, exactly
            w = src[l][:, ids].reshape(2, -1).view(torch.int16).to(torch.int32) & 0xFFFF
            ref = torch.stack([torch.bincount((p >> 7) & 0xFF, minlength=256) for p in w]).to(torch.int32)
            if not torch.equal(ref, hist[l]):
                raise RuntimeError(f"layer {l}: histogram differs from bincount")
            h = hist[l].cpu().tolist()
            books = bytes(S.rank_top16(h[0]) + S.rank_top16(h[1]))
            if len(books) == 32 and bytes(tables[l].cpu().numpy().tobytes()) != S.build_top16_tables(books):
                raise RuntimeError(f"layer {l}: device table differs from the ranking rule")
        alg = {"ExpHistogramKernel": raw + 2048 * L, "Top16TablesKernel": 2048 * L + 552 * L}
        dominant = "ExpHistogramKernel"
        metric = "calibration GB/s of raw bf16 KV per GPU (exponent histograms + top16 tables)"
        extra_cfg = {"layers": L, "tokens": cfg.tokens, "tables_bytes": 544 * L}
        tables_host = torch.empty((L, 544), dtype=torch.uint8).pin_memory()
        obs_host = torch.empty((L, 2), dtype=torch.int32).pin_memory()

        def e2e_step():
            step()
            tables_host.copy_(tables, non_blocking=True)
            obs_host.copy_(observed, non_blocking=True)

        e2e_io = (0, tables.numel() + observed.numel() * 4,
                  "KV cache resident in HBM -> histograms -> device tables -> pinned host tables")

        def cpu_line():
            sample = 2
            host = [P["host_words"][l].reshape(2, -1) for l in range(sample)]
            t0 = time.perf_counter()
            for words in host:
                counts = [np.bincount((p >> 7) & 0xFF, minlength=256) for p in words]
                _ = [S.rank_top16(c) for c in counts]
            dt = time.perf_counter() - t0
            return sample * raw / L / dt / 1e9, 1, f"{sample} of {L} layers, numpy bincount + ranking"
    elif args.workload == "writeback":  # auto encode + writeback over the blocks, configs[1]
        L = args.layers or cfg.layers
        blocks, pool = cfg.blocks, cfg.blocks * cfg.pool_factor
        start = pool - blocks  # one contiguous run per layer (the reference writes back single runs)
        run_ids = torch.arange(start, start + blocks, device=device)
        kv = torch.empty((L, 2, pool, cfg.block_tokens, cfg.kv_heads, cfg.head_dim), dtype=torch.bfloat16,
                         device=device)
        books = b"".join(W.fill_layer_device(kv[l], cfg, l, run_ids.cpu().numpy(), shard=rank) for l in range(L))
        tables = torch.tensor(np.frombuffer(b"".join(S.build_top16_tables(books[l * 32:(l + 1) * 32])
                                                     for l in range(L)), np.uint8).reshape(L, 544).copy(),
                              device=device)
        original = kv.clone()
        n = 2 * blocks * cfg.block_words
        cap = (S.auto_capacity(n) + 15) // 16 * 16
        buf = torch.zeros(L * cap, dtype=torch.uint8, device=device)
        enc = S.job_array([S.make_job(kv[l], None, buf[l * cap:(l + 1) * cap], cap, tables[l], start, blocks)
                           for l in range(L)])
        S.encode_auto_batch(enc)
        torch.cuda.synchronize()
        heads = buf.view(L, cap)[:, :8].cpu().numpy()
        lengths = [S.stream_length(bytes(h), n) for h in heads]
        wb = S.job_array([S.writeback_job(kv[l], buf[l * cap:(l + 1) * cap], lengths[l], start, blocks)
                          for l in range(L)])
        raw = 2 * L * n
        stream_total = sum(lengths)
        host = torch.empty(stream_total, dtype=torch.uint8).pin_memory()

        def step():
            # the writeback of all layers' streams (the encode that made them
            # is the c1 workload's; once written back the blocks hold the
            # stream, so a step repeats the same copy)
            if S.writeback_batch(wb) != stream_total:
                raise RuntimeError("writeback declined")

        step()
        torch.cuda.synchronize()
        for l in range(L):
            staged = torch.cat(S.writeback_segments(kv[l], start, blocks))[:lengths[l]]
            if not torch.equal(staged, buf[l * cap:l * cap + lengths[l]]):
                raise RuntimeError(f"layer {l}: written-back bytes differ from the stream")
            if not torch.equal(kv[l][:, :start], original[l][:, :start]):
                raise RuntimeError(f"layer {l}: blocks outside the run changed")
        del original
        alg = {"WritebackKernel": 2 * stream_total}
        dominant = "WritebackKernel"
        metric = "codec writeback GB/s of raw bf16 KV per GPU (configs[1] streams over their own blocks)"
        extra_cfg = {"layers": L, "tokens": cfg.tokens, "stream_bytes_per_step": stream_total,
                     "modes": [int(h[0]) for h in heads]}

        def e2e_step():
            step()
            offset = 0
            for l in range(L):  # the host stages from the blocks, as the reference does
                for seg in S.writeback_segments(kv[l], start, blocks):
                    take = min(seg.numel(), lengths[l] - (offset - sum(lengths[:l])))
                    if take <= 0:
                        break
                    host[offset:offset + take].copy_(seg[:take], non_blocking=True)
                    offset += take

        e2e_io = (0, stream_total, "writeback_batch -> D2H from the blocks to pinned host (the reference's staging)")

        def cpu_line():
            t0 = time.perf_counter()
            for l in range(2):
                src = buf[l * cap:l * cap + lengths[l]].cpu().numpy()
                segs = [np.empty(2 * blocks * cfg.block_words, dtype=np.uint8) for _ in range(2)]
                k = min(lengths[l], segs[0].size)
                segs[0][:k] = src[:k]
                segs[1][:lengths[l] - k] = src[k:]
            dt = time.perf_counter() - t0
            return 2 * 2 * n * 2 / dt / 1e9, 1, "2 layers, host memcpy of the stream into the segments"
    else:  # modes: GPU torch-op encode + decode_any round trip
        L = args.layers or 12
        blocks, pool = cfg.blocks, cfg.blocks * cfg.pool_factor
        src_ids = torch.as_tensor(W.block_table(pool, blocks, 3000), device=device)
        dst_ids = torch.as_tensor(W.block_table(pool, blocks, 3001), device=device)
        bw = cfg.block_tokens * cfg.kv_heads * cfg.head_dim
        shape = (2, pool, bw)
        rng = np.random.Generator(np.random.PCG64(4100 + rank))
        src = torch.zeros((L,) + shape, dtype=torch.int16, device=device)
        for l in range(L):
            src[l][:, src_ids] = torch.from_numpy(modes_layer_words(l, (2, blocks, bw), rng).view(np.int16)).to(device)
        src = src.view(torch.bfloat16)
        dst = torch.zeros_like(src)
        n = 2 * blocks * bw
        cap = S.torchop_capacity(n)
        streams = torch.zeros(L * cap, dtype=torch.uint8, device=device)
        enc = S.job_array([S.make_job(src[l], src_ids, streams[l * cap:(l + 1) * cap]) for l in range(L)])
        S.encode_torchop_batch(enc)
        torch.cuda.synchronize()
        heads = streams.view(L, cap)[:, :8].cpu().numpy()
        lengths = [S.stream_length(bytes(h), n) for h in heads]
        tables = torch.from_numpy(np.frombuffer(S.build_top16_tables(S._DEFAULT_TOP16_CODEBOOKS[:32]),
                                                np.uint8).copy()).to(device)
        dec = S.job_array([S.make_job(dst[l], dst_ids, streams[l * cap:(l + 1) * cap], lengths[l], tables)
                           for l in range(L)])
        raw = 2 * L * n
        stream_total = sum(lengths)

        def encode():
            if S.encode_torchop_batch(enc) is None:
                raise RuntimeError("torch-op encode declined")

        def decode():
            if S.decode_any_batch(dec) is None:
                raise RuntimeError("decode declined")

        def step():
            encode()
            decode()

        step()
        torch.cuda.synchronize()
        for l in range(L):
            if not torch.equal(dst[l][:, dst_ids].view(torch.int16), src[l][:, src_ids].view(torch.int16)):
                raise RuntimeError(f"layer {l}: round trip differs")
        alg = {"TorchopStatsKernel": raw, "TorchopEncodeKernel": raw + stream_total,
               "ModeDecodeKernel": stream_total + raw}
        dominant = None
        metric = "torch-op codec round trip GB/s of raw bf16 KV per GPU (modes 2, 0, 1: GPU encode + receiver decode)"
        extra_cfg = {"layers": L, "tokens": cfg.tokens, "modes": [int(h[0]) for h in heads],
                     "stream_bytes_per_step": stream_total, "ratio": round(raw / stream_total, 4)}
        host = torch.empty(L * cap, dtype=torch.uint8).pin_memory()

        def e2e_step():
            # each stream's exact bytes (lengths from the headers) leave and
            # come back through pinned host memory
            encode()
            for l in range(L):
                host[l * cap:l * cap + lengths[l]].copy_(streams[l * cap:l * cap + lengths[l]], non_blocking=True)
            for l in range(L):
                streams[l * cap:l * cap + lengths[l]].copy_(host[l * cap:l * cap + lengths[l]], non_blocking=True)
            decode()

        e2e_io = (stream_total, stream_total, "encode_torchop_batch -> D2H pinned -> H2D -> decode_any_batch")

        def cpu_line():
            from oracle import oracle

            ids = W.block_table(pool, blocks, 3000)
            sample = 3
            caches = []
            for l in range(sample):
                cache = np.zeros(shape, dtype=np.uint16)
                cache[:, ids] = src[l][:, src_ids].view(torch.int16).cpu().numpy().view(np.uint16)
                caches.append(cache)
            t0 = time.perf_counter()
            for cache in caches:
                _, stream_c = oracle.encode_torchop_blocks(cache, ids)
                target = np.zeros(shape, dtype=np.uint16)
                oracle.decode_modes_blocks(stream_c, target, ids)
            dt = time.perf_counter() - t0
            return sample * raw / L / dt / 1e9, 1, f"{sample} layers (one of each mode), oracle encode + receiver, 1 thread"

    sampler = ctx.sampler()
    ms_step, repeats, timed_ms = ctx.timed_repeats(step, args.steps, args.warmup, args.min_timed_ms)
    if sampler:
        sampler.stop()
    prof_steps = max(1, min(args.steps, 100))
    prof = ctx.profile(step, prof_steps)
    e2e = None
    if not args.skip_e2e:
        e2e_ms = ctx.timed(e2e_step, args.e2e_steps) / args.e2e_steps
        e2e = {"value": round(ctx.world * raw / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": e2e_io[0], "d2h_bytes_per_step": e2e_io[1], "ms_per_step": round(e2e_ms, 4),
               "path": e2e_io[2]}
    kernels = kernel_table(prof, alg, prof_steps)
    if dominant is None:
        dominant = max((k for k in kernels if k in alg), key=lambda k: kernels[k]["ms_per_launch"])
    cpu = None
    if not args.no_cpu_baseline and rank == 0:
        gbs, threads, sample = cpu_line()
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample,
               "cpu": cpu_model()}
    ctx.emit({
        "metric": metric, "value": round(ctx.world * raw / (ms_step * 1e-3) / 1e9, 3), "unit": "GB/s",
        "n_gpus": ctx.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "repeats": repeats, "timed_ms": round(timed_ms, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u16",
        "data": "synthetic (seeded draws, configs[1] shape)",
        "config": {"workload": args.workload, **extra_cfg, "raw_bytes_per_step": raw,
                   "l2": "raw KV per step larger than L2",
                   "parallelism": f"independent per-GPU shards x{ctx.world} (no collective)"},
        "roofline": roofline_of(kernels, dominant, args.workload),
        "kernels": kernels,
        "gpu_launches": int(round(sum(nl for _, nl in prof.values()) / prof_steps * args.steps * repeats)),
        "clocks": sampler.summary() if sampler else None,
        "cpu_baseline": cpu,
        "e2e": e2e,
    })


# ------------------------------------------------------------------ main


def b200_main(args):
    import torch

    from unchainkv_b200 import workloads as W

    ctx = Ctx(args)
    try:
        if args.workload in ("calib", "modes", "writeback"):
            aux_run(ctx)
            return
        if args.workload == "transfer":
            if ctx.world < 2 or ctx.world % 2:
                raise SystemExit("--workload transfer needs an even number of GPUs >= 2 (sender, receiver pairs)")
            r = transfer_run(ctx, args.min_timed_ms)
            ctx.emit({**{k: r[k] for k in ("metric", "value", "unit", "ms_per_step", "repeats")},
                      "n_gpus": ctx.world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "u16",
                      "data": "synthetic (seeded host draw of the configs[1] distribution)",
                      "config": {"workload": "transfer", "layers": r["layers"], "pairs": r["pairs"],
                                 "raw_bytes_per_step": r["raw_bytes_per_step"], "parallelism": r["parallelism"]},
                      "transfer": r, "roofline": r["roofline"], "cpu_baseline": None, "e2e": None,
                      "e2e_note": "device-resident KV to device-resident KV: no host copy is part of this path"})
            return
        if args.workload == "c4":
            r = attention_run(ctx, args.attn_streams, args.min_timed_ms)
            cfg = r.pop("_cfg")
            ctx.emit({"metric": "decode attention over compressed KV: GB/s of raw bf16 KV attended per GPU",
                      "value": r.pop("value"), "unit": "GB/s", "n_gpus": ctx.world, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": r.pop("ms_per_step"), "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 accumulation)",
                      "data": ("synthetic (seeded device draw of the configs[0] distribution, fixed6 streams)"
                               if args.attn_streams == "fixed6" else
                               "synthetic (seeded device draw: exponents from a 16-entry book per plane, 0.3% "
                               "escapes, top16 streams)"),
                      "config": cfg, **r})
            return
        if args.workload == "top16":
            r = top16_run(ctx, args.min_timed_ms)
            ref = r["reference_abi"]
            ctx.emit({"metric": METRIC, "value": round(ctx.world * r["raw_bytes_per_step"] /
                                                       ((ref["ms_encode"] + ref["ms_decode"]) * 1e-3) / 1e9, 3),
                      "unit": "GB/s", "n_gpus": ctx.world, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(ref["ms_encode"] + ref["ms_decode"], 5), "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "u16", "data": r["data"],
                      "config": {"workload": "top16", "layers": r["layers"]}, "top16": r,
                      "cpu_baseline": None, "e2e": None})
            return
        cfg = W.CONFIGS[args.workload]
        L = args.layers or cfg.layers
        data = ("synthetic (seeded numpy draw of the config distribution, the bytes the reference arm encodes; "
                "other pool blocks device draws)" if args.workload != "c3" else
                "synthetic (seeded device draw of the shifted distribution)")
        r = codec_run(ctx, cfg, L, args.min_timed_ms, parity_jobs=None if args.workload != "c3" else 16,
                      workload=args.workload)
        line = codec_line(ctx, cfg, r, data)
        if args.workload == "c1" and not args.no_blocks:
            bms = args.block_timed_ms
            blocks = {}
            # rank r codes kv head r of the 70B TP=8 shard
            c2 = W.CONFIGS["c2"]
            r2 = codec_run(ctx, c2, args.layers or c2.layers, bms, parity_jobs=8, e2e=False, cpu=False,
                           clocks=True, workload="c2")
            plan2 = r2.pop("_plan")
            blocks["tp8_shard"] = {
                "workload": c2.name, "kv_head_of_rank": "rank r codes kv head r (mod 8) of every layer",
                "value": r2["value"], "unit": "GB/s", "ms_per_step": r2["ms_per_step"], "repeats": r2["repeats"],
                "aggregate_hbm_frac": r2["hbm_frac_round_trip"],
                "aggregate_hbm_frac_note": "algorithmic bytes of all ranks' round trips per step / max-over-ranks "
                                           "step time / (N x measured HBM GB/s)",
                "encode_gbs_per_gpu": r2["encode_gbs_per_gpu"], "decode_gbs_per_gpu": r2["decode_gbs_per_gpu"],
                "ratio": r2["ratio"], "modes": r2["modes"], "escape_rate": r2["escape_rate"],
                "parity": r2["parity"], "roofline": r2["roofline"], "clocks": r2["clocks"],
                "config": codec_config(c2, plan2, ctx.world)}
            blocks["top16"] = top16_run(ctx, bms)
            att = {}
            for codec in ("fixed6", "top16"):
                ra = attention_run(ctx, codec, bms, e2e=(codec == "fixed6"), cpu=False, clocks=False)
                acfg = ra.pop("_cfg")
                att[codec] = {"value": ra["value"], "unit": "GB/s (raw bf16 KV attended)",
                              "ms_per_step": ra["ms_per_step"], "repeats": ra["repeats"],
                              "max_abs_err_vs_fp32": ra["max_abs_err_vs_fp32"],
                              "max_err_over_tolerance": ra["max_err_over_tolerance"], "tolerance": ra["tolerance"],
                              "roofline": ra["roofline"], "e2e": ra["e2e"], "config": acfg}
            blocks["attention"] = att
            if ctx.rank == 0:
                blocks["reference_api"] = reference_api_run(ctx, bms)
            if ctx.world >= 2 and ctx.world % 2 == 0:
                blocks["transfer"] = transfer_run(ctx, bms)
            line.update(blocks)
        ctx.emit(line)
    finally:
        ctx.close()


def main():
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
    else:
        b200_main(args)


if __name__ == "__main__":
    main()
