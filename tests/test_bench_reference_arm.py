"""bench.py's reference arm (`--impl reference`) on the host cores.

The round-end driver runs this arm beside the GPU arm and parses its one
JSON line, so the line's keys are checked here: the BASELINE metric and
unit, a cpu_baseline describing the run, and an e2e object with no host
copies (the arm works on host memory).  Under torchrun only rank 0 prints.
Each run times a bounded sample and takes a few seconds.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def run_reference(*args, rank=None):
    env = dict(os.environ)
    if rank is not None:
        env["RANK"] = str(rank)
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args], cwd=ROOT,
                         env=env, capture_output=True, text=True, timeout=300, check=True)
    return [json.loads(line) for line in out.stdout.splitlines() if line.startswith("{")]


def check_common(line, steps, warmup):
    assert line["impl"] == "reference"
    assert line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["value"] > 0
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, steps, warmup)
    assert line["scaling"] == "weak" and line["vs_baseline"] is None
    cpu = line["cpu_baseline"]
    assert cpu["kind"] in ("reference", "port")
    assert cpu["cores"] >= 1 and cpu["value"] == line["value"] and cpu["unit"] == line["unit"]
    assert cpu["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_default_workload_line_reports_the_baseline_metric():
    lines = run_reference("--steps", "2", "--warmup", "1", "--cpu-layers", "1")
    assert len(lines) == 1
    line = lines[0]
    check_common(line, 2, 1)
    baseline = json.loads((ROOT / "BASELINE.json").read_text())
    assert line["metric"] == baseline["metric"]
    assert line["dtype"] == "u16"
    assert line["config"]["workload"] == "c1_llama3_8b_prefill_4096"
    # the sample takes the producer's fallback chain: every mode is a stream form
    assert set(line["cpu_baseline"]["modes"]) <= {"3", "5", "6"}


def test_attention_workload_line():
    lines = run_reference("--workload", "c4", "--steps", "1", "--warmup", "1")
    assert len(lines) == 1
    check_common(lines[0], 1, 1)
    assert lines[0]["metric"].startswith("decode attention over compressed KV")


def test_ranks_other_than_zero_print_nothing():
    assert run_reference("--steps", "1", "--warmup", "1", rank=1) == []
