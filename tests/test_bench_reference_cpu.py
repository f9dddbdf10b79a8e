"""The reference arm of bench.py on CPU: `bench.py --impl reference` under a
two-rank torchrun prints exactly one JSON line (rank 0), rank 1 exits 0
without work, and the line carries the fields the benchmark driver reads:
metric, value, unit, step counts, timing, the CPU-baseline description and
an e2e block with no host<->device traffic. One warm-up and one timed step of
the 2B-shape oracle decode over the seeded C4 sample; about a minute here.
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.slow
@pytest.mark.timeout(900)
def test_reference_arm_two_ranks_one_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1"]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=850)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    line = json.loads(lines[0])

    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["n_gpus"] == 2 and line["steps"] == 1 and line["warmup"] == 1
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert "workload" in line["config"]

    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference")
    assert cb["cores"] >= 1 and cb["value"] == line["value"] and cb["unit"] == line["unit"]
    assert cb["sample"]

    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
