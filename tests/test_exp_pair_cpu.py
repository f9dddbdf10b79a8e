"""The softmax's exp on the device (exp_pair in bitnetrs_b200/csrc/common.cuh)
against the host libm's expf, through a C mirror of its exact float
operations (tests/exp_pair_mirror.c): on every 61st float of [-87, 0], each
input that is not a table candidate rounds to exactly the host's expf, and
the float pair stays within 1e-3 ulp of exp(x) (the table rule needs it
within 0.003).  Running the mirror with stride 1 checks every float."""
import shutil
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_exp_pair_matches_host_expf(tmp_path):
    exe = tmp_path / "exp_pair_mirror"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", str(HERE / "exp_pair_mirror.c"), "-o", str(exe), "-lm"],
                   check=True)
    r = subprocess.run([str(exe), "61"], capture_output=True, text=True, timeout=600)
    f = dict(zip(r.stdout.split()[::2], r.stdout.split()[1::2]))
    assert r.returncode == 0, r.stdout
    assert int(f["checked"]) > 18_000_000
    assert int(f["non_candidate_mismatches"]) == 0
    assert float(f["max_err_ulp"]) < 1e-3
    assert 0 < int(f["candidates"]) < int(f["checked"]) // 100
