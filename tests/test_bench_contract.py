"""bench.py's reference arm on the CPU: one JSON line with the contract's keys.

The driver runs ``bench.py --impl reference`` next to the B200 arm and reads
exactly one JSON line from stdout.  The reference arm times the reference's
CPU path (the numpy restatement of the C2 op set) on host cores only, so it
is checked here without a GPU: the line parses, names the same metric as the
B200 arm, and carries ``impl``, ``cpu_baseline`` and ``e2e``."""

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.timeout(600)
def test_reference_arm_prints_one_contract_line():
    p = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, p.stdout[-2000:]
    d = json.loads(lines[0])
    sys.path.insert(0, REPO)
    import bench

    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC
    for key in ("value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
