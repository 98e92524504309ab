"""bench.py's reference arm runs on the host cores only: it must print exactly
one JSON line carrying the keys of the benchmark contract (metric, value,
unit, n_gpus, steps, warmup, higher_is_better, config) plus the reference
arm's own (impl, cpu_baseline, e2e with zero transfer bytes).  The device
arm's line is produced and checked by the bench run on a GPU."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libpfref.so")):
        pytest.skip("reference library not built (oracle/Makefile)")

    def two_cores():  # the arm starts one reference process per usable core: keep the test small
        os.sched_setaffinity(0, sorted(os.sched_getaffinity(0))[:2])

    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=900,
                       preexec_fn=two_cores if hasattr(os, "sched_setaffinity") else None)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "config", "impl",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["metric"] == "accepted tok/s" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] >= 3
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and 1 <= d["cpu_baseline"]["cores"] <= 2
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]
