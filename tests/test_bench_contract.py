"""bench.py's command-line contract, checked on the CPU: the reference arm
(``--impl reference``), which times the oracle port of the reference's CPU path
on the host cores, prints exactly one JSON line with the keys the benchmark
driver reads; too few warm-up steps are refused.  The GPU arm is exercised by
the round-end bench run itself."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(*args, timeout=600):
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT,
                          capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("workload", [None, "optim", "loader"])
def test_reference_arm_json_line(workload):
    extra = ("--workload", workload) if workload else ()
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "3", *extra)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True and d["value"] > 0
    assert "workload" in d["config"]
    assert d["config"]["rows_per_sample"] >= 1 and d["config"]["processes"] >= 1
    if workload is None:
        # the default line carries every other BASELINE config's reference figure
        assert set(d["per_workload"]) == {"rms", "ce", "embedding", "mlp_block"}
        for entry in d["per_workload"].values():
            assert entry["value"] > 0 and entry["config"]["rows_per_sample"] >= 1
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference")
    assert cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_warmup_below_three_is_refused():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "2", timeout=120)
    assert r.returncode != 0
    assert "--warmup must be >= 3" in r.stderr
