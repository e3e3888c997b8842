"""The bench's contract on the host (CPU only): the reference arm's JSON line
and the helpers every configuration's line is built from."""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_reference_arm_prints_the_contract_line():
    """`bench.py --impl reference` times the host-CPU restatement of the
    reference's path on the headline workload and prints one JSON line with
    the arm's keys: the same metric, unit and direction as the GPU arm, its
    own cpu_baseline, and an e2e with no host-device traffic."""
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True and d["value"] > 0
    assert (d["n_gpus"], d["steps"], d["warmup"]) == (1, 1, 0)
    assert d["config"]["workload"].startswith("c5")
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1
    assert cpu["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_error_metrics_forms():
    """The three error forms every check reports: scaled by sum|a b|,
    elementwise against 1 + |y|, and normwise."""
    want = np.array([1.0, -2.0, 0.0, 4.0])
    got = want + np.array([1e-6, 0.0, 2e-6, -4e-6])
    absum = np.array([10.0, 1.0, 1.0, 8.0])
    m = bench.err_metrics(got, want, absum)
    assert abs(m["max_err_over_sum_abs"] - 2e-6) < 1e-15
    assert abs(m["max_rel_err_elementwise"] - 2e-6) < 1e-15
    assert abs(m["normwise"] - 1e-6) < 1e-15


def test_check_rows_cover_every_row_tile():
    """Checked rows spread over all 128-row tiles of the output."""
    rows = bench.check_rows(8192)
    assert rows == sorted(set(rows)) and len(rows) == 64 and max(rows) < 8192
    assert {r // 128 for r in rows} == set(range(64))
    rows = bench.check_rows(2048, 16)
    assert len(rows) == 16 and {r // 128 for r in rows} == set(range(16))
    assert bench.check_rows(100, 4) == sorted(set(bench.check_rows(100, 4))) and max(bench.check_rows(100, 4)) < 100


def test_cpu_baseline_line():
    line = bench._cpu_line(2e12, 4.0, 16, "sample text")
    assert line == {"value": 0.5, "unit": "TFLOP/s", "cores": 16, "kind": "port", "sample": "sample text"}
