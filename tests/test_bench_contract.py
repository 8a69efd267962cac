"""The benchmark's output contract on the reference arm, which runs on the host cores: one
JSON line on stdout with the metric, the timing fields, the CPU-baseline description and an
e2e block (no host-device copies for a host-only implementation)."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(not (ROOT / "oracle" / "_ref" / "libefref.so").exists(), reason="reference library not built")
def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2", "--warmup", "3"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "Q4_0 matvec HBM GB/s (config 4: 131072x8192, row-sharded over the job's GPUs)"
    assert d["unit"] == "GB/s"
    assert d["n_gpus"] == 1 and d["steps"] == 2 and d["warmup"] == 3 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"] == "config4_q4_0_matvec_131072x8192"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == d["value"] and cb["cores"] >= 1
    assert cb["physical_cores"] is None or 1 <= cb["physical_cores"] <= cb["logical_cpus"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
