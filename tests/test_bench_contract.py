"""bench.py's reference arm on the host CPU: one JSON line with the keys the
round-end driver reads (the base contract plus `impl`, `cpu_baseline` and an
`e2e` object with zero copy bytes).  The reference is the C path compiled
from its own sources (oracle/_ref), timed as the reference runtime times
gpt2_forward per decode step; this run is a short sample of it."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_line():
    if not (ROOT / "oracle" / "_ref" / "libecref.so").exists():
        pytest.skip("the reference build (oracle/_ref) is absent")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "4", "--warmup", "3",
                        "--cpu-seconds", "1"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    o = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in o, k
    assert o["impl"] == "reference"
    assert o["value"] > 0 and o["unit"] == "tok/s" and o["higher_is_better"] is True
    assert o["warmup"] >= 3 and o["steps"] >= 4
    assert isinstance(o["config"], dict) and "workload" in o["config"]
    cb = o["cpu_baseline"]
    assert cb["value"] == o["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    e = o["e2e"]
    assert e["value"] == o["value"] and e["unit"] == o["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
