"""bench.py's reference arm keeps the JSON-line contract (CPU, tiny architecture).

The reference arm times the CPU restatement of the tuning step; on the test
architecture it finishes in seconds and must print one JSON line with the
metric, a positive value, ``impl: reference``, a ``cpu_baseline`` describing
the run and an ``e2e`` block with zero transfer bytes.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--arch", "tiny-qwen2", "--steps", "2", "--warmup", "1"],
                         capture_output=True, text=True, cwd=ROOT, env=env, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, out.stdout
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference"
    assert rec["unit"] == "blocks/s" and rec["higher_is_better"] is True
    assert rec["value"] > 0 and rec["ms_per_step"] > 0
    assert rec["steps"] == 2 and rec["warmup"] == 1
    cpu = rec["cpu_baseline"]
    assert cpu["value"] == rec["value"] and cpu["kind"] == "port" and cpu["cores"] >= 1
    assert "restatement" in cpu["sample"]
    e2e = rec["e2e"]
    assert e2e["value"] == rec["value"] and e2e["unit"] == rec["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert rec["config"]["global_batch"] == 8 and rec["config"]["seq_len"] == 2048
