"""bench.py's reference arm runs on the host and prints the JSON line the driver reads (no GPU)."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_the_contract_line():
    proc = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"],
        capture_output=True, text=True, timeout=600, cwd=ROOT,
    )
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = [l for l in proc.stdout.splitlines() if l.startswith("{")][-1]
    out = json.loads(line)
    assert out["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "config", "cpu_baseline",
                "e2e"):
        assert key in out, key
    assert out["value"] > 0 and out["higher_is_better"] is True
    assert out["cpu_baseline"]["value"] == out["value"]
    assert out["cpu_baseline"]["kind"] in ("port", "reference") and out["cpu_baseline"]["cores"] >= 1
    assert out["e2e"]["value"] == out["value"]
    assert out["e2e"]["h2d_bytes_per_step"] == 0 and out["e2e"]["d2h_bytes_per_step"] == 0
