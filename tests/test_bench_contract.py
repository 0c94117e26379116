"""bench.py's JSON contract on the CPU (no GPU): the reference arm (`--impl reference`, the CPU
restatement of the reference's arithmetic timed on the host cores) prints one JSON line with the
keys the driver reads, for a small config. The GPU arm's line is checked on the B200 by the
round-end bench itself."""

import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def test_reference_arm_json_line(tmp_path):
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--config", "tiny", "--steps", "2",
                          "--warmup", "1"], cwd=REPO, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["value"] > 0
    assert d["higher_is_better"] is True and d["n_gpus"] == 1 and d["data"] == "synthetic"
    assert "tiny" in d["metric"] and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
