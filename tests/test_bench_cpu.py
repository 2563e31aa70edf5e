"""bench.py's reference arm (the CPU restatement timed on host cores) and its
JSON line, on the small synthetic model: no GPU involved."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "tiny", "--steps", "3",
                        "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == "decode_tok_per_s" and d["unit"] == "tok/s"
    assert d["value"] > 0 and d["steps"] == 3 and d["warmup"] == 1 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] == "port"
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["sample"] and d["cpu_baseline"]["cpu"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    for k in ("workload", "model", "global_batch", "seq_len", "parallelism"):
        assert k in d["config"], k
