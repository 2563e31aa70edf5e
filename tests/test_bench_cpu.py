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


def test_tensor_parallel_groups_for_the_scaling_run():
    """bench.py --gpus N: one tensor-parallel group over the largest degree
    that divides N and both head counts; C3 (28 query / 4 KV heads) runs two
    TP4 groups at N = 8, the 32B and 72B shapes one TP8 group."""
    sys.path.insert(0, ROOT)
    import bench
    from furnace_b200 import synth

    want = {"c3": {1: 1, 2: 2, 4: 4, 8: 4}, "c4": {8: 8}, "c5": {2: 2, 8: 8}, "c1": {8: 2}, "c2": {4: 2, 8: 2}}
    for name, cases in want.items():
        spec = synth.spec(name)
        for n, tp in cases.items():
            got = bench.default_tp(n, spec)
            assert got == tp, (name, n, got)
            assert n % got == 0 and spec.n_heads % got == 0 and spec.n_kv_heads % got == 0


def test_ncu_traffic_only_for_the_workload_it_was_captured_on():
    sys.path.insert(0, ROOT)
    import bench

    d = bench.ncu_traffic("c3", None, 1)
    assert d is not None and d["dram_bytes_per_launch"] > 0
    assert bench.ncu_traffic("c3", 2, 1) is None  # layer-truncated
    assert bench.ncu_traffic("c3", None, 2) is None  # tensor-parallel share
    assert bench.ncu_traffic("c5", None, 1) is None
