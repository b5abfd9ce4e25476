"""The benchmark's reference arm (`bench.py --impl reference`) on the host cores: one JSON line in
the contract's shape, on the same metric, unit and workload as the GPU arm, with a CPU baseline
and an e2e figure that moves no bytes; under torchrun only rank 0 reports. It times the
reference's CPU algorithm (the oracle's restatement) and run.c when that was built, so it needs no
GPU."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def run_bench(env_extra):
    env = dict(os.environ, **env_extra)
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    return [json.loads(line) for line in res.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    import bench
    lines = run_bench({"RANK": "0", "WORLD_SIZE": "1"})
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 0
    assert d["config"]["workload"] == bench.workload_config(bench.WORKLOAD)["workload"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_reports_on_rank_zero_only():
    assert run_bench({"RANK": "1", "WORLD_SIZE": "2"}) == []
