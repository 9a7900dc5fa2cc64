"""bench.py's reference arm on the host (no GPU): the JSON line the driver reads."""
import json
import os
import subprocess
import sys


def test_bench_reference_arm_prints_the_contract_line():
    """bench.py --impl reference (the CPU restatement timed on the host) prints one JSON line with
    the fields the driver reads: the metric, value, unit and direction, the cpu_baseline object
    describing the run, and an e2e object with no host/device copies."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "toy", "--steps", "1",
                          "--warmup", "3"], cwd=root, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["warmup"] >= 3 and d["steps"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_bench_reference_arm_other_ranks_exit_without_work():
    """Under torchrun only rank 0 runs the reference arm and prints; the other ranks exit 0."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "toy", "--gpus", "2",
                          "--steps", "1", "--warmup", "3"], cwd=root, env=env, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    assert not [l for l in out.stdout.splitlines() if l.startswith("{")]
