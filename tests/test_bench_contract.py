"""The benchmark's driver contract on CPU: the reference arm (the CPU algorithm through the oracle
port) prints one JSON line with the metric, config and baseline fields the driver reads."""

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line():
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
           "--warmup", "3", "--ref-targets", "1"]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=REPO)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"].startswith("segmented-attn TFLOP/s & ms/image")
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]


def test_warmup_below_three_is_rejected():
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
           "--warmup", "2"]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=REPO)
    assert res.returncode != 0
    assert "--warmup must be >= 3" in res.stderr


def test_reference_arm_loads_no_code_of_this_package():
    """The reference arm times the reference's CPU path on the recorded schedule: neither the
    package nor its native library may be loaded in that process."""
    code = (
        "import sys, types, bench\n"
        "args = types.SimpleNamespace(workload='c5', shard='auto', global_rows=64, budget=0.10,\n"
        "    model='2b', rows=2, exchange='p2p', ref_layers=1, ref_targets=1, steps=1, warmup=3)\n"
        "bench.run_reference(args, 0, 1)\n"
        "bad = [m for m in sys.modules if m.startswith('heatkv_b200')]\n"
        "so = [m for m in bench._loaded_native() if 'heatkv' in m]\n"
        "assert not bad and not so, (bad, so)\n"
        "print('clean')\n")
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd=REPO)
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip().endswith("clean")
    line = json.loads(res.stdout.strip().splitlines()[0])
    assert line["cpu_baseline"]["sample"].startswith("2B 10% layers/targets 0:8..8")
