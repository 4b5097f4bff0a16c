"""The benchmark's reference arm runs on CPU and prints the contract's JSON line.

`bench.py --impl reference` times the reference's CPU path (the oracle
restating references.py) on a row sample of the headline workload; it needs
no GPU, so its output contract is checked here (about 15 s).
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import ROOT

REQUIRED = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
            "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "e2e",
            "cpu_baseline", "gpu_launches"}


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "3"], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=600, check=True)
    lines = [line for line in out.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert REQUIRED <= set(d)
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["value"] > 0
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["workload"].startswith("llama_mlp_block")


def test_reference_arm_is_silent_on_other_ranks():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--gpus", "2", "--steps", "1", "--warmup", "3"], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=300, check=True)
    assert out.stdout.strip() == ""


def test_bench_rejects_fewer_than_three_warmup_steps():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--warmup", "2"], cwd=ROOT,
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 2 and "--warmup must be >= 3" in out.stderr
