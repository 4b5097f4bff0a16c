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


def _bench_module():
    import importlib.util

    spec = importlib.util.spec_from_file_location("col_bench", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_parity_check_flags_a_planted_error():
    """The benchmark's parity block: identical rows pass; one element moved
    past the bf16 bar (2e-2 + 2e-2 |expected|) is counted as a violation."""
    import torch

    bench = _bench_module()
    g = torch.Generator()
    g.manual_seed(11)
    expected = torch.randn(8, 64, generator=g).to(torch.bfloat16)
    same = bench.parity_check(expected.clone(), expected, 8)
    assert same["ok"] and same["violations"] == 0 and same["max_abs_err"] == 0.0
    planted = expected.clone()
    planted[3, 7] = float(expected[3, 7]) + 0.05 + 0.05 * abs(float(expected[3, 7]))
    bad = bench.parity_check(planted, expected, 8)
    assert not bad["ok"] and bad["violations"] == 1 and bad["max_err_over_bound"] > 1.0


def test_benchmark_inputs_are_shared_by_every_arm_and_shard():
    """Each rank's packed shard holds exactly its gate and up rows of the one
    seeded W that the CPU arms use (checked on a reduced N for speed)."""
    import torch

    bench = _bench_module()
    bench.M, bench.K, bench.N = 64, 32, 96
    full = bench.make_inputs(1, 0, "cpu")
    for world in (2, 4):
        for rank in range(world):
            part = bench.make_inputs(world, rank, "cpu")
            nl = 96 // world
            assert torch.equal(part["x"], full["x"]) and torch.equal(part["w_norm"], full["w_norm"])
            gate = full["packed"][rank * nl:(rank + 1) * nl]
            up = full["packed"][96 + rank * nl:96 + (rank + 1) * nl]
            assert torch.equal(part["packed"], torch.cat((gate, up)))
