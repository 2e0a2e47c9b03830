"""bench.py's reference arm on the CPU: `--impl reference` times the oracle
(the reference's CPU algorithm restated) and prints one JSON line carrying the
same metric and unit as the GPU arm, with its cpu_baseline and e2e; under a
multi-rank launch only rank 0 runs and prints."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def run_bench(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "3", *args], capture_output=True, text=True, cwd=ROOT, env=env, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    return [json.loads(line) for line in proc.stdout.splitlines() if line.startswith("{")]


@pytest.mark.parametrize("args,unit", [
    ([], "GB/s"),
    (["--workload", "attention"], "GB/s"),
    (["--workload", "attention", "--kv", "q4_0"], "GB/s"),
    (["--workload", "imrope"], "us/op"),
    (["--workload", "prefill"], "int8 TOP/s"),
    (["--workload", "q8_1"], "us/op"),
    (["--workload", "q8_1_batched"], "GB/s"),
])
def test_reference_arm_prints_the_contract_line(args, unit):
    lines = run_bench(args)
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference"
    assert line["unit"] == unit and line["value"] > 0
    assert line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 3
    cpu = line["cpu_baseline"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["sample"]
    assert cpu["value"] == pytest.approx(line["value"], rel=1e-3)
    e2e = line["e2e"]
    assert e2e["unit"] == unit and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in line["config"]
    if "--kv" in args:
        assert "Q4_0" in line["metric"]


def test_reference_arm_prints_on_rank_zero_only():
    assert run_bench(["--workload", "attention"], {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []


def test_reference_arm_reports_every_cpu_arm_and_the_gpu_arms_config():
    """Default workload: the C port on all threads (the contract's value), the
    C port on 1 thread and the pure-Python path on 1 thread beside it; the
    config dict is the one the GPU arm prints."""
    sys.path.insert(0, str(ROOT))
    import bench
    line = run_bench([])[0]
    others = line["cpu_baseline"]["others"]
    assert [o["cores"] for o in others] == [1, 1]
    assert "pyport" in others[1]["sample"] and all(o["value"] > 0 for o in others)
    assert line["config"] == bench.matvec_config("q4k_matvec", 1, True)


@pytest.mark.parametrize("workload,config", [
    ("imrope", lambda bench: bench.imrope_config(False, 1)),
    ("q8_1", lambda bench: bench.q8_1_config(False, 2560, 1)),
])
def test_reference_arm_config_is_the_gpu_arms(workload, config):
    sys.path.insert(0, str(ROOT))
    import bench
    assert run_bench(["--workload", workload])[0]["config"] == config(bench)


def test_e2e_split_keeps_every_item_and_both_joins_inside_the_step():
    """The overlapped e2e step's split: inputs [0, n_in) before the chain,
    outputs [tail, n) after it; no split with collectives in the step."""
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.e2e_split(50) == (15, 42)
    assert bench.e2e_split(400) == (40, 352)
    assert bench.e2e_split(132) == (40, 111)
    assert bench.e2e_split(2) == (2, 1)
    assert bench.e2e_split(1) == (1, 0)
    assert bench.e2e_split(400, overlap=False) == (400, 0)
    for n in range(1, 600):
        n_in, tail = bench.e2e_split(n)
        assert 1 <= n_in <= n and 0 <= tail < n
