"""The native timing / correctness harness (lib/mllb200_harness): the
reference's harness pattern (benchmark/q4_compare.c) around this library --
graphs of serialised reps, ABBA arms, clocks per sample, red zones and the
tolerance check after timing, the reference's exit codes."""
import json
import subprocess

import pytest

import ref_fixtures as rfx
from mojo_llm_lab_b200 import build

HARNESS = build.HARNESS


def run(*args, timeout=300):
    return subprocess.run([str(HARNESS), *map(str, args)], capture_output=True, text=True, timeout=timeout)


def test_usage_and_bad_input_exit_codes(tmp_path):
    assert HARNESS.exists(), "build() makes lib/mllb200_harness"
    assert run().returncode == 2
    assert run(tmp_path, "--op", "softmax").returncode == 2
    assert run(tmp_path, "--rows", "100").returncode == 2  # not a multiple of 64
    assert run(tmp_path).returncode == 4                    # no activations.bin
    rfx.write_q4_matvec_fixtures(tmp_path)
    (tmp_path / "weights.bin").write_bytes((tmp_path / "weights.bin").read_bytes()[:-1])
    assert run(tmp_path).returncode == 4                    # weights not whole rows


@pytest.mark.gpu
@pytest.mark.parametrize("op,options", [("matvec", {}), ("gate_up", {"gate_up": True}),
                                        ("gate_up", {"gate_up": True, "factor_seed": 739,
                                                     "activation_scale_seed": 971})])
def test_harness_times_both_arms_and_checks_them(tmp_path, op, options):
    rfx.write_q4_matvec_fixtures(tmp_path, **options)
    proc = run(tmp_path, "--op", op, "--rows", 9728, "--reps", 16, "--rounds", 4)
    assert proc.returncode == 0, proc.stderr[-2000:]
    out = json.loads(proc.stdout)
    assert out["correct"] is True and out["red_zones"] == "intact"
    assert len(out["samples"]) == 16
    assert [s["arm"] for s in out["samples"][:4]] == ["native", "compat", "compat", "native"]
    for s in out["samples"]:
        assert s["gpu_us_per_operation"] > 0 and s["sm_clock_after_mhz"] > 0
    assert out["worst_error_over_tolerance"]["native"] < 0.5
    assert out["native_us_per_operation"] > 0 and out["compat_us_per_operation"] > 0
