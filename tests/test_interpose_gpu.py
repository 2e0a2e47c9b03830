"""The LD_PRELOAD drop-in for GGML's fused Q4_K gate/up launch.

tests/interpose/fake_ggml.cu stands in for a GGML CUDA build: a kernel with
GGML's name, parameters and launch shape whose own body only writes NaN.  Run
under lib/libmllb200_interpose.so with MLLB_REPLACE=1 its outputs must be
this library's up * silu(gate) (within 1e-5 + 1e-5 |ref| of the oracle),
eager and inside a captured CUDA graph; an ineligible launch (another GLU) is
left alone; MLLB_VALIDATE catches a wrong GGML output.
"""
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

from gpu_util import assert_within_tolerance
from mojo_llm_lab_b200 import build as B
from mojo_llm_lab_b200 import fixtures as fx

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent / "interpose"
FAKE = HERE / "_build" / "fake_ggml"


@pytest.fixture(scope="module")
def fake_ggml():
    src = HERE / "fake_ggml.cu"
    if not FAKE.exists() or FAKE.stat().st_mtime < src.stat().st_mtime:
        FAKE.parent.mkdir(exist_ok=True)
        subprocess.run([B.nvcc(), "-O2", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "shared", "-o",
                        str(FAKE), str(src)], check=True, capture_output=True)
    B.build()
    return FAKE


def case(tmp_path, orc, rows, width, seed):
    up = fx.seeded_q4k_matrix(rows, width, seed=seed)
    gate = fx.seeded_q4k_matrix(rows, width, seed=seed + 1)
    q8 = orc.quantize_q8_1(fx.seeded_activation(width, seed=seed + 2))
    paths = {name: tmp_path / f"{name}.bin" for name in ("up", "gate", "q8", "out")}
    paths["up"].write_bytes(up.tobytes())
    paths["gate"].write_bytes(gate.tobytes())
    paths["q8"].write_bytes(q8)
    ref = orc.q4k_gate_up(up, gate, q8, rows, width)[2]
    return paths, ref


def run(fake, paths, rows, width, env_extra, mode="eager", launches=1):
    env = dict(os.environ)
    env.update(env_extra)
    cmd = [str(fake), str(rows), str(width), str(paths["up"]), str(paths["gate"]), str(paths["q8"]),
           str(paths["out"]), mode, str(launches)]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=120)
    out = np.fromfile(paths["out"], dtype=np.float32) if proc.returncode == 0 else None
    return proc, out


def counts(stderr):
    line = [l for l in stderr.splitlines() if l.startswith("mllb_interpose matched=")][-1]
    return dict(kv.split("=") for kv in line.split()[1:])


@pytest.mark.parametrize("rows,width", [(9728, 2560), (6144, 2048), (2048, 4096)])
def test_replaces_ggml_launch(fake_ggml, tmp_path, orc, rows, width):
    paths, ref = case(tmp_path, orc, rows, width, seed=rows)
    proc, out = run(fake_ggml, paths, rows, width, {})
    assert proc.returncode == 0, proc.stderr
    assert np.isnan(out).all(), "the stand-in kernel writes NaN"
    proc, out = run(fake_ggml, paths, rows, width,
                    {"LD_PRELOAD": str(B.INTERPOSE), "MLLB_REPLACE": "1"}, launches=3)
    assert proc.returncode == 0, proc.stderr
    assert_within_tolerance(out, ref, "replaced gate/up")
    c = counts(proc.stderr)
    assert c["matched"] == "3" and c["eligible"] == "3" and c["replaced"] == "3", proc.stderr


def test_replaces_inside_graph_capture(fake_ggml, tmp_path, orc):
    rows, width = 9728, 2560
    paths, ref = case(tmp_path, orc, rows, width, seed=5)
    proc, out = run(fake_ggml, paths, rows, width, {"LD_PRELOAD": str(B.INTERPOSE), "MLLB_REPLACE": "1"},
                    mode="graph", launches=4)
    assert proc.returncode == 0, proc.stderr
    assert_within_tolerance(out, ref, "gate/up replayed from a captured graph")
    c = counts(proc.stderr)
    assert c["replaced"] == "4" and c["captured"] == "3", proc.stderr


def test_ineligible_launch_left_alone(fake_ggml, tmp_path, orc):
    rows, width = 2048, 2560
    paths, _ = case(tmp_path, orc, rows, width, seed=9)
    proc, out = run(fake_ggml, paths, rows, width,
                    {"LD_PRELOAD": str(B.INTERPOSE), "MLLB_REPLACE": "1", "FAKE_GLU": "1"})
    assert proc.returncode == 0, proc.stderr
    assert np.isnan(out).all()
    c = counts(proc.stderr)
    assert c["matched"] == "1" and c["eligible"] == "0" and c["replaced"] == "0", proc.stderr


def test_validation_catches_a_wrong_ggml_output(fake_ggml, tmp_path, orc):
    rows, width = 2048, 2560
    paths, _ = case(tmp_path, orc, rows, width, seed=11)
    proc, _ = run(fake_ggml, paths, rows, width, {"LD_PRELOAD": str(B.INTERPOSE), "MLLB_VALIDATE": "1"})
    assert proc.returncode != 0
    assert "validation mismatch" in proc.stderr
