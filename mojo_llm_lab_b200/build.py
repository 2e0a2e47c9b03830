"""Build the sm_100a artefacts in-tree with nvcc.

* lib/libmllb200.so        -- the C ABI of include/mllb200.h (csrc/capi.cu, one
                              translation unit holding every kernel)
* lib/mllb200_compat.cubin -- reference-named kernel entries for driver-API
                              harnesses (csrc/compat.cu)
* lib/libmllb200_interpose.so -- LD_PRELOAD library that sends GGML's fused
                              Q4_K gate/up launch to libmllb200.so
                              (csrc/interpose.cpp, host code only)
* lib/mllb200_harness       -- native timing / correctness harness (CUDA
                              graphs of serialised reps, ABBA arms, NVML
                              clocks, red zones; csrc/harness.cpp)

Both target `-gencode arch=compute_100a,code=sm_100a` only (B200).  The build
is incremental on source mtimes; `python -m mojo_llm_lab_b200.build` forces it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "lib"
INCLUDE = ROOT / "include"
LIB = LIBDIR / "libmllb200.so"
CUBIN = LIBDIR / "mllb200_compat.cubin"
INTERPOSE = LIBDIR / "libmllb200_interpose.so"
HARNESS = LIBDIR / "mllb200_harness"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xptxas", "-v", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build mojo_llm_lab_b200")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.cpp")) + [INCLUDE / "mllb200.h"]


def _stale(target: Path) -> bool:
    if not target.exists():
        return True
    newest = max(p.stat().st_mtime for p in _sources())
    return target.stat().st_mtime < newest


def _run(cmd: list[str], log: Path, verbose: bool) -> None:
    env = dict(os.environ)
    # nvcc picks its host compiler from PATH; a CC/CXX override pointing at a
    # wrapper without its spec files must not leak in.
    env.pop("CC", None)
    env.pop("CXX", None)
    proc = subprocess.run(cmd, capture_output=True, text=True, env=env)
    log.write_text(" ".join(cmd) + "\n\n" + proc.stdout + proc.stderr)
    if verbose:
        sys.stderr.write(proc.stderr)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr[-4000:]}")


def build(force: bool = False, verbose: bool = False) -> dict:
    LIBDIR.mkdir(exist_ok=True)
    built = {}
    if force or _stale(LIB):
        tmp = LIB.with_suffix(".so.tmp")
        _run([nvcc(), *COMMON, *ARCH, "-Xcompiler", "-fPIC", "-shared", "-o", str(tmp), str(CSRC / "capi.cu")],
             LIBDIR / "build_lib.log", verbose)
        tmp.replace(LIB)
        built["lib"] = str(LIB)
    if force or _stale(INTERPOSE) or INTERPOSE.stat().st_mtime < LIB.stat().st_mtime:
        tmp = INTERPOSE.with_suffix(".so.tmp")
        cuda_inc = Path(nvcc()).resolve().parent.parent / "include"
        _run([shutil.which("g++") or "g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-I{INCLUDE}", f"-I{cuda_inc}",
              "-o", str(tmp), str(CSRC / "interpose.cpp"), f"-L{LIBDIR}", "-lmllb200", "-ldl",
              "-Wl,-rpath,$ORIGIN"], LIBDIR / "build_interpose.log", verbose)
        tmp.replace(INTERPOSE)
        built["interpose"] = str(INTERPOSE)
    if force or _stale(HARNESS) or HARNESS.stat().st_mtime < LIB.stat().st_mtime:
        tmp = HARNESS.with_suffix(".tmp")
        _run([nvcc(), "-O2", "-std=c++17", f"-I{INCLUDE}", "-o", str(tmp), str(CSRC / "harness.cpp"),
              f"-L{LIBDIR}", "-lmllb200", "-ldl",
              "-Xlinker", "-rpath,$ORIGIN"], LIBDIR / "build_harness.log", verbose)
        tmp.replace(HARNESS)
        built["harness"] = str(HARNESS)
    if force or _stale(CUBIN):
        tmp = CUBIN.with_suffix(".cubin.tmp")
        _run([nvcc(), *COMMON, *ARCH, "-cubin", "-o", str(tmp), str(CSRC / "compat.cu")],
             LIBDIR / "build_cubin.log", verbose)
        tmp.replace(CUBIN)
        built["cubin"] = str(CUBIN)
    return built


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
