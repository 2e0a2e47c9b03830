"""Benchmark of the decode hot path on B200 (driver contract: one JSON line).

Default workload: the Q4_K x Q8_1 matvec, N = 4096 rows, K = 2560 (10 Q4_K
super-blocks per row), fp16 d ~ U(1e-3, 1e-2), dmin ~ U(0, 5e-3), uniform
6-bit scales/mins and nibbles, x ~ N(0, 1) quantised to Q8_1.  Metric: HBM
GB/s of the matvec (algorithmic bytes: weights 5,898,240 + activation 2,880 +
output 16,384 = 5,917,504 per launch).

One step = R back-to-back matvec launches over R distinct weight copies and R
distinct activations (R * 5.9 MB > 2 x the 126 MB L2, so every launch reads
its weights from HBM; no flush needed).  `value` = bytes / device time with
everything resident; `e2e` = the same launches through the public Python API
(mojo_llm_lab_b200.ops) with each step's fp32 activations copied from pinned
host memory, quantised on the device, and the outputs copied back.

--impl reference times the CPU restatement of the reference's path (the
oracle in oracle/, OpenMP over all host threads) on a bounded sample of the
same workload.  Multi-GPU (torchrun): this matvec is a "stay on one GPU" op,
so N ranks run N independent replicas (weak scaling, no collective).

--workload decode: the 36-layer synthetic Qwen3-style decode (hidden 2560,
32/8 heads of 128, SwiGLU 9728, vocab 151936; Q4_K layers, Q6_K output; fp16
KV cache prefilled with N(0, 1) at context 4096).  One step = 128 greedy
tokens from the prefilled context (the state reset on the device at the
start of the step), replaying one captured CUDA graph per token.  Metric:
tokens/s of the whole job; with N ranks the gate/up and vocabulary matvecs
are row-sharded (NCCL all-gather / all-reduce) and every rank decodes the
same token stream (strong scaling).

--workload imrope: the fused RMSNorm + gamma + IMROPE op on one Q tensor (32
heads x 128 fp32, gamma[128], runtime fp32 theta scale 0x3f492c27, positions
(7, 13, 29, 0)): µs/op over a CUDA graph of 128 serial launches on 128
distinct input copies (the reference's measurement, benchmark/bench.c:33);
--workload imrope_batched: the same op over 4096 tokens x 32 heads (134 MB
per launch, HBM-bound throughput mode).  One GPU; N ranks are replicas.

--workload prefill: the batched-token form, 512 tokens x 4096 x 2560 Q4_K on
the tensor cores (mllb_q4k_matmul_tokens); metric int8 TOP/s.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0

WORKLOADS = {
    # the headline metric's configuration: Q4_K x Q8_1, 4096 x 2560
    "q4k_matvec": dict(kind="q4k", rows=4096, k=2560, kernel="resident_q4k_kernel<10>",
                       profile="q4k_matvec_n4096_k2560"),
    # fused gate/up, two 9728x2560 matrices, outputs up, gate, up*silu(gate)
    "gate_up": dict(kind="gate_up", rows=9728, k=2560, kernel="team_stream_kernel<Q4kFormat,10,2,4,6,3>",
                    profile="q4k_gate_up_n9728_k2560"),
    # the Q5_K matvec at the headline shape (4096 x 2560)
    "q5k_matvec": dict(kind="q5k", rows=4096, k=2560, kernel="resident_q5k_kernel<10>",
                       profile="q5k_matvec_n4096_k2560"),
    # Q6_K vocabulary projection 151936x2560
    "q6k_vocab": dict(kind="q6k", rows=151936, k=2560, kernel="team_stream_kernel<Q6kFormat,10,1,4,6,5>",
                      profile="q6k_vocab_n151936_k2560"),
}


DECODE = dict(kind="decode", profile="decode_36layer_ctx4096")


def weight_bytes(kind: str, rows: int, k: int) -> int:
    per_row = k // 256 * {"q6k": 210, "q5k": 176}.get(kind, 144)
    return rows * per_row * (2 if kind == "gate_up" else 1)


def algorithmic_bytes(kind: str, rows: int, k: int) -> int:
    """Bytes one launch must move: weights + Q8_1 activation + fp32 outputs."""
    outputs = 3 if kind == "gate_up" else 1
    return weight_bytes(kind, rows, k) + k // 32 * 36 + outputs * rows * 4


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:  # noqa: BLE001
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(name: str):
    """Per-launch DRAM bytes from the committed ncu summary, if present."""
    p = ROOT / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples (every 20 ms) around the timed region.

    Started under load shortly before the timed region and stopped right after
    it (the recipe's `nvidia-smi ... -lms` line)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        samples = [[c.strip() for c in ln.split(",")] for ln in self.lines]
        samples = [s for s in samples if len(s) >= 9]
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [v for v in (num(s[1]) for s in samples) if v is not None]
        smax = [v for v in (num(s[2]) for s in samples) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in samples for i in range(4) if s[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(samples),
                "window": "every 20 ms over ~1 s of the same graph replayed just before the timed region, "
                          "and the timed region"}


# A step lasts at least this long: the clock sampler's nvidia-smi queries
# (every 20 ms) can stall the GPU for tens of microseconds, which must stay a
# small fraction of a step.
STEP_TARGET_MS = 1.0


def passes_for(graph, stream, world: int, device) -> int:
    """Passes over a workload's copies per step so that a step lasts about
    STEP_TARGET_MS: one replay of `graph` (one pass) is timed on the device;
    at N ranks the maximum is taken (every rank must replay alike)."""
    import torch
    import torch.distributed as dist
    for _ in range(2):
        graph.replay()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(3):
        graph.replay()
    b.record(stream)
    torch.cuda.synchronize()
    pass_ms = a.elapsed_time(b) / 3
    passes = max(1, int(-(-STEP_TARGET_MS // max(pass_ms, 1e-3))))
    if world > 1:
        t = torch.tensor([passes], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        passes = int(t.item())
    return passes


def preroll(graph, seconds: float = 1.0) -> None:
    """Replay `graph` for about `seconds` (untimed) so that the clock samples
    taken around the timed region describe the same load.  For graphs with no
    collectives (every rank may replay a different number of times)."""
    import torch

    t0 = time.perf_counter()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    n = max(1, int(seconds / max((time.perf_counter() - t0) / 3, 1e-6)))
    for _ in range(n):
        graph.replay()
    torch.cuda.synchronize()


def e2e_split(n: int, overlap: bool = True) -> tuple[int, int]:
    """(items copied in before the chain, first item whose output is copied
    out after it) for an overlapped e2e step of n items: ~30 % in / ~16 % out
    for short steps, ~10 % / ~12 % from 200 items on (the rest of the inputs
    still arrives well before the chain reaches it; 400-launch Q4_K step:
    2214-2223 against 2191-2197 GB/s with the short-step fractions; the
    132-launch gate/up step, whose outputs are 117 KB a launch, needs the
    longer tail for its copy back: 3157 against 3222-3244)."""
    if not overlap:
        return n, 0
    f_in, f_out = (0.1, 0.12) if n >= 200 else (0.3, 0.16)
    n_in = max(1, round(f_in * n)) if n >= 10 else n
    tail = n - max(1, round(f_out * n)) if n >= 2 else 0
    return n_in, tail


def overlapped_e2e(torch, device, stream, n, copy_in, op, copy_out, warmup, steps, overlap=True,
                   before_timing=None):
    """Device time (ms) of one end-to-end step over n independent items:
    pinned H2D of their inputs, the op on each (a PDL chain), D2H of their
    outputs, all captured in one CUDA graph.  The copies overlap the chain
    with two stream joins only: the first inputs (e2e_split) come in on the
    compute stream, the rest on a side stream before the chain reaches them,
    and the outputs of all but the last few go back on a side stream while
    those run.  copy_in(a, b) / copy_out(a, b) issue the copies of items
    [a, b) on the current stream; op(i) launches item i (item 0 and item
    n_in start their input halves).  overlap=False (steps with collectives):
    all inputs, the chain, all outputs, in order.  Returns (ms, items copied
    in before the chain, items copied out after it).  (Five equal chunks with
    a join each measured 1666-1687 GB/s against 1851 for this arrangement on
    the Q4_K matvec, one box; with fewer than 10 items all inputs come in
    first and only the last output's copy stays exposed.)"""
    n_in, tail = e2e_split(n, overlap)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = torch.cuda.Event()

    def step():
        cur = torch.cuda.current_stream(device)
        copy_in(0, n_in)
        if n_in < n:
            s_in.wait_stream(cur)
            with torch.cuda.stream(s_in):
                copy_in(n_in, n)
                ev_in.record(s_in)
        for i in range(n):
            if i == n_in:
                cur.wait_event(ev_in)
            if i == tail and tail > 0:
                s_out.wait_stream(cur)
                with torch.cuda.stream(s_out):
                    copy_out(0, tail)
            op(i)
        copy_out(tail, n)
        if tail > 0:
            cur.wait_stream(s_out)

    step()  # eager once: launch attributes set outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if before_timing:
        before_timing()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del g  # before any process group goes away: the graph may hold collectives
    return ms, n_in, n - tail


# ----------------------------------------------------------------------------- inputs

def host_weights(kind: str, rows: int, k: int, seed: int):
    from mojo_llm_lab_b200 import fixtures as fx
    if kind == "q6k":
        return [fx.seeded_q6k_matrix(rows, k, seed)]
    if kind == "q5k":
        return [fx.seeded_q5k_matrix(rows, k, seed)]
    if kind == "gate_up":
        return [fx.seeded_q4k_matrix(rows, k, seed), fx.seeded_q4k_matrix(rows, k, seed + 1)]
    return [fx.seeded_q4k_matrix(rows, k, seed)]


def oracle_outputs(kind: str, ws, act: bytes, rows: int, k: int, threads: int = 0):
    import oracle
    if kind == "q6k":
        return [oracle.q6k_matvec(ws[0], act, rows, k, threads)]
    if kind == "q5k":
        return [oracle.q5k_matvec(ws[0], act, rows, k, threads)]
    if kind == "gate_up":
        return list(oracle.q4k_gate_up(ws[0], ws[1], act, rows, k, threads))
    return [oracle.q4k_matvec(ws[0], act, rows, k, threads)]


# ----------------------------------------------------------------------------- reference arm

def cpu_reference(workload: str, target_s: float = 10.0, threads: int = 0):
    """Time the oracle (CPU restatement of the reference's path) on a bounded
    sample: whole operations of the workload, repeated for ~target_s.
    threads = 0: all host threads (OpenMP over rows)."""
    import oracle
    from mojo_llm_lab_b200 import fixtures as fx

    wl = WORKLOADS[workload]
    kind, rows, k = wl["kind"], wl["rows"], wl["k"]
    threads = threads or os.cpu_count() or 1
    ws = host_weights(kind, rows, k, seed=1)
    act = oracle.quantize_q8_1(fx.seeded_activation(k, seed=2))
    t0 = time.perf_counter()
    oracle_outputs(kind, ws, act, rows, k, threads)  # warm
    first = time.perf_counter() - t0
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.quantize_q8_1(fx.seeded_activation(k, seed=3 + reps))
        oracle_outputs(kind, ws, act, rows, k, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= target_s or reps >= 10_000 or (first > target_s / 2):
            break
    per_op = algorithmic_bytes(kind, rows, k)
    return {"value": reps * per_op / el / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{reps} x ({wl['kind']} {rows}x{k} incl. Q8_1 quantise) in {el:.1f} s "
                      f"(oracle/oracle.c, OpenMP {threads} threads, fsum per row)",
            "seconds_per_op": el / reps}


def cpu_python_reference(workload: str, target_s: float = 6.0):
    """The reference's own CPU path, pure Python on one core (oracle/pyport.py,
    the same float64 arithmetic as tests/q4_reference.py:36-47): whole rows for
    ~target_s, scaled to the workload's rows.  None for formats the reference's
    Python has no code for (Q5_K, Q6_K)."""
    import math

    import oracle
    from oracle import pyport
    from mojo_llm_lab_b200 import fixtures as fx

    wl = WORKLOADS[workload]
    kind, rows, k = wl["kind"], wl["rows"], wl["k"]
    if kind not in ("q4k", "gate_up"):
        return None
    sample_rows = rows
    mats = [w.tobytes() for w in host_weights(kind, sample_rows, k, seed=1)]
    act = oracle.quantize_q8_1(fx.seeded_activation(k, seed=2))
    row_bytes = k // 256 * 144
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < target_s and done < sample_rows:
        r = slice(done * row_bytes, (done + 1) * row_bytes)
        vals = [pyport.dot_q4_q8(m[r], act) for m in mats]
        if kind == "gate_up":
            up, gate = vals
            vals.append(up * (gate / (1.0 + math.exp(-gate))))
        done += 1
    el = time.perf_counter() - t0
    per_op_s = el / done * rows
    return {"value": algorithmic_bytes(kind, rows, k) / per_op_s / 1e9, "unit": "GB/s", "cores": 1,
            "kind": "port", "seconds_per_op": per_op_s,
            "sample": f"{done} of {rows} rows in {el:.1f} s, scaled to all rows (oracle/pyport.py: the "
                      f"reference's pure-Python dot_q4_q8 arithmetic, 1 thread)"}


def cpu_baselines(workload: str, target_s: float = 10.0) -> dict:
    """The contract's cpu_baseline (the C port on all host threads) with the
    other CPU arms beside it: the C port on 1 thread and the reference's own
    pure-Python path on 1 thread."""
    main = cpu_reference(workload, target_s=target_s)
    line = {kk: main[kk] for kk in ("value", "unit", "cores", "kind", "sample")}
    others = []
    one = cpu_reference(workload, target_s=min(4.0, target_s), threads=1)
    others.append({kk: one[kk] for kk in ("value", "unit", "cores", "kind", "sample")})
    py = cpu_python_reference(workload)
    if py is not None:
        others.append({kk: py[kk] for kk in ("value", "unit", "cores", "kind", "sample")})
    line["others"] = others
    line["host"] = host_cpu()
    return line


def host_cpu() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return f"{ln.split(':', 1)[1].strip()} ({os.cpu_count()} threads)"
    except OSError:
        pass
    return f"{os.cpu_count()} threads"


def matvec_config(workload: str, world: int, pdl: bool, copies: int = 0) -> dict:
    """The config dict of a matvec workload, the same in both arms."""
    wl = WORKLOADS[workload]
    kind, rows, k = wl["kind"], wl["rows"], wl["k"]
    sharded = kind in ("gate_up", "q6k") and world > 1
    my_rows = rows // world if sharded else rows
    wbytes = weight_bytes(kind, my_rows, k)
    copies = copies or max(2, -(-int(2.2 * L2_BYTES) // wbytes))
    return {"workload": describe(workload), "rows": rows, "k": k, "weight_copies": copies,
            "bytes_per_op": algorithmic_bytes(kind, rows, k),
            "l2": f"{copies} distinct weight copies ({copies * wbytes / 2**20:.0f} MiB per GPU) > 2x L2 per pass "
                  f"over them; no flush; a step is as many passes as make ~{STEP_TARGET_MS:g} ms",
            "parallelism": (f"rows/{world} per rank + NCCL all-gather" if sharded else
                            (f"replicas x{world}" if world > 1 else "single GPU")),
            "pdl": pdl}


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    ref = cpu_reference(args.workload, target_s=max(3.0, min(30.0, 1.5 * args.steps)))
    base = cpu_baselines(args.workload, target_s=3.0)
    base.update({kk: ref[kk] for kk in ("value", "unit", "cores", "kind", "sample")})
    line = {"metric": f"{describe(args.workload)} HBM GB/s", "value": round(ref["value"], 4), "unit": "GB/s",
            "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ref["seconds_per_op"] * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8/s8 dp4a, f64 accumulate",
            "data": "synthetic (seeded; the reference benchmark's value distributions)",
            "config": matvec_config(args.workload, world, not args.no_pdl, args.copies),
            "cpu_baseline": base,
            "e2e": {"value": round(ref["value"], 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def describe(workload: str) -> str:
    wl = WORKLOADS[workload]
    return {"q4k": f"Q4_K x Q8_1 matvec N={wl['rows']} K={wl['k']}",
            "gate_up": f"fused gate/up Q4_K x Q8_1 2x{wl['rows']}x{wl['k']} + SwiGLU",
            "q6k": f"Q6_K x Q8_1 vocab matvec N={wl['rows']} K={wl['k']}",
            "q5k": f"Q5_K x Q8_1 matvec N={wl['rows']} K={wl['k']}"}[wl["kind"]]


# ----------------------------------------------------------------------------- our arm

def run_ours(args, rank: int, world: int):
    import torch
    import torch.distributed as dist

    from mojo_llm_lab_b200 import fixtures as fx
    from mojo_llm_lab_b200 import ops

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    wl = WORKLOADS[args.workload]
    kind, rows, k = wl["kind"], wl["rows"], wl["k"]
    # The plain Q4_K matvec stays on one GPU: N ranks are replicas.  gate/up and the
    # vocab projection are row-sharded with an all-gather of the outputs.
    sharded = kind in ("gate_up", "q6k") and world > 1
    if sharded and rows % world:
        raise SystemExit(f"{rows} rows do not split over {world} ranks")
    my_rows = rows // world if sharded else rows
    n_out = 3 if kind == "gate_up" else 1
    per_op = algorithmic_bytes(kind, rows, k)              # whole operation (all ranks' rows)
    my_bytes = algorithmic_bytes(kind, my_rows, k)          # this rank's launch
    wbytes = weight_bytes(kind, my_rows, k)
    copies = args.copies or max(2, -(-int(2.2 * L2_BYTES) // wbytes))
    pdl = not args.no_pdl

    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    torch.cuda.set_stream(stream)

    from mojo_llm_lab_b200.shard import RowShard, all_gather_rows
    shard = RowShard(rows, world if sharded else 1, rank if sharded else 0)
    full = host_weights(kind, rows, k, seed=1)
    row_bytes = weight_bytes(kind, 1, k) // (2 if kind == "gate_up" else 1)
    lo = shard.start
    mine = [shard.slice_weights(torch.from_numpy(w), row_bytes).to(device) for w in full]
    weights = [mine] + [[w.clone() for w in mine] for _ in range(copies - 1)]
    xs_host = np.stack([fx.seeded_activation(k, seed=100 + i) for i in range(copies)])
    x_dev = torch.from_numpy(xs_host).to(device)
    # One contiguous Q8_1 buffer: row i is copy i's activation.
    acts = torch.stack([ops.quantize_q8_1(x_dev[i]) for i in range(copies)])
    outs = torch.empty(copies, n_out, my_rows, dtype=torch.float32, device=device)
    gathered = torch.empty(copies, world, n_out, my_rows, dtype=torch.float32, device=device) if sharded else None

    def launch_on(w, a, o, g):
        if kind == "q6k":
            ops.q6_k_q8_1_matvec(w[0], a, o[0], pdl=pdl)
        elif kind == "q5k":
            ops.q5_k_q8_1_matvec(w[0], a, o[0], pdl=pdl)
        elif kind == "gate_up":
            ops.q4k_gate_up(w[0], w[1], a, o[0], o[1], o[2], pdl=pdl)
        else:
            ops.q4_k_q8_1_matvec(w[0], a, o[0], pdl=pdl)
        if sharded:
            dist.all_gather_into_tensor(g.view(-1), o.view(-1))  # = shard.all_gather_rows layout

    def launch(i: int):
        launch_on(weights[i], acts[i], outs[i], gathered[i] if sharded else None)

    def step():
        for i in range(copies):
            launch(i)

    # Correctness gate before timing (copy 0, rank 0's rows, against the oracle).
    if not args.skip_check:
        import oracle
        step()
        torch.cuda.synchronize()
        ref = oracle_outputs(kind, [w[lo * row_bytes:(lo + my_rows) * row_bytes] for w in full],
                             acts[0].cpu().numpy().tobytes(), my_rows, k)
        got = outs[0].cpu().numpy().astype(np.float64)
        for j in range(n_out):
            if not np.all(np.abs(got[j] - ref[j]) <= 1e-5 + 1e-5 * np.abs(ref[j])):
                raise SystemExit(f"correctness gate failed on rank {rank}: output {j} differs from the oracle")
        if sharded:
            g = gathered[0].cpu().numpy()
            if not np.array_equal(g[rank], outs[0].cpu().numpy()):
                raise SystemExit("all-gather placed this rank's rows wrongly")

    # Capture the step in a CUDA graph: host launch overhead out of the device
    # timing.  A step is `passes` passes over the copies (at least ~1 ms).
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    one_pass = torch.cuda.CUDAGraph()
    with torch.cuda.graph(one_pass, stream=stream):
        step()
    passes = passes_for(one_pass, stream, world, device)
    del one_pass
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(passes):
            step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # ~1 s of the same load before the timed region (untimed) so that the
    # clock samples describe it; every rank replays the same number of times
    # (the graph may hold collectives).
    t0 = time.perf_counter()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    n_load = max(1, int(1.0 / max((time.perf_counter() - t0) / 3, 1e-6)))
    if world > 1:
        t = torch.tensor([n_load], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        n_load = int(t.item())
    with ClockSampler(local) as clocks:
        for _ in range(n_load):
            graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        stop.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / args.steps

    # Kernel-only timing of the same launches (no collective) for the roofline.
    if sharded:
        kgraph = torch.cuda.CUDAGraph()
        saved = sharded
        with torch.cuda.graph(kgraph, stream=stream):
            for i in [c for _ in range(passes) for c in range(copies)]:
                w, o = weights[i], outs[i]
                if kind == "q6k":
                    ops.q6_k_q8_1_matvec(w[0], acts[i], o[0], pdl=pdl)
                else:
                    ops.q4k_gate_up(w[0], w[1], acts[i], o[0], o[1], o[2], pdl=pdl)
        for _ in range(args.warmup):
            kgraph.replay()
        ks, ke = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ks.record(stream)
        for _ in range(args.steps):
            kgraph.replay()
        ke.record(stream)
        torch.cuda.synchronize()
        kernel_ms = ks.elapsed_time(ke) / args.steps
        del kgraph, saved
    else:
        kernel_ms = ms
    if world > 1:
        t = torch.tensor([ms, kernel_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, kernel_ms = float(t[0].item()), float(t[1].item())
        dist.barrier()
    torch.cuda.synchronize()
    launch_ms = kernel_ms / (copies * passes)
    achieved = my_bytes / (launch_ms * 1e-3) / 1e9
    job_ops = copies * passes * (1 if sharded else world)
    value = job_ops * per_op / (ms * 1e-3) / 1e9

    # e2e through the public API with host buffers: the same step as the
    # timed one (passes x copies launches over the weight copies), each launch
    # with its own fp32 activation copied from pinned host memory, quantised
    # on the device, and its own outputs (all-gathered) copied back.  Without
    # collectives in the launches (replicas) the copies overlap the chain
    # (overlapped_e2e); the first launch of each input half also quantises
    # that half's activations in one launch.
    n_e = passes * copies
    x_pin = torch.from_numpy(np.tile(xs_host, (passes, 1))).pin_memory()
    x_stage = torch.empty(n_e, k, dtype=torch.float32, device=device)
    e_acts = torch.empty(n_e, acts.shape[1], dtype=acts.dtype, device=device)
    e_outs = torch.empty(n_e, n_out, my_rows, dtype=torch.float32, device=device)
    e_gath = torch.empty(n_e, world, n_out, my_rows, dtype=torch.float32, device=device) if sharded else None
    e_result = e_gath if sharded else e_outs
    out_pin = torch.empty(e_result.shape, dtype=torch.float32).pin_memory()
    overlap = not sharded
    e2e_halves = [0, e2e_split(n_e, overlap)[0]]

    def e2e_in(a, b):
        x_stage[a:b].copy_(x_pin[a:b], non_blocking=True)

    def e2e_op(i):
        if i == 0 or i == e2e_halves[1]:
            b = e2e_halves[1] if i == 0 else n_e
            ops.quantize_q8_1(x_stage[i:b].reshape(-1), e_acts[i:b].reshape(-1))
        launch_on(weights[i % copies], e_acts[i], e_outs[i], e_gath[i] if sharded else None)

    def e2e_out(a, b):
        out_pin[a:b].copy_(e_result[a:b], non_blocking=True)

    e_ms, n_in, n_last = overlapped_e2e(torch, device, stream, n_e, e2e_in, e2e_op, e2e_out, args.warmup,
                                        args.steps, overlap=overlap,
                                        before_timing=dist.barrier if world > 1 else None)
    assert n_in == e2e_halves[1]
    if world > 1:
        t = torch.tensor([e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e_value = n_e * (1 if sharded else world) * per_op / (e_ms * 1e-3) / 1e9
    derr = ops.device_error()
    if derr:
        raise SystemExit(f"device error word set: {derr:#x}")
    del graph
    if world > 1:
        dist.barrier()

    if rank == 0:
        peak, peak_kind = measured_peak()
        cpu = None if args.no_cpu_baseline or world > 1 else cpu_baselines(args.workload, target_s=10.0)
        clk = clocks.summary()
        line = {
            "metric": f"{describe(args.workload)} HBM GB/s", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 6),
            "higher_is_better": True, "scaling": "strong" if sharded else "weak", "vs_baseline": None,
            "dtype": "u8/s8 dp4a, f64 accumulate", "data": "synthetic (seeded; the reference benchmark's value distributions)",
            "config": matvec_config(args.workload, world, pdl, args.copies),
            "passes_per_step": passes, "launches_per_step": copies * passes,
            "us_per_op": round(ms * 1e3 / (copies * passes), 4),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": n_e * k * 4,
                    "d2h_bytes_per_step": int(e_result.numel() * 4), "ms_per_step": round(e_ms, 6),
                    "launches_per_step": n_e,
                    "path": "ops.quantize_q8_1 over the activations (two launches), then ops.<matvec> per launch "
                            "(ctypes C-ABI), with the pinned H2D/D2H copies overlapping the chain "
                            f"(first {n_in} activations in before it, last {n_last} outputs out after it); "
                            "the step captured in a CUDA graph"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": profiled_traffic(wl["profile"]), "kernel": wl["kernel"],
                         "us_per_launch": round(launch_ms * 1e3, 4)},
            "cpu_baseline": cpu,
            "clocks": clk,
            "gpu_launches": args.steps * copies * passes,
        }
        return line


# ----------------------------------------------------------------------------- prefill workload

PREFILL = dict(rows=4096, k=2560, tokens=512, profile="prefill_q4k_n4096_k2560_t512")


def prefill_describe() -> str:
    return f"batched Q4_K x Q8_1 {PREFILL['tokens']} tokens x {PREFILL['rows']}x{PREFILL['k']} (tcgen05 int8)"


def prefill_cpu_reference(target_s: float = 10.0):
    """The oracle's matvec over tokens of the same workload, all host threads, ~target_s."""
    import oracle
    from mojo_llm_lab_b200 import fixtures as fx
    rows, k = PREFILL["rows"], PREFILL["k"]
    threads = os.cpu_count() or 1
    w = fx.seeded_q4k_matrix(rows, k, seed=1)
    reps, t0 = 0, time.perf_counter()
    while True:
        a = oracle.quantize_q8_1(fx.seeded_activation(k, seed=3 + reps))
        oracle.q4k_matvec(w, a, rows, k, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= target_s or reps >= PREFILL["tokens"]:
            break
    return {"value": 2.0 * reps * rows * k / el / 1e12, "unit": "int8 TOP/s", "cores": threads, "kind": "port",
            "sample": f"{reps} tokens x {rows}x{k} (oracle/oracle.c matvec per token incl. Q8_1 quantise, "
                      f"OpenMP {threads} threads) in {el:.1f} s", "seconds": el, "tokens": reps}


def run_prefill_reference(args, rank: int, world: int):
    if rank != 0:
        return
    ref = prefill_cpu_reference(target_s=max(3.0, min(30.0, 1.5 * args.steps)))
    line = {"metric": f"{prefill_describe()} int8 TOP/s", "value": round(ref["value"], 6), "unit": "int8 TOP/s",
            "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ref["seconds"] / ref["tokens"] * PREFILL["tokens"] * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot / f64 sum", "data": "synthetic (seeded)",
            "config": {"workload": prefill_describe()},
            "cpu_baseline": {kk: ref[kk] for kk in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": round(ref["value"], 6), "unit": "int8 TOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_prefill(args, rank: int, world: int):
    """One step = `copies` batched launches over distinct weight and activation copies (> 2x L2)."""
    import torch
    import torch.distributed as dist

    from mojo_llm_lab_b200 import fixtures as fx
    from mojo_llm_lab_b200 import ops

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    rows, k, tokens = PREFILL["rows"], PREFILL["k"], PREFILL["tokens"]
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    w_host = fx.seeded_q4k_matrix(rows, k, seed=1)
    per_copy = w_host.size + tokens * k // 32 * 36
    copies = args.copies or max(2, -(-int(2.2 * L2_BYTES) // per_copy))
    w0 = torch.from_numpy(w_host).to(device)
    ws = [w0] + [w0.clone() for _ in range(copies - 1)]
    gen = torch.Generator(device=device)
    gen.manual_seed(7)
    xs = torch.randn(copies, tokens * k, generator=gen, device=device)
    acts = torch.stack([ops.quantize_q8_1(xs[i]) for i in range(copies)])   # per-token Q8_1 rows
    outs = torch.empty(copies, tokens, rows, dtype=torch.float32, device=device)

    if not args.skip_check:
        import oracle
        ops.q4k_matmul_tokens(ws[0], acts[0], outs[0], k=k)
        torch.cuda.synchronize()
        a_host = acts[0].cpu().numpy().reshape(tokens, -1)
        got = outs[0].cpu().numpy()
        for t in (0, tokens // 2, tokens - 1):
            ref = oracle.q4k_matvec(w_host, a_host[t].tobytes(), rows, k)
            if not np.all(np.abs(got[t] - ref) <= 1e-5 + 1e-5 * np.abs(ref)):
                raise SystemExit(f"correctness gate failed: token {t} differs from the oracle")

    def step():
        for i in range(copies):
            ops.q4k_matmul_tokens(ws[i], acts[i], outs[i], k=k)

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        preroll(graph)
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        stop.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    if world > 1:  # the slowest rank's time
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ops_per_launch = 2.0 * rows * k * tokens
    value = copies * ops_per_launch / (ms * 1e-3) / 1e12

    # e2e: fp32 activations from pinned host memory, one quantiser launch over
    # all tokens, the batched launch, the fp32 outputs back; graph-captured.
    x_pin = xs[0].cpu().pin_memory()
    out_pin = torch.empty(tokens, rows, dtype=torch.float32).pin_memory()
    x_dev = torch.empty(tokens * k, dtype=torch.float32, device=device)
    a_dev = torch.empty(tokens * k // 32 * 36, dtype=torch.uint8, device=device)

    def e2e_step():
        x_dev.copy_(x_pin, non_blocking=True)
        ops.quantize_q8_1(x_dev, a_dev)
        ops.q4k_matmul_tokens(ws[0], a_dev, outs[0], k=k)
        out_pin.copy_(outs[0], non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e_graph, stream=stream):
        e2e_step()
    for _ in range(args.warmup):
        e_graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e_graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    del graph, e_graph
    if ops.device_error():
        raise SystemExit("device error word set")
    if rank == 0:
        peak = None
        try:
            peak = 2.0 * float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
        except Exception:  # noqa: BLE001
            pass
        cpu = None if args.no_cpu_baseline else prefill_cpu_reference(10.0)
        achieved = ops_per_launch / (ms / copies * 1e-3) / 1e12
        line = {
            "metric": f"{prefill_describe()} int8 TOP/s", "value": round(value * world, 3), "unit": "int8 TOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 6),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u8 x s8 tcgen05 MMA (s32 per group), f64 scaling", "data": "synthetic (seeded)",
            "config": {"workload": prefill_describe(), "rows": rows, "k": k, "tokens": tokens,
                       "launches_per_step": copies, "us_per_launch": round(ms * 1e3 / copies, 3),
                       "l2": f"{copies} weight + activation copies ({copies * per_copy / 2**20:.0f} MiB) > 2x L2",
                       "parallelism": "single GPU" if world == 1 else f"replicas x{world}"},
            "e2e": {"value": round(ops_per_launch / (e_ms * 1e-3) / 1e12 * world, 3), "unit": "int8 TOP/s",
                    "h2d_bytes_per_step": tokens * k * 4, "d2h_bytes_per_step": tokens * rows * 4,
                    "ms_per_step": round(e_ms, 6),
                    "path": "ops.quantize_q8_1 + ops.q4k_matmul_tokens with pinned H2D/D2H, graph-captured"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 3), "peak": peak, "unit": "int8 TOP/s",
                         "frac": round(achieved / peak, 5) if peak else None,
                         "peak_source": "2 x measured bf16 dense (the int8 dense rate)" if peak else None,
                         "traffic": profiled_traffic(PREFILL["profile"]), "kernel": "prefill_q4k_kernel",
                         "us_per_launch": round(ms * 1e3 / copies, 3),
                         "note": "bound in practice by the fp64 scaling of every group's int32 dots"},
            "cpu_baseline": None if cpu is None else {kk: cpu[kk] for kk in ("value", "unit", "cores", "kind", "sample")},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps * copies,
        }
        return line


# ----------------------------------------------------------------------------- attention workload

ATTN = dict(q_heads=32, kv_heads=8, extra_rows=128, profile="attn_split_ctx32k_f16_q4_0")


def attention_describe(context: int, kv: str) -> str:
    return (f"decode attention, {ATTN['q_heads']} q / {ATTN['kv_heads']} KV heads x 128, {context + 1} keys, "
            f"{'fp16' if kv == 'f16' else 'Q4_0'} KV cache (fused q/k norm + IMROPE + append)")


def attention_kv_bytes(context: int, kv: str) -> int:
    """K and V bytes one call reads (the context rows and the appended one)."""
    per_row = 512 if kv == "f16" else 144
    return ATTN["kv_heads"] * (context + 1) * per_row


def attention_host_cache(kv: str, capacity: int, seed: int):
    """Seeded N(0, 1) K / V rows [kv_heads, capacity, 128] as the cache holds them."""
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((ATTN["kv_heads"], capacity, 128), dtype=np.float32)
    v = rng.standard_normal((ATTN["kv_heads"], capacity, 128), dtype=np.float32)
    if kv == "f16":
        return k.astype(np.float16), v.astype(np.float16)
    return k, v


def attention_cpu_reference(context: int, kv: str, target_s: float = 8.0):
    """The oracle's attention (oracle/oracle.c, OpenMP over all host threads) on the same shapes."""
    import oracle

    hq, hkv = ATTN["q_heads"], ATTN["kv_heads"]
    capacity = context + ATTN["extra_rows"]
    k, v = attention_host_cache(kv, capacity, seed=1)
    if kv == "q4_0":
        kq, kd = oracle.kv_q4_0_rows(k)
        vq, vd = oracle.kv_q4_0_rows(v)
        d = np.ascontiguousarray(np.concatenate([kd, vd], axis=-1))
    else:
        k, v = k.view(np.uint16), v.view(np.uint16)
    q = np.random.default_rng(2).standard_normal(hq * 128).astype(np.float32)
    threads = os.cpu_count() or 1
    reps, t0 = 0, time.perf_counter()
    while True:
        if kv == "q4_0":
            oracle.attention_q4_0(q, kq, vq, d, context + 1, hq, hkv, threads)
        else:
            oracle.attention(q, k, v, context + 1, hq, hkv, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= target_s:
            break
    per = el / reps
    return {"value": attention_kv_bytes(context, kv) / per / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{reps} attention calls over {context + 1} keys ({kv} cache) in {el:.1f} s "
                      f"(oracle/oracle.c, OpenMP {threads} threads, float64)", "seconds_per_call": per}


def run_attention_reference(args, rank: int, world: int):
    if rank != 0:
        return
    ref = attention_cpu_reference(args.context, args.kv, target_s=max(3.0, min(20.0, 1.0 * args.steps)))
    line = {"metric": f"{attention_describe(args.context, args.kv)} KV GB/s", "value": round(ref["value"], 4),
            "unit": "GB/s", "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ref["seconds_per_call"] * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded N(0,1) K/V)",
            "config": {"workload": attention_describe(args.context, args.kv)},
            "cpu_baseline": {kk: ref[kk] for kk in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": round(ref["value"], 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def attention_profiled_traffic(context: int, kv: str):
    """Per-launch DRAM bytes of the split kernel from the committed ncu summary (32768-key context only)."""
    p = ROOT / "profiles" / f"{ATTN['profile']}.txt"
    if context != 32768 or not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            for part in line.split(":", 1)[1].split(","):
                name, _, val = part.strip().partition(" ")
                if name == kv:
                    try:
                        return int(val.strip("() "))
                    except ValueError:
                        return None
    return None


def run_attention(args, rank: int, world: int):
    """One step = `copies` fused attention calls (decode_attention_qkv[_q4_0]) over distinct caches
    (> 2x L2 together), PDL-chained in one CUDA graph: q/k RMSNorm + IMROPE, the K/V append at
    row `context`, attention over context + 1 keys, combine -> fp32 + Q8_1."""
    import torch
    import torch.distributed as dist

    from mojo_llm_lab_b200 import decode as D
    from mojo_llm_lab_b200 import formats as F
    from mojo_llm_lab_b200 import ops

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    hq, hkv, kv, context = ATTN["q_heads"], ATTN["kv_heads"], args.kv, args.context
    capacity = context + ATTN["extra_rows"]
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    kh, vh = attention_host_cache(kv, capacity, seed=1)
    per_copy = attention_kv_bytes(capacity - 1, kv)
    copies = args.copies or max(2, -(-int(2.2 * L2_BYTES) // per_copy))

    def make_cache():
        if kv == "f16":
            return torch.from_numpy(kh).to(device), torch.from_numpy(vh).to(device)
        c = D.Q4_0Cache.zeros(1, hkv, capacity, device)
        kq, vq, d = c.layer(0)
        ops.kv_q4_0_store(torch.from_numpy(kh).to(device), torch.from_numpy(vh).to(device), kq, vq, d)
        return kq, vq, d

    caches = [make_cache()]
    caches += [tuple(t.clone() for t in caches[0]) for _ in range(copies - 1)]
    rng = np.random.default_rng(3)
    qkv_host = (rng.standard_normal((hq + 2 * hkv) * 128) * 30).astype(np.float32)
    qg = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    kg = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    qkv, q_gamma, k_gamma = (torch.from_numpy(a).to(device) for a in (qkv_host, qg, kg))
    state = torch.frombuffer(bytearray(D.state_bytes(0, context)), dtype=torch.uint8).to(device)
    theta = F.theta_scale_f32()
    out = torch.empty(hq * 128, dtype=torch.float32, device=device)
    q8 = torch.empty(hq * 128 // 32 * 36, dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        scratch = torch.empty(int(ops.lib().mllb_decode_attention_scratch(hq, hkv, capacity)), dtype=torch.float64,
                              device=device)

    def call(i, pdl=True):
        c = caches[i]
        if kv == "f16":
            ops.decode_attention_qkv(qkv, q_gamma, k_gamma, state, c[0], c[1], hq, theta, out, q8, scratch, pdl=pdl)
        else:
            ops.decode_attention_qkv_q4_0(qkv, q_gamma, k_gamma, state, c[0], c[1], c[2], hq, theta, out, q8,
                                          scratch, pdl=pdl)

    call(0, pdl=False)
    torch.cuda.synchronize()
    if not args.skip_check and rank == 0:
        import oracle
        got = out.cpu().numpy()
        if kv == "f16":
            q_ref, _, _ = oracle.qk_rope_append(qkv_host, hq, hkv, qg, kg, context, theta)
            ref = oracle.attention(q_ref, caches[0][0].cpu().numpy().view(np.uint16),
                                   caches[0][1].cpu().numpy().view(np.uint16), context + 1, hq, hkv)
        else:
            q_ref, _, _ = oracle.qk_rope_f32(qkv_host, hq, hkv, qg, kg, context, theta)
            c = caches[0]
            ref = oracle.attention_q4_0(q_ref, c[0].cpu().numpy(), c[1].cpu().numpy(),
                                        np.ascontiguousarray(c[2].cpu().numpy().view(np.uint16)), context + 1, hq, hkv)
        if not np.all(np.abs(got - ref) <= 1e-5 + 1e-5 * np.abs(ref)):
            raise SystemExit("attention correctness gate failed against the oracle")

    def step():
        for i in range(copies):
            call(i)

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        preroll(graph)
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        stop.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    if world > 1:  # the slowest rank's time
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    kv_bytes = attention_kv_bytes(context, kv)
    us_call = ms * 1e3 / copies
    gbs = kv_bytes / (us_call * 1e-6) / 1e9

    # e2e through the public API with host buffers: the raw QKV projection from
    # pinned host memory, the fused attention, its fp32 output back; graph-captured.
    qkv_pin = torch.from_numpy(qkv_host).pin_memory()
    out_pin = torch.empty(hq * 128, dtype=torch.float32).pin_memory()

    def e2e_step():
        qkv.copy_(qkv_pin, non_blocking=True)
        call(0)
        out_pin.copy_(out, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e_graph, stream=stream):
        e2e_step()
    for _ in range(args.warmup):
        e_graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e_graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    del graph, e_graph
    if ops.device_error():
        raise SystemExit("device error word set")
    if rank == 0:
        peak, peak_kind = measured_peak()
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            c = attention_cpu_reference(context, kv)
            cpu = {kk: c[kk] for kk in ("value", "unit", "cores", "kind", "sample")}
        line = {
            "metric": f"{attention_describe(context, kv)} KV GB/s", "value": round(gbs * world, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 6),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": ("fp16" if kv == "f16" else "Q4_0") + " cache, f64 scores / softmax / P.V",
            "data": "synthetic (seeded N(0,1) K/V, N(0,30) QKV projection)",
            "config": {"workload": attention_describe(context, kv), "context": context, "kv_cache": kv,
                       "launches_per_step": 2 * copies, "us_per_call": round(us_call, 3),
                       "kv_bytes_per_call": kv_bytes,
                       "l2": f"{copies} cache copies ({copies * per_copy / 2**20:.0f} MiB) > 2x L2; no flush",
                       "chain": "PDL-chained split + combine launches in one CUDA graph",
                       "parallelism": "single GPU" if world == 1 else f"replicas x{world}"},
            "e2e": {"value": round(kv_bytes / (e_ms * 1e-3) / 1e9 * world, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": qkv_host.nbytes, "d2h_bytes_per_step": hq * 128 * 4,
                    "ms_per_step": round(e_ms, 6),
                    "path": "ops.decode_attention_qkv[_q4_0] with pinned H2D of the QKV row and D2H of the output, "
                            "graph-captured"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 5), "peak_source": peak_kind,
                         "traffic": attention_profiled_traffic(context, kv),
                         "kernel": "attn_split_kernel + attn_combine_kernel (timed together)",
                         "us_per_launch": round(us_call, 3),
                         "note": "issue-bound: fp64 arithmetic on converted cache values, not HBM"},
            "cpu_baseline": cpu, "clocks": clocks.summary(), "gpu_launches": args.steps * copies * 2,
        }
        return line


# ----------------------------------------------------------------------------- decode workload

DECODE_TOKENS = 128


def decode_host_cache(cfg, kv: str, dev):
    """Host copy of the seeded KV cache for the oracle: fp16 bits (k, v) or,
    for kv == "q4_0", None, None and the Q4_0 planes (k_qs, v_qs, d bits)."""
    from mojo_llm_lab_b200 import decode as D

    if kv == "f16":
        k, v = D.generate_kv_cache(cfg, dev)
        return k.cpu().numpy().view(np.uint16).copy(), v.cpu().numpy().view(np.uint16).copy(), None
    if str(dev).startswith("cuda"):
        c = D.generate_kv_cache_q4_0(cfg, dev)
        planes = (c.k_qs.cpu().numpy().copy(), c.v_qs.cpu().numpy().copy(), c.d.cpu().numpy().view(np.uint16).copy())
    else:  # no GPU: the oracle's quantiser over the same seeded rows
        import oracle

        qs = (cfg.layers, cfg.kv_heads, cfg.ctx_capacity, 64)
        planes = (np.zeros(qs, np.uint8), np.zeros(qs, np.uint8), np.zeros(qs[:3] + (8,), np.uint16))
        for layer in range(cfg.layers):
            for slot, p, lo in ((9, planes[0], 0), (10, planes[1], 4)):
                rows = D._kv_values(cfg, layer, slot, dev).numpy()
                p[layer, :, :cfg.context], planes[2][layer, :, :cfg.context, lo:lo + 4] = oracle.kv_q4_0_rows(rows)
    return None, None, planes


def decode_cpu_reference(target_s: float = 15.0, kv: str = "f16", context: int = 4096):
    """Time the oracle's decode step (oracle/decode.py over oracle/oracle.c, OpenMP over all
    host threads) on the 36-layer stack: whole tokens from the prefilled context."""
    import torch

    from mojo_llm_lab_b200 import decode as D
    from oracle import decode as OD

    cfg = D.DecodeConfig(context=context)
    # Data preparation only (torch's CPU generator takes ~30 s for 2.4 GB).
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    w = D.generate_weights(cfg, dev)
    host = OD.host_model(w)
    kh, vh, planes = decode_host_cache(cfg, kv, dev)
    del w
    threads = os.cpu_count() or 1
    token, pos, n, t0 = 17, cfg.context, 0, time.perf_counter()
    while True:
        _, token = OD.reference_step(host, kh, vh, token, pos, threads, q4_0=planes)
        pos, n = pos + 1, n + 1
        el = time.perf_counter() - t0
        if el >= target_s or pos >= cfg.ctx_capacity:
            break
    del torch
    return {"value": n / el, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} greedy tokens of the 36-layer stack from context {context} ({kv} KV) in {el:.1f} s "
                      f"(oracle/decode.py + oracle/oracle.c, OpenMP {threads} threads, float64)",
            "seconds_per_token": el / n}


def run_decode_reference(args, rank: int, world: int):
    if rank != 0:
        return
    ref = decode_cpu_reference(target_s=max(5.0, min(30.0, 2.0 * args.steps)), kv=args.kv, context=args.context)
    line = {"metric": "36-layer synthetic Q4_K decode tokens/s", "value": round(ref["value"], 4),
            "unit": "tokens/s", "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ref["seconds_per_token"] * DECODE_TOKENS * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded)",
            "config": {"workload": f"36-layer Qwen3-style decode, ctx {args.context}, 128 greedy tokens"
                                   + ("" if args.kv == "f16" else ", Q4_0 KV cache")},
            "cpu_baseline": {kk: ref[kk] for kk in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": round(ref["value"], 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_decode(args, rank: int, world: int):
    import torch
    import torch.distributed as dist

    from mojo_llm_lab_b200 import decode as D
    from mojo_llm_lab_b200 import ops

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    cfg = D.DecodeConfig(context=args.context)
    # Replicas: every rank decodes its own sequence on the whole model (no
    # sharding, no collective in the step); value = all ranks' tokens/s.
    replicas = getattr(args, "decode_replicas", False) and world > 1
    shard_world = 1 if replicas else world
    group = dist.group.WORLD if shard_world > 1 else None
    weights = D.generate_weights(cfg, device, world=shard_world, rank=rank if shard_world > 1 else 0)
    if args.kv == "q4_0":
        k_cache, v_cache = D.generate_kv_cache_q4_0(cfg, device), None
    else:
        k_cache, v_cache = D.generate_kv_cache(cfg, device)
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    torch.cuda.set_stream(stream)
    dec = D.Decoder(weights, k_cache, v_cache, pdl=not args.no_pdl, fused=args.fused, group=group)
    start_token = 17

    # Correctness gate: the first token's full logits against the oracle
    # (rank 0; the logit shards are gathered first).
    dec.reset(start_token)
    dec.step()
    torch.cuda.synchronize()
    if shard_world > 1:
        logits = torch.empty(weights.vocab_shard.per_rank * world, dtype=torch.float32, device=device)
        dist.all_gather_into_tensor(logits, dec.b.logits)
        logits = logits[:cfg.vocab]
    else:
        logits = dec.b.logits
    agreement = None
    if rank == 0 and not args.skip_check:
        from oracle import decode as OD
        full = weights if shard_world == 1 else D.generate_weights(cfg, device)
        host = OD.host_model(full)
        del full
        kh, vh, planes = decode_host_cache(cfg, args.kv, device)
        ref, ref_next = OD.reference_step(host, kh, vh, start_token, cfg.context, q4_0=planes)
        agreement = OD.logit_agreement(ref, logits.cpu().numpy())
        if agreement["violations"] or not agreement["top_match"]:
            raise SystemExit(f"decode correctness gate failed: {agreement}")
        if dec.read_state()["next_token"] != ref_next:
            raise SystemExit("decode correctness gate failed: next token differs from the oracle")
        del host, kh, vh, planes
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # One graph per token; a step = reset (device-to-device copy of the seed
    # state) + 128 replays.
    dec.reset(start_token)
    seed = dec.b.state.clone()
    dec.capture()
    if world > 1:
        dist.barrier()

    def step():
        dec.b.state.copy_(seed, non_blocking=True)
        for _ in range(DECODE_TOKENS):
            dec.replay()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        stop.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = DECODE_TOKENS / (ms * 1e-3) * (world if replicas else 1)

    # e2e through the public API: Decoder.generate (H2D of the seed state,
    # 128 graph replays, D2H of the generated tokens).
    e_ms_all = []
    tokens = None
    for i in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        tokens = dec.generate(start_token, DECODE_TOKENS)
        if i >= args.warmup:
            e_ms_all.append((time.perf_counter() - t0) * 1e3)
    e_ms = statistics.median(e_ms_all)
    if world > 1:
        t = torch.tensor([e_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    derr = ops.device_error()
    if derr:
        raise SystemExit(f"device error word set: {derr:#x}")
    if world > 1:
        toks = torch.tensor(tokens, device=device)
        allt = torch.empty(world, len(tokens), dtype=toks.dtype, device=device)
        dist.all_gather_into_tensor(allt, toks)
        if not bool((allt == allt[0]).all()):
            raise SystemExit("ranks decoded different token streams")
    launches = dec.launches_per_step()
    dec.graph = None
    if world > 1:
        dist.barrier()

    if rank == 0:
        peak, peak_kind = measured_peak()
        mean_keys = cfg.context + (DECODE_TOKENS + 1) / 2
        rank_bytes = (cfg.q4k_bytes() - 2 * cfg.layers * (cfg.ffn - weights.ffn_shard.local_rows) * cfg.hidden
                      // 256 * 144 + weights.vocab_shard.local_rows * cfg.hidden // 256 * 210
                      + cfg.kv_bytes_read(int(mean_keys), args.kv))
        us_per_token = ms * 1e3 / DECODE_TOKENS
        achieved = rank_bytes / (us_per_token * 1e-6) / 1e9
        cpu = None if args.no_cpu_baseline or world > 1 else decode_cpu_reference(target_s=10.0, kv=args.kv,
                                                                                   context=args.context)
        line = {
            "metric": "36-layer synthetic Q4_K decode tokens/s", "value": round(value, 2), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak" if replicas else "strong", "vs_baseline": None,
            "dtype": "Q4_K/Q6_K x Q8_1 dp4a, f64 accumulate; " + ("fp16" if args.kv == "f16" else "Q4_0")
                     + " KV, f64 attention",
            "data": "synthetic (seeded random weights, N(0,1) KV prefill)",
            "config": {"workload": "36-layer Qwen3-style decode (hidden 2560, 32/8 heads x 128, SwiGLU 9728, "
                                   f"vocab 151936), ctx {args.context}, 128 greedy tokens per step"
                                   + ("" if args.kv == "f16" else ", Q4_0 KV cache"),
                       "kv_cache": args.kv,
                       "us_per_token": round(us_per_token, 3), "bytes_per_token_per_gpu": int(rank_bytes),
                       "parallelism": (f"replicas x{world}: one independent sequence per GPU, whole model on each"
                                       if replicas else
                                       (f"gate/up + vocab rows/{world} per rank; " + ("peer-store Q8_1 all-gather over NVLink" if dec.peer is not None else "NCCL all-gather") + ", NCCL all-reduce of the argmax key") if world > 1 else "single GPU"),
                       "l2": "2.4 GB of weights per token > L2; no flush", "pdl": not args.no_pdl,
                       "fused_activations": dec.fused,
                       "logit_agreement": agreement},
            "e2e": {"value": round(DECODE_TOKENS / (e_ms * 1e-3) * (world if replicas else 1), 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": 32,
                    "d2h_bytes_per_step": 32 + DECODE_TOKENS * 4, "ms_per_step": round(e_ms, 4),
                    "path": "Decoder.generate (C-ABI launches captured in a CUDA graph), host seed state in, tokens out"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind, "traffic": None,
                         "kernel": "whole decode step (algorithmic bytes: weights + KV rows read, per GPU)",
                         "us_per_launch": round(us_per_token / launches, 4)},
            "cpu_baseline": None if cpu is None else {kk: cpu[kk] for kk in ("value", "unit", "cores", "kind", "sample")},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps * DECODE_TOKENS * launches,
        }
        return line


# ----------------------------------------------------------------------------- IMROPE workloads


def run_imrope_reference(args, rank: int, world: int, batched: bool):
    if rank != 0:
        return
    c = imrope_cpu_reference(4096 if batched else 1, target_s=max(3.0, min(20.0, args.steps)))
    if batched:
        value, unit, hib = imrope_bytes(1) / c["per_token_s"] / 1e9, "GB/s", True
        metric = "fused RMSNorm+gamma+IMROPE throughput (4096 tokens x 32 heads x 128) GB/s"
    else:
        value, unit, hib = c["us_per_token_op"], "us/op", False
        metric = "fused RMSNorm+gamma+IMROPE 32x128 us/op"
    line = {"metric": metric, "value": round(value, 4), "unit": unit, "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": c["per_token_s"] * 1e3,
            "higher_is_better": hib, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded)", "config": imrope_config(batched, world),
            "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": 1, "kind": "port",
                             "sample": c["sample"]},
            "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)

def imrope_config(batched: bool, world: int) -> dict:
    from mojo_llm_lab_b200 import fixtures as fx
    tokens = 4096 if batched else 1
    return {"workload": "imrope batched" if batched else "imrope 32x128", "tokens": tokens, "heads": 32,
            "bytes_per_op": imrope_bytes(tokens), "positions": list(fx.SEEDED_IMROPE_CASES["distinct_axes"]),
            "chain": "PDL-chained launches in one CUDA graph",
            "l2": ("4 copies x 67 MB in > 2x L2; no flush" if batched else
                   "128 distinct 16 KB inputs (L2-resident, like the reference's graph)"),
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU"}


IMROPE_PUBLISHED_US = 2.072   # reference, Mojo fused kernel on RTX A2000 (README.md:17-21)


def imrope_bytes(tokens: int, heads: int = 32) -> int:
    """q in + out (fp32) + gamma + positions + theta scale."""
    return tokens * heads * 128 * 4 * 2 + 128 * 4 + tokens * 16 + 4


def imrope_cpu_reference(tokens: int, target_s: float = 5.0):
    import oracle
    from mojo_llm_lab_b200 import fixtures as fx

    inp = fx.imrope_seeded_inputs(fx.SEEDED_IMROPE_CASES["distinct_axes"], seed=1)
    theta = oracle.runtime_theta_scale()
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < target_s:
        oracle.imrope(inp["q"], inp["gamma"], inp["positions_axis_major"], theta)
        reps += 1
    el = time.perf_counter() - t0
    per_token = el / reps
    return {"us_per_token_op": per_token * 1e6, "cores": 1, "kind": "port",
            "sample": f"{reps} x (32 heads x 128, one token) in {el:.1f} s (oracle/oracle.c orc_imrope, 1 thread)",
            "per_token_s": per_token}


def run_imrope(args, rank: int, world: int, batched: bool):
    import torch
    import torch.distributed as dist

    from mojo_llm_lab_b200 import fixtures as fx
    from mojo_llm_lab_b200 import formats as F
    from mojo_llm_lab_b200 import ops

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    tokens, heads = (4096, 32) if batched else (1, 32)
    copies = 4 if batched else 128
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    inp = fx.imrope_seeded_inputs(fx.SEEDED_IMROPE_CASES["distinct_axes"], seed=1, heads=heads * tokens)
    gen = torch.Generator(device=device)
    gen.manual_seed(5)
    qs = [torch.from_numpy(inp["q"]).to(device).view(-1)]
    qs += [torch.randn(tokens * heads * 128, generator=gen, device=device) for _ in range(copies - 1)]
    gamma = torch.from_numpy(inp["gamma"]).to(device)
    pos = torch.tensor(list(fx.SEEDED_IMROPE_CASES["distinct_axes"]) * tokens, dtype=torch.int32, device=device)
    theta = torch.tensor([F.theta_scale_f32()], dtype=torch.float32, device=device)
    outs = torch.empty(copies, tokens * heads * 128, device=device)

    def launch(i, pdl=True):
        # PDL-chained through the batched entry (theta from device memory, as
        # the reference ABI passes it; gamma / positions / theta, which no
        # kernel of the chain writes, read before the dependency wait);
        # pdl=False is the reference entry.
        if batched or pdl:
            ops.rmsnorm_imrope_q(qs[i], gamma, pos, theta, out=outs[i], heads_per_token=heads, pdl=pdl,
                                 const_aux=pdl)
        else:
            ops.fused_q_imrope_runtime_fastpow(qs[i], gamma, pos, outs[i], theta)

    # Correctness gate: the three position cases (distinct axes, all 32768, fourth-axis fallback) against the oracle.
    if not args.skip_check:
        import oracle
        for name, case in fx.SEEDED_IMROPE_CASES.items():
            c = fx.imrope_seeded_inputs(case, seed=2)
            got = ops.fused_q_imrope_runtime_fastpow(
                torch.from_numpy(c["q"]).to(device).view(-1), torch.from_numpy(c["gamma"]).to(device),
                torch.tensor(case, dtype=torch.int32, device=device), torch.empty(32 * 128, device=device), theta)
            ref = oracle.imrope(c["q"], c["gamma"], case, oracle.runtime_theta_scale())
            g = got.cpu().numpy().astype(np.float64).reshape(ref.shape)
            if not np.all(np.abs(g - ref) <= 1e-5 + 1e-5 * np.abs(ref)):
                raise SystemExit(f"IMROPE correctness gate failed ({name})")
        if batched:
            launch(0)
            torch.cuda.synchronize()
            ref = oracle.imrope(inp["q"][:heads], inp["gamma"], list(fx.SEEDED_IMROPE_CASES["distinct_axes"]),
                                oracle.runtime_theta_scale())
            g = outs[0][:heads * 128].cpu().numpy().astype(np.float64).reshape(ref.shape)
            if not np.all(np.abs(g - ref) <= 1e-5 + 1e-5 * np.abs(ref)):
                raise SystemExit("IMROPE batched correctness gate failed")

    for i in range(copies):
        launch(i)
    torch.cuda.synchronize()
    one_pass = torch.cuda.CUDAGraph()
    with torch.cuda.graph(one_pass, stream=stream):
        for i in range(copies):
            launch(i)
    passes = passes_for(one_pass, stream, world, device)  # a step lasts ~1 ms or more
    del one_pass
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(passes):
            for i in range(copies):
                launch(i)
    # The reference's own measurement: serial launches of its entry in a graph.
    serial = torch.cuda.CUDAGraph()
    with torch.cuda.graph(serial, stream=stream):
        for _ in range(passes):
            for i in range(copies):
                launch(i, pdl=False)
    for _ in range(args.warmup):
        graph.replay()
        serial.replay()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        serial.replay()
    s1.record(stream)
    torch.cuda.synchronize()
    serial_us = s0.elapsed_time(s1) / args.steps * 1e3 / (copies * passes)
    del serial
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        preroll(graph)  # load before the timed region (clock samples)
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        stop.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    us_op = ms * 1e3 / (copies * passes)
    per_op = imrope_bytes(tokens, heads)
    gbs = per_op / (us_op * 1e-6) / 1e9

    # e2e through the public API with host buffers: pinned H2D of each q, the
    # op (the PDL-chained entry), D2H of its output; the step captured in a
    # CUDA graph, copies overlapping the chain (one op a step in the
    # many-token form).
    n_e = 1 if batched else copies
    q_pin = torch.stack([qs[i].cpu() for i in range(n_e)]).pin_memory()
    q_stage = torch.empty(n_e, tokens * heads * 128, device=device)
    out_pin = torch.empty(n_e, tokens * heads * 128, dtype=torch.float32).pin_memory()

    def e2e_in(a, b):
        q_stage[a:b].copy_(q_pin[a:b], non_blocking=True)

    def e2e_op(i):
        ops.rmsnorm_imrope_q(q_stage[i], gamma, pos, theta, out=outs[i], heads_per_token=heads, pdl=True,
                             const_aux=True)

    def e2e_out(a, b):
        out_pin[a:b].copy_(outs[a:b], non_blocking=True)

    e_ms, e_first, e_last = overlapped_e2e(torch, device, stream, n_e, e2e_in, e2e_op, e2e_out, args.warmup,
                                          args.steps)
    e_us = e_ms * 1e3 / n_e
    if ops.device_error():
        raise SystemExit("device error word set")
    del graph
    if rank != 0:
        return
    peak, peak_kind = measured_peak()
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        c = imrope_cpu_reference(tokens)
        cpu = ({"value": round(c["us_per_token_op"], 3), "unit": "us/op", "cores": 1, "kind": "port",
                "sample": c["sample"]} if not batched else
               {"value": round(imrope_bytes(1, heads) / c["per_token_s"] / 1e9, 4), "unit": "GB/s", "cores": 1,
                "kind": "port", "sample": c["sample"]})
    if batched:
        value, unit, hib = round(gbs, 2), "GB/s", True
        e2e = {"value": round(per_op / (e_us * 1e-6) / 1e9, 2), "unit": "GB/s"}
        metric = "fused RMSNorm+gamma+IMROPE throughput (4096 tokens x 32 heads x 128) GB/s"
    else:
        value, unit, hib = round(us_op, 4), "us/op", False
        e2e = {"value": round(e_us, 3), "unit": "us/op"}
        metric = "fused RMSNorm+gamma+IMROPE 32x128 us/op"
    e2e.update({"h2d_bytes_per_step": tokens * heads * 512 * n_e, "d2h_bytes_per_step": tokens * heads * 512 * n_e,
                "ops_per_step": n_e,
                "path": f"ops.rmsnorm_imrope_q (PDL-chained) over {n_e} pinned inputs a step, H2D / D2H overlapping "
                        f"the chain (first {e_first} in before it, last {e_last} out after it), in a CUDA graph"})
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 6), "higher_is_better": hib,
            "scaling": "weak", "vs_baseline": None if batched else round(us_op / IMROPE_PUBLISHED_US, 4),
            "dtype": "f32 in/out, f64 norm and angles", "data": "synthetic (seeded N(0,1) q, U(0.5,1.5) gamma)",
            "config": imrope_config(batched, world), "us_per_op": round(us_op, 4),
            "us_per_op_serial_graph": round(serial_us, 4), "passes_per_step": passes,
            "launches_per_step": copies * passes, "e2e": e2e,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 5), "peak_source": peak_kind,
                         "traffic": profiled_traffic("imrope_q_32x128_and_4096_tokens") if batched else None,
                         "kernel": "imrope_q_kernel", "us_per_launch": round(us_op, 4)},
            "cpu_baseline": cpu, "clocks": clocks.summary(), "gpu_launches": args.steps * copies * passes}
    return line


# ----------------------------------------------------------------------------- Q8_1 quantiser workloads

Q8_1_TOKENS_BATCHED = 4096


def q8_1_bytes_per_op(k: int, tokens: int = 1) -> int:
    """fp32 read + Q8_1 write (36 bytes per 32 values)."""
    return tokens * (k * 4 + k // 32 * 36)


def q8_1_cpu_reference(k: int, target_s: float = 3.0):
    import oracle
    from mojo_llm_lab_b200 import fixtures as fx

    x = fx.seeded_activation(k, seed=3)
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < target_s:
        oracle.quantize_q8_1(x)
        reps += 1
    el = time.perf_counter() - t0
    return {"per_op_s": el / reps, "cores": 1, "kind": "port",
            "sample": f"{reps} x quantise fp32[{k}] in {el:.1f} s (oracle/oracle.c orc_q8_1_quantize, 1 thread)"}


def q8_1_describe(batched: bool, k: int) -> str:
    return (f"Q8_1 quantiser {Q8_1_TOKENS_BATCHED} tokens x {k}" if batched else f"Q8_1 quantiser fp32[{k}]")


def run_q8_1_reference(args, rank: int, world: int, batched: bool):
    if rank != 0:
        return
    k = args.k
    c = q8_1_cpu_reference(k, target_s=max(3.0, min(20.0, args.steps)))
    if batched:
        value, unit, hib = q8_1_bytes_per_op(k) / c["per_op_s"] / 1e9, "GB/s", True
    else:
        value, unit, hib = c["per_op_s"] * 1e6, "us/op", False
    line = {"metric": f"{q8_1_describe(batched, k)} {unit}", "value": round(value, 4), "unit": unit,
            "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": c["per_op_s"] * 1e3, "higher_is_better": hib, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 -> s8 + f16", "data": "synthetic (seeded N(0,1))",
            "config": q8_1_config(batched, k, world),
            "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": 1, "kind": "port",
                             "sample": c["sample"]},
            "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def q8_1_config(batched: bool, k: int, world: int) -> dict:
    tokens = Q8_1_TOKENS_BATCHED if batched else 1
    copies = 6 if batched else 128
    return {"workload": q8_1_describe(batched, k), "k": k, "tokens": tokens, "inputs": copies,
            "bytes_per_op": q8_1_bytes_per_op(k, tokens),
            "l2": (f"{copies} inputs x {tokens * k * 4 / 2**20:.0f} MiB > 2x L2; no flush" if batched else
                   f"{copies} distinct {k * 4 // 1024} KB inputs (L2-resident, as a decode step's activations)"),
            "chain": "PDL-chained launches in one CUDA graph",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU"}


def run_q8_1(args, rank: int, world: int, batched: bool):
    """The activation quantiser alone: one fp32 vector of k (latency: us/op over
    128 PDL-chained launches on distinct inputs) or 4096 such vectors in one
    launch (HBM throughput mode)."""
    import torch
    import torch.distributed as dist

    import ctypes as C
    from mojo_llm_lab_b200 import ops
    from mojo_llm_lab_b200._lib import LAUNCH_PDL, S_D_SUMQ, check, lib

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    k = args.k
    tokens = Q8_1_TOKENS_BATCHED if batched else 1
    cfg = q8_1_config(batched, k, world)
    copies = cfg["inputs"]
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    gen = torch.Generator(device=device)
    gen.manual_seed(7)
    xs = torch.randn(copies, tokens * k, generator=gen, device=device)
    outs = torch.empty(copies, tokens * k // 32 * 36, dtype=torch.uint8, device=device)
    lib_ = lib()

    def launch(i, pdl=True):
        check(lib_.mllb_q8_1_quantize_ex(xs[i].data_ptr(), outs[i].data_ptr(), tokens * k, S_D_SUMQ,
                                         LAUNCH_PDL if pdl else 0, C.c_void_p(stream.cuda_stream)), "q8_1")

    if not args.skip_check:
        import oracle
        launch(0, pdl=False)
        torch.cuda.synchronize()
        x0 = xs[0][: min(tokens * k, 1 << 20)].cpu().numpy()
        if outs[0][: x0.size // 32 * 36].cpu().numpy().tobytes() != oracle.quantize_q8_1(x0):
            raise SystemExit("Q8_1 correctness gate failed: bytes differ from the oracle")
    for i in range(copies):
        launch(i)
    torch.cuda.synchronize()
    one_pass = torch.cuda.CUDAGraph()
    with torch.cuda.graph(one_pass, stream=stream):
        for i in range(copies):
            launch(i)
    passes = passes_for(one_pass, stream, world, device)  # a step lasts ~1 ms or more
    del one_pass
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(passes):
            for i in range(copies):
                launch(i)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        preroll(graph)
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        stop.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    us_op = ms * 1e3 / (copies * passes)
    per_op = q8_1_bytes_per_op(k, tokens)
    gbs = per_op / (us_op * 1e-6) / 1e9

    # e2e through the public API with host buffers: pinned H2D of each x, the
    # quantiser (the C ABI, PDL-chained), D2H of its Q8_1 bytes; the step
    # captured in a CUDA graph, copies overlapping the chain (one op a step in
    # the many-token form).
    n_e = 1 if batched else copies
    x_pin = xs[:n_e].cpu().pin_memory()
    o_pin = torch.empty(n_e, outs.shape[1], dtype=torch.uint8).pin_memory()
    x_stage = torch.empty_like(xs[:n_e])

    def e2e_in(a, b):
        x_stage[a:b].copy_(x_pin[a:b], non_blocking=True)

    def e2e_op(i):
        check(lib_.mllb_q8_1_quantize_ex(x_stage[i].data_ptr(), outs[i].data_ptr(), tokens * k, S_D_SUMQ,
                                         LAUNCH_PDL, C.c_void_p(torch.cuda.current_stream(device).cuda_stream)),
              "q8_1")

    def e2e_out(a, b):
        o_pin[a:b].copy_(outs[a:b], non_blocking=True)

    e_ms, e_first, e_last = overlapped_e2e(torch, device, stream, n_e, e2e_in, e2e_op, e2e_out, args.warmup,
                                          args.steps)
    e_us = e_ms * 1e3 / n_e
    if ops.device_error():
        raise SystemExit("device error word set")
    del graph
    if rank != 0:
        return
    peak, peak_kind = measured_peak()
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        c = q8_1_cpu_reference(k)
        cpu = ({"value": round(q8_1_bytes_per_op(k) / c["per_op_s"] / 1e9, 4), "unit": "GB/s", "cores": 1,
                "kind": "port", "sample": c["sample"]} if batched else
               {"value": round(c["per_op_s"] * 1e6, 3), "unit": "us/op", "cores": 1, "kind": "port",
                "sample": c["sample"]})
    if batched:
        value, unit, hib = round(gbs, 2), "GB/s", True
        e2e = {"value": round(per_op / (e_us * 1e-6) / 1e9, 2), "unit": "GB/s"}
    else:
        value, unit, hib = round(us_op, 4), "us/op", False
        e2e = {"value": round(e_us, 3), "unit": "us/op"}
    e2e.update({"h2d_bytes_per_step": tokens * k * 4 * n_e, "d2h_bytes_per_step": tokens * k // 32 * 36 * n_e,
                "ops_per_step": n_e,
                "path": f"mllb_q8_1_quantize_ex (PDL-chained) over {n_e} pinned inputs a step, H2D / D2H overlapping "
                        f"the chain (first {e_first} in before it, last {e_last} out after it), in a CUDA graph"})

    line = {"metric": f"{q8_1_describe(batched, k)} {unit}", "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 6), "higher_is_better": hib,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 -> s8 + f16", "data": "synthetic (seeded N(0,1))",
            "config": cfg, "us_per_op": round(us_op, 4), "passes_per_step": passes,
            "launches_per_step": copies * passes, "e2e": e2e,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 5), "peak_source": peak_kind,
                         "traffic": profiled_traffic("q8_1_quantize_k2560_and_4096x2560") if batched else None,
                         "kernel": "q8_1_quantize_x4_kernel", "us_per_launch": round(us_op, 4)},
            "cpu_baseline": cpu, "clocks": clocks.summary(), "gpu_launches": args.steps * copies * passes}
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["decode", "imrope", "imrope_batched", "prefill",
                                                               "attention", "q8_1", "q8_1_batched"],
                    default="q4k_matvec")
    ap.add_argument("--fused", action="store_true", help="decode: norms / quantisers built into the matvecs")
    ap.add_argument("--decode-replicas", action="store_true",
                    help="decode at N GPUs: one independent sequence per GPU (no sharding); tokens/s of all")
    ap.add_argument("--context", type=int, default=4096, help="decode: prefilled KV rows")
    ap.add_argument("--kv", choices=["f16", "q4_0"], default="f16",
                    help="decode: KV cache type (q4_0: GGML Q4_0, the reference's llama.cpp setting)")
    ap.add_argument("--copies", type=int, default=0)
    ap.add_argument("--k", type=int, default=2560, help="q8_1 workloads: values per activation vector")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--skip-check", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--headline-only", action="store_true",
                    help="default workload: skip the other configurations measured after the headline")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if args.workload == "decode":
            run_decode_reference(args, rank, world)
        elif args.workload == "prefill":
            run_prefill_reference(args, rank, world)
        elif args.workload == "attention":
            run_attention_reference(args, rank, world)
        elif args.workload.startswith("imrope"):
            run_imrope_reference(args, rank, world, batched=args.workload == "imrope_batched")
        elif args.workload.startswith("q8_1"):
            run_q8_1_reference(args, rank, world, batched=args.workload == "q8_1_batched")
        else:
            run_reference(args, rank, world)
        return
    runner = {"decode": run_decode, "prefill": run_prefill, "attention": run_attention,
              "imrope": lambda a, r, w: run_imrope(a, r, w, batched=False),
              "imrope_batched": lambda a, r, w: run_imrope(a, r, w, batched=True),
              "q8_1": lambda a, r, w: run_q8_1(a, r, w, batched=False),
              "q8_1_batched": lambda a, r, w: run_q8_1(a, r, w, batched=True)}.get(args.workload, run_ours)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))))
        try:
            line = runner(args, rank, world)
            if args.workload == "q4k_matvec" and not args.headline_only:
                # the row-sharded configurations at this N (every rank runs them, in the same order)
                others = other_configs(args, rank, world, OTHER_CONFIGS_SHARDED)
                if line is not None:
                    line["other_configs"] = others
        finally:
            dist.destroy_process_group()
    else:
        line = runner(args, rank, world)
        if line is not None and args.workload == "q4k_matvec" and not args.headline_only:
            line["other_configs"] = other_configs(args, rank, world, OTHER_CONFIGS)
    if line is not None:
        print(json.dumps(line), flush=True)


# The other benchmark configurations, measured in the same run as the headline:
# each entry is that workload's own line, trimmed.  One GPU: all of them;
# N GPUs: the row-sharded ones (gate/up and the vocabulary projection with an
# NCCL all-gather, the 36-layer decode with both sharded).
OTHER_CONFIGS = (("imrope", {}), ("imrope_batched", {}), ("q8_1", {}), ("gate_up", {}), ("q6k_vocab", {}),
                 ("decode", {"steps": 3, "warmup": 3}))
OTHER_CONFIGS_SHARDED = (("gate_up", {}), ("q6k_vocab", {}), ("decode", {"steps": 3, "warmup": 3}),
                         ("decode_replicas", {"steps": 3, "warmup": 3}))


def other_configs(args, rank: int, world: int, which) -> dict:
    import gc

    import torch
    runners = {"decode": run_decode, "decode_replicas": run_decode,
               "imrope": lambda a, r, w: run_imrope(a, r, w, batched=False),
               "imrope_batched": lambda a, r, w: run_imrope(a, r, w, batched=True),
               "q8_1": lambda a, r, w: run_q8_1(a, r, w, batched=False)}
    keep = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "higher_is_better", "vs_baseline", "dtype",
            "config", "e2e", "roofline", "clocks", "gpu_launches", "us_per_op", "passes_per_step",
            "launches_per_step")
    out = {}
    for name, over in which:
        sub = argparse.Namespace(**vars(args))
        sub.workload, sub.no_cpu_baseline, sub.copies = name, True, 0
        sub.decode_replicas = name == "decode_replicas"
        sub.steps, sub.warmup = over.get("steps", args.steps), over.get("warmup", args.warmup)
        t0 = time.perf_counter()
        if world > 1:  # collectives inside: every rank runs it to the end or the job fails together
            line = runners.get(name, run_ours)(sub, rank, world)
            if line is not None:
                out[name] = {kk: line[kk] for kk in keep if kk in line}
        else:
            try:
                line = runners.get(name, run_ours)(sub, rank, world)
                out[name] = {kk: line[kk] for kk in keep if kk in line}
            except SystemExit as e:  # a failed correctness gate: recorded, the headline stands
                out[name] = {"error": str(e)}
        if name in out:
            out[name]["wall_s"] = round(time.perf_counter() - t0, 1)
        gc.collect()
        torch.cuda.empty_cache()
    return out


if __name__ == "__main__":
    sys.path.insert(0, str(ROOT))
    main()
