"""Reference-ABI entries in lib/mllb200_compat.cubin, driven exactly the way
the reference's harnesses drive a kernel: cuModuleLoad + cuModuleGetFunction +
cuLaunchKernel with a flat pointer list and the reference launch geometry
(tools/q4_comparison_worker.py:29-34, benchmark/bench.c:240-258), output
canaries included."""
import ctypes as C

import numpy as np
import pytest
import torch

from gpu_util import assert_within_tolerance, canaries_intact, dev, dev_bytes, with_canaries
from mojo_llm_lab_b200 import build
from mojo_llm_lab_b200 import fixtures as fx
import ref_fixtures as rfx
from mojo_llm_lab_b200 import formats as F

pytestmark = pytest.mark.gpu


class Driver:
    def __init__(self):
        torch.zeros(1, device="cuda")  # make the primary context current
        self.cuda = C.CDLL("libcuda.so.1")
        self.module = C.c_void_p()
        self._ok(self.cuda.cuModuleLoad(C.byref(self.module), str(build.CUBIN).encode()), "cuModuleLoad")

    def _ok(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"{what} failed: {rc}")

    def launch(self, entry: str, grid: int, block: int, *tensors):
        fn = C.c_void_p()
        self._ok(self.cuda.cuModuleGetFunction(C.byref(fn), self.module, entry.encode()), entry)
        ptrs = [C.c_uint64(t.data_ptr()) for t in tensors]
        params = (C.c_void_p * len(ptrs))(*[C.cast(C.byref(p), C.c_void_p) for p in ptrs])
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        self.cuda.cuLaunchKernel.argtypes = [C.c_void_p, C.c_uint, C.c_uint, C.c_uint, C.c_uint, C.c_uint,
                                             C.c_uint, C.c_uint, C.c_void_p, C.c_void_p, C.c_void_p]
        self._ok(self.cuda.cuLaunchKernel(fn, grid, 1, 1, block, 1, 1, 0, stream, params, None), "cuLaunchKernel")
        torch.cuda.synchronize()

    def close(self):
        self.cuda.cuModuleUnload(self.module)


@pytest.fixture(scope="module")
def drv():
    d = Driver()
    yield d
    d.close()


@pytest.mark.parametrize("entry,block", [("q4_k_q8_1_matvec_dp4a", 32), ("q4_k_q8_1_matvec_dp4a_128", 128),
                                         ("q4_k_q8_1_matvec", 32)])
def test_plain_matvec_entries(drv, golden, entry, block):
    # q4_comparison_worker.py: 64-row fixture tiled x152 to 9728 rows, grid rows x block 32
    g = golden["q4_reference_fixtures"]["default"]
    files = rfx.q4_matvec_fixtures()
    w = dev_bytes(fx.tile_rows(files["weights.bin"], 1440, 9728))
    act = dev_bytes(files["activations.bin"])
    buf, out = with_canaries(9728)
    drv.launch(entry, 9728, block, w, act, out)
    got = out.cpu().numpy()
    assert got.astype(np.float64).tolist() == g["dot_weights"] * 152  # exact, as the worker requires
    assert canaries_intact(buf)


def test_gate_order_entry(drv, orc, golden):
    g = golden["q4_reference_fixtures"]["varied_activations"]
    files = rfx.q4_matvec_fixtures(**g["options"])
    w, gw, act = (dev_bytes(files[n]) for n in ("weights.bin", "gate.bin", "activations.bin"))
    buf, out = with_canaries(64)
    drv.launch("q4_k_q8_1_gate_order", 64, 128, w, gw, act, out)
    ref = [orc.swiglu(u, gg) for u, gg in zip(g["dot_weights"], g["dot_gate"])]
    assert_within_tolerance(out.cpu().numpy(), ref, "gate_order entry")
    assert canaries_intact(buf)


def test_gate_order_2b_entry(drv, orc, golden):
    g = golden["q4_reference_fixtures"]["width2048"]
    files = rfx.q4_matvec_fixtures(**g["options"])
    w, gw, act = (dev_bytes(files[n]) for n in ("weights.bin", "gate.bin", "activations.bin"))
    out = torch.empty(64, dtype=torch.float32, device="cuda")
    drv.launch("q4_k_q8_1_gate_order_2b", 64, 128, w, gw, act, out)
    ref = [orc.swiglu(u, gg) for u, gg in zip(g["dot_weights"], g["dot_gate"])]
    assert_within_tolerance(out.cpu().numpy(), ref, "gate_order_2b entry")


def test_imrope_entry(drv, orc):
    # benchmark/bench.c: grid 32 x block 128, theta bits 0x3f492c27, canaries
    q, gamma, pos = fx.parse_imrope(fx.serialize_imrope(rfx.imrope_reference_inputs(rfx.IMROPE_CASES["long_position"])))
    theta = torch.tensor([F.THETA_SCALE_BITS], dtype=torch.int64).to(torch.int32).view(torch.float32).cuda()
    buf, out = with_canaries(4096, guard=1, fill=float("nan"))
    drv.launch("fused_q_imrope_runtime_fastpow", 32, 128, dev(q), dev(gamma), dev(pos), out, theta)
    ref = orc.imrope(q, gamma, pos, orc.runtime_theta_scale())
    assert_within_tolerance(out.cpu().numpy(), ref.reshape(-1), "imrope entry")
    host = buf.cpu().numpy()
    assert np.isnan(host[0]) and np.isnan(host[-1])


def test_q6k_entry(drv, orc):
    rows = 40
    w = fx.seeded_q6k_matrix(rows, 2560, seed=3)
    a = orc.quantize_q8_1(fx.seeded_activation(2560, seed=4))
    out = torch.empty(rows, dtype=torch.float32, device="cuda")
    drv.launch("q6_k_q8_1_matvec", rows, 128, dev(w), dev_bytes(a), out)
    assert_within_tolerance(out.cpu().numpy(), orc.q6k_matvec(w, a, rows, 2560), "q6k entry")


def test_stream_read_roofline_entry(drv):
    # tools/run_bandwidth_roofline.py:33-37: the buffer is memset to a 32-bit
    # pattern; thread g XORs ceil((WORDS-g)/stride) identical words.
    nbytes, pattern = 417177600, 0x5A5A5A5A
    data = torch.full((nbytes // 4,), pattern, dtype=torch.int64).to(torch.int32).cuda()
    for grid in (640, 1280):
        out = torch.empty(grid * 128, dtype=torch.int64, device="cuda")
        drv.launch("stream_read_roofline", grid, 128, data, out)
        stride, words = grid * 128, nbytes // 8
        word = (pattern << 32) | pattern
        expect = [word if ((words - g + stride - 1) // stride) % 2 else 0 for g in range(stride)]
        assert out.cpu().numpy().view(np.uint64).tolist() == expect
    del data
