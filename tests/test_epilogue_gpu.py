"""The fused gate/up that also writes the Q8_1 of its product
(mllb_q4k_gate_up_q8), against the plain gate/up and the oracle's quantiser:
the product is bit-identical to mllb_q4k_gate_up_ex's and its Q8_1 bytes equal
the oracle's.  Called twice in a row: the group counters come back to zero.
"""
import numpy as np
import pytest
import torch

from gpu_util import dev
from mojo_llm_lab_b200 import fixtures as fx
from mojo_llm_lab_b200 import formats as F
from mojo_llm_lab_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,k", [(9728, 2560), (4864, 2560), (4096, 2048), (2048, 4096)])
def test_gate_up_q8_tail(orc, rows, k):
    up = dev(fx.seeded_q4k_matrix(rows, k, seed=21))
    gate = dev(fx.seeded_q4k_matrix(rows, k, seed=22))
    a = ops.quantize_q8_1(dev(fx.seeded_activation(k, seed=23)))
    _, _, prod_ref = ops.q4k_gate_up(up, gate, a, want=("prod",))
    prod_ref = prod_ref.cpu().numpy()
    q8_ref = orc.quantize_q8_1(prod_ref)
    counters = torch.zeros(rows // 32, dtype=torch.int32, device="cuda")
    for call in range(2):
        prod = torch.full((rows,), 3.0, device="cuda")
        q8 = torch.zeros(F.q8_1_bytes(rows), dtype=torch.uint8, device="cuda")
        ops.q4k_gate_up_q8(up, gate, a, prod, q8, counters, pdl=call == 1)
        torch.cuda.synchronize()
        assert np.array_equal(prod.cpu().numpy().view(np.uint32), prod_ref.view(np.uint32)), f"call {call}"
        assert q8.cpu().numpy().tobytes() == q8_ref, f"call {call}: Q8_1 of the product"
        assert not counters.cpu().numpy().any()
    assert ops.device_error() == 0


@pytest.mark.parametrize("rows,k", [(4864, 2560), (1216, 2560)])
def test_gate_up_q8_gather_on_one_rank(orc, rows, k):
    """The gate/up + peer-gather launch with world = 1 (the only form one GPU
    can run: ranks that wait on each other never share a GPU): its product's
    Q8_1 lands in the buffer, the rank's arrival is counted once per gather,
    the gather count advances, the counters return to zero, call after call.
    The multi-GPU decode test covers world > 1."""
    import ctypes as C
    from mojo_llm_lab_b200._lib import PeerGather, check, lib
    up = dev(fx.seeded_q4k_matrix(rows, k, seed=31))
    gate = dev(fx.seeded_q4k_matrix(rows, k, seed=32))
    a = ops.quantize_q8_1(dev(fx.seeded_activation(k, seed=33)))
    _, _, prod_ref = ops.q4k_gate_up(up, gate, a, want=("prod",))
    prod_ref = prod_ref.cpu().numpy()
    q8_ref = orc.quantize_q8_1(prod_ref)
    counters = torch.zeros(rows // 32 + 1, dtype=torch.int32, device="cuda")
    buf = torch.zeros(F.q8_1_bytes(rows), dtype=torch.uint8, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    count = torch.zeros(1, dtype=torch.int32, device="cuda")
    pg = PeerGather()
    pg.rank, pg.world = 0, 1
    pg.buffers[0], pg.flags[0], pg.count = buf.data_ptr(), flags.data_ptr(), count.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(3):
        prod = torch.full((rows,), 3.0, device="cuda")
        buf.zero_()
        check(lib().mllb_q4k_gate_up_q8_gather(up.data_ptr(), gate.data_ptr(), a.data_ptr(), None, None,
                                               prod.data_ptr(), counters.data_ptr(), rows, k, C.byref(pg),
                                               1 if call else 0, C.c_void_p(stream)), "gate_up_q8_gather")
        torch.cuda.synchronize()
        assert np.array_equal(prod.cpu().numpy().view(np.uint32), prod_ref.view(np.uint32)), f"call {call}"
        assert buf.cpu().numpy().tobytes() == q8_ref, f"call {call}: gathered Q8_1 of the product"
        assert not counters.cpu().numpy().any()
        assert count.item() == call + 1 and flags.item() == call + 1
    assert ops.device_error() == 0


def test_gate_up_q8_rejects_bad_shapes():
    from mojo_llm_lab_b200._lib import lib
    k = 2560
    w = torch.zeros(48 * F.q4k_row_bytes(k), dtype=torch.uint8, device="cuda")
    a = torch.zeros(F.q8_1_bytes(k), dtype=torch.uint8, device="cuda")
    prod = torch.zeros(48, device="cuda")
    q8 = torch.zeros(F.q8_1_bytes(64), dtype=torch.uint8, device="cuda")
    counters = torch.zeros(2, dtype=torch.int32, device="cuda")
    L = lib()
    # 48 rows: not whole Q8_1 groups
    assert L.mllb_q4k_gate_up_q8(w.data_ptr(), w.data_ptr(), a.data_ptr(), None, None, prod.data_ptr(),
                                 q8.data_ptr(), counters.data_ptr(), 48, k, 0, None) != 0
    # no product buffer / no counters
    assert L.mllb_q4k_gate_up_q8(w.data_ptr(), w.data_ptr(), a.data_ptr(), None, None, None, q8.data_ptr(),
                                 counters.data_ptr(), 32, k, 0, None) != 0
    assert L.mllb_q4k_gate_up_q8(w.data_ptr(), w.data_ptr(), a.data_ptr(), None, None, prod.data_ptr(),
                                 q8.data_ptr(), None, 32, k, 0, None) != 0
    torch.cuda.synchronize()
    assert not counters.cpu().numpy().any()


# ------------------------------------------------ residual + RMSNorm epilogue

@pytest.mark.parametrize("rows,k", [(2560, 4096), (2560, 9728), (2560, 2560), (4096, 2560), (2048, 2048),
                                    (1024, 4096)])
def test_matvec_norm_equals_matvec_then_norm(orc, rows, k):
    """mllb_q4k_matvec_norm == mllb_q4k_matvec_ex + the oracle's residual +
    RMSNorm + Q8_1, twice in a row (the grid counters come back to zero)."""
    w = dev(fx.seeded_q4k_matrix(rows, k, seed=31))
    a = ops.quantize_q8_1(dev(fx.seeded_activation(k, seed=32)))
    rng = np.random.default_rng(rows + k)
    x = (rng.standard_normal(rows) * 3).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, rows).astype(np.float32)
    delta = ops.q4_k_q8_1_matvec(w, a).cpu().numpy()
    h_ref, q8_ref = orc.rmsnorm_q8_1(x, delta, gamma, 1e-6)
    ws = ops.q4k_matvec_norm_workspace(rows, k, "cuda")
    for call in range(2):
        x_out = torch.full((rows,), 7.0, device="cuda")
        out = torch.full((rows,), 5.0, device="cuda")
        q8 = torch.zeros(F.q8_1_bytes(rows), dtype=torch.uint8, device="cuda")
        ops.q4k_matvec_norm(w, a, dev(x), dev(gamma), 1e-6, x_out=x_out, q8_out=q8, out=out, workspace=ws,
                            pdl=call == 1)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), delta.view(np.uint32)), f"call {call}: delta"
        assert np.array_equal(x_out.cpu().numpy(), h_ref), f"call {call}: residual"
        assert np.array_equal(q8.cpu().numpy(), q8_ref), f"call {call}: Q8_1 of the norm"
        assert not ws[:16].cpu().numpy().any()
    assert ops.device_error() == 0


def test_matvec_norm_in_place_and_without_delta(orc):
    rows, k = 2560, 4096
    w = dev(fx.seeded_q4k_matrix(rows, k, seed=41))
    a = ops.quantize_q8_1(dev(fx.seeded_activation(k, seed=42)))
    rng = np.random.default_rng(3)
    x = rng.standard_normal(rows).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, rows).astype(np.float32)
    delta = ops.q4_k_q8_1_matvec(w, a).cpu().numpy()
    h_ref, q8_ref = orc.rmsnorm_q8_1(x, delta, gamma, 1e-6)
    xd = dev(x)
    _, q8, _ = ops.q4k_matvec_norm(w, a, xd, dev(gamma), 1e-6, x_out=xd)
    assert np.array_equal(xd.cpu().numpy(), h_ref)
    assert np.array_equal(q8.cpu().numpy(), q8_ref)


def test_matvec_norm_rejects_bad_arguments():
    from mojo_llm_lab_b200._lib import lib
    k, rows = 2560, 48
    w = torch.zeros(64 * F.q4k_row_bytes(k), dtype=torch.uint8, device="cuda")
    a = torch.zeros(F.q8_1_bytes(k), dtype=torch.uint8, device="cuda")
    x = torch.zeros(64, device="cuda")
    q8 = torch.zeros(F.q8_1_bytes(64), dtype=torch.uint8, device="cuda")
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    L = lib()
    P = lambda t: t.data_ptr()  # noqa: E731
    # 48 rows: not whole Q8_1 groups
    assert L.mllb_q4k_matvec_norm(P(w), P(a), None, rows, k, P(x), P(x), P(x), 1e-6, P(q8), P(ws), ws.numel(), 0,
                                  None) != 0
    # workspace too small
    assert L.mllb_q4k_matvec_norm(P(w), P(a), None, 64, k, P(x), P(x), P(x), 1e-6, P(q8), P(ws), 8, 0, None) != 0
    # x_out overlapping x off by one element
    assert L.mllb_q4k_matvec_norm(P(w), P(a), None, 32, k, P(x), P(x) + 4, P(q8), 1e-6, P(q8), P(ws), ws.numel(),
                                  0, None) != 0
    # K with no streaming configuration
    assert L.mllb_q4k_matvec_norm(P(w), P(a), None, 32, 768, P(x), P(x), P(x), 1e-6, P(q8), P(ws), ws.numel(), 0,
                                  None) != 0
    torch.cuda.synchronize()
    assert not ws.cpu().numpy().any()
