"""Q4_K x Q8_1 matvec and fused gate/up on the GPU against the oracle.

Integer sub-block dots: bit-exact.  fp32 outputs: |got - ref| <= 1e-5 + 1e-5|ref|
against the float64 oracle (which reproduces the reference's dot_q4_q8 bit
for bit, see test_oracle_golden.py)."""
import numpy as np
import pytest
import torch

from gpu_util import assert_within_tolerance, canaries_intact, dev, dev_bytes, with_canaries
from mojo_llm_lab_b200 import fixtures as fx
import ref_fixtures as rfx
from mojo_llm_lab_b200 import ops

pytestmark = pytest.mark.gpu

REF_CASES = ["default", "random_quants", "gate_up", "gate_up_rows128", "varied_factors", "varied_activations",
             "default_activation_scales", "width2048"]


@pytest.mark.parametrize("case", REF_CASES)
def test_reference_fixtures_match_golden(golden, case):
    g = golden["q4_reference_fixtures"][case]
    files = rfx.q4_matvec_fixtures(**g["options"])
    act = dev_bytes(files["activations.bin"])
    for key in ("weights", "gate"):
        if "dot_" + key not in g:
            continue
        w = dev_bytes(files[key + ".bin"])
        buf, out = with_canaries(len(g["dot_" + key]))
        ops.q4_k_q8_1_matvec(w, act, out)
        got = out.cpu().numpy()
        assert_within_tolerance(got, g["dot_" + key], f"{case}/{key}")
        assert canaries_intact(buf)
        if case == "default":
            # dyadic fixture: the exact float64 dot is representable in fp32
            assert got.astype(np.float64).tolist() == g["dot_" + key]
    assert ops.device_error() == 0


@pytest.mark.parametrize("case", ["gate_up", "varied_factors", "varied_activations", "width2048"])
def test_reference_gate_up_fixtures(orc, golden, case):
    g = golden["q4_reference_fixtures"][case]
    files = rfx.q4_matvec_fixtures(**g["options"])
    k = g["options"].get("input_width", 2560)
    rows = len(g["dot_weights"])
    up_w, gate_w, act = (dev_bytes(files[n]) for n in ("weights.bin", "gate.bin", "activations.bin"))
    up, gate, prod = ops.q4k_gate_up(up_w, gate_w, act)
    ref_prod = [orc.swiglu(u, gg) for u, gg in zip(g["dot_weights"], g["dot_gate"])]
    assert_within_tolerance(up.cpu().numpy(), g["dot_weights"], "up")
    assert_within_tolerance(gate.cpu().numpy(), g["dot_gate"], "gate")
    assert_within_tolerance(prod.cpu().numpy(), ref_prod, "prod")
    # the reference-named entry emits only the product
    only = ops.q4_k_q8_1_gate_order(up_w, gate_w, act)
    assert torch.equal(only, prod)
    assert rows == prod.numel() and k in (2048, 2560)


def test_reference_fixture_tiled_to_9728_rows(golden):
    # benchmark/q4_compare.c:148-163 tiles the 64-row file to ROWS=9728
    g = golden["q4_reference_fixtures"]["varied_activations"]
    files = rfx.q4_matvec_fixtures(**g["options"])
    w = dev_bytes(fx.tile_rows(files["weights.bin"], 1440, 9728))
    gw = dev_bytes(fx.tile_rows(files["gate.bin"], 1440, 9728))
    act = dev_bytes(files["activations.bin"])
    up, gate, prod = ops.q4k_gate_up(w, gw, act)
    assert_within_tolerance(up.cpu().numpy(), g["dot_weights"] * 152, "up tiled")
    assert_within_tolerance(gate.cpu().numpy(), g["dot_gate"] * 152, "gate tiled")


@pytest.mark.parametrize("rows,k", [(4096, 2560), (1, 2560), (15, 2560), (17, 2560), (4097, 2560),
                                    (1000, 2048), (333, 4096), (70, 9728), (64, 512)])
def test_seeded_matvec_against_oracle(orc, rows, k):
    w = fx.seeded_q4k_matrix(rows, k, seed=rows * 7 + k)
    x = fx.seeded_activation(k, seed=k)
    a = orc.quantize_q8_1(x)
    ref = orc.q4k_matvec(w, a, rows, k)
    buf, out = with_canaries(rows)
    ops.q4_k_q8_1_matvec(dev(w), dev_bytes(a), out)
    ratio = assert_within_tolerance(out.cpu().numpy(), ref, f"{rows}x{k}")
    assert canaries_intact(buf)
    # fp64 accumulation: errors are at the fp32 rounding level, far inside tolerance
    assert ratio < 0.1


@pytest.mark.parametrize("rows,k", [(4736, 2560), (4737, 2560), (2560, 4096), (1024, 2560), (29, 4096),
                                    (296, 2560)])
def test_resident_shapes_against_oracle(orc, rows, k):
    """Shapes around the resident-weights kernel's limits (at most 32 rows per
    SM, K = 2560 / 4096; 4737 rows fall back to the streaming kernel), odd
    rows per CTA (an idle half-warp) and a partial last CTA."""
    w = fx.seeded_q4k_matrix(rows, k, seed=rows + 3 * k)
    a = orc.quantize_q8_1(fx.seeded_activation(k, seed=k + 1))
    ref = orc.q4k_matvec(w, a, rows, k)
    buf, out = with_canaries(rows)
    ops.q4_k_q8_1_matvec(dev(w), dev_bytes(a), out)
    ratio = assert_within_tolerance(out.cpu().numpy(), ref, f"{rows}x{k}")
    assert canaries_intact(buf)
    assert ratio < 0.1


@pytest.mark.parametrize("rows,k", [(4096, 2560), (2560, 4096)])
def test_pdl_chain_reads_each_activation_after_its_producer(orc, rows, k):
    """quantiser -> matvec -> quantiser -> ... on ONE activation buffer, every
    launch PDL-chained: each matvec prefetches its weights before the
    quantiser that feeds it has finished, and must still use that
    quantiser's output (a stale read shows as the previous step's answer)."""
    import ctypes as C
    from mojo_llm_lab_b200._lib import LAUNCH_PDL, S_D_SUMQ, check, lib
    steps = 6
    w = fx.seeded_q4k_matrix(rows, k, seed=77)
    xs = np.stack([fx.seeded_activation(k, seed=300 + i) * (1 + i) for i in range(steps)])
    wd, xd = dev(w), dev(xs)
    act = torch.empty(k // 32 * 36, dtype=torch.uint8, device="cuda")
    outs = torch.empty(steps, rows, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for i in range(steps):
        check(lib().mllb_q8_1_quantize_ex(xd[i].data_ptr(), act.data_ptr(), k, S_D_SUMQ, LAUNCH_PDL,
                                          C.c_void_p(stream)), "quantize")
        ops.q4_k_q8_1_matvec(wd, act, outs[i], pdl=True)
    got = outs.cpu().numpy()
    for i in range(steps):
        ref = orc.q4k_matvec(w, orc.quantize_q8_1(xs[i]), rows, k)
        assert_within_tolerance(got[i], ref, f"step {i}")
    assert ops.device_error() == 0


def test_seeded_gate_up_full_config(orc):
    rows, k = 9728, 2560
    up_w = fx.seeded_q4k_matrix(rows, k, seed=101)
    gate_w = fx.seeded_q4k_matrix(rows, k, seed=102)
    a = orc.quantize_q8_1(fx.seeded_activation(k, seed=103))
    ref_up, ref_gate, ref_prod = orc.q4k_gate_up(up_w, gate_w, a, rows, k)
    up, gate, prod = ops.q4k_gate_up(dev(up_w), dev(gate_w), dev_bytes(a))
    assert_within_tolerance(up.cpu().numpy(), ref_up, "up")
    assert_within_tolerance(gate.cpu().numpy(), ref_gate, "gate")
    assert_within_tolerance(prod.cpu().numpy(), ref_prod, "prod")
    # every output optional: prod only, up only
    p_only = ops.q4k_gate_up(dev(up_w), dev(gate_w), dev_bytes(a), want=("prod",))[2]
    assert torch.equal(p_only, prod)
    u_only = ops.q4k_gate_up(dev(up_w), dev(gate_w), dev_bytes(a), want=("up",))[0]
    assert torch.equal(u_only, up)


@pytest.mark.parametrize("rows,k", [(64, 2560), (37, 2048), (5, 9728)])
def test_subdots_bit_exact(orc, rows, k):
    w = fx.seeded_q4k_matrix(rows, k, seed=5)
    a = orc.quantize_q8_1(fx.seeded_activation(k, seed=6) * 3)
    dots, sums = ops.q4k_subdots(dev(w), dev_bytes(a))
    ref_dots, ref_sums = orc.q4k_subdots(w, a, rows, k)
    assert np.array_equal(dots.cpu().numpy(), ref_dots)
    assert np.array_equal(sums.cpu().numpy(), ref_sums)


def test_edge_blocks_zero_and_subnormal_factors(orc):
    rows, k = 32, 2560
    w = fx.seeded_q4k_matrix(rows, k, seed=9).reshape(-1, 144).copy()
    w[0::3, 0:4] = 0                                  # d = dmin = 0
    w[1::3, 0:2] = np.array([1, 0], dtype=np.uint8)   # smallest subnormal d
    w[2::5, 2:4] = np.array([0xFF, 0x7B], dtype=np.uint8)  # dmin = 65504
    w = w.reshape(-1)
    x = fx.seeded_activation(k, seed=10)
    x[:32] = 0.0                                      # an all-zero Q8_1 block
    a = orc.quantize_q8_1(x)
    ref = orc.q4k_matvec(w, a, rows, k)
    out = ops.q4_k_q8_1_matvec(dev(w), dev_bytes(a))
    assert_within_tolerance(out.cpu().numpy(), ref, "edge blocks")


def test_rejects_mismatched_sizes():
    w = torch.zeros(1440 * 4, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError):
        ops.q4_k_q8_1_matvec(w, torch.zeros(2879, dtype=torch.uint8, device="cuda"))
    with pytest.raises(ValueError):
        ops.q4_k_q8_1_matvec(w[:1000], torch.zeros(2880, dtype=torch.uint8, device="cuda"))
    with pytest.raises(ValueError):  # misaligned weights
        ops.q4_k_q8_1_matvec(torch.zeros(1440 * 4 + 1, dtype=torch.uint8, device="cuda")[1:],
                             torch.zeros(2880, dtype=torch.uint8, device="cuda"))
