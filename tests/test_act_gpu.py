"""Streaming matvecs that build their Q8_1 activation in the kernel from fp32.

Each must equal the two-kernel path (mllb_rmsnorm_q8_1 or mllb_q8_1_quantize,
then the matvec) and the oracle: bit for bit without a norm (the Q8_1 bytes
are the same), within the 1e-5 + 1e-5 |ref| tolerance with one (the norm's
sum of squares is added in another order, so r can differ in its last bit).
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_within_tolerance, dev
from mojo_llm_lab_b200 import decode as D
from mojo_llm_lab_b200 import fixtures as fx
from mojo_llm_lab_b200 import ops

pytestmark = pytest.mark.gpu


def vectors(k, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(k) * scale).astype(np.float32)
    d = (rng.standard_normal(k) * scale).astype(np.float32)
    g = rng.uniform(0.5, 1.5, k).astype(np.float32)
    return x, d, g


@pytest.mark.parametrize("rows,k", [(6144, 2560), (2560, 9728), (4096, 2048), (333, 4096), (17, 2560)])
def test_q4k_matvec_act_norm_against_oracle(orc, rows, k):
    w = fx.seeded_q4k_matrix(rows, k, seed=rows + k)
    x, d, g = vectors(k, seed=k, scale=40.0)
    x_out = torch.full((k,), 5.0, device="cuda")
    out = torch.empty(rows, device="cuda")
    ops.q4k_matvec_act(dev(w), ops.act_f32(dev(x), dev(d), dev(g), x_out), k, out)
    h_ref, q8 = orc.rmsnorm_q8_1(x, d, g)
    assert np.array_equal(x_out.cpu().numpy(), h_ref)
    ref = orc.q4k_matvec(w, q8, rows, k)
    assert_within_tolerance(out.cpu().numpy(), ref, f"q4k act {rows}x{k}")
    assert ops.device_error() == 0


@pytest.mark.parametrize("rows,k", [(2560, 9728), (2560, 2560), (64, 4096)])
def test_q4k_matvec_act_plain_quantise_is_bit_exact(rows, k):
    w = dev(fx.seeded_q4k_matrix(rows, k, seed=3))
    x = dev(vectors(k, seed=4, scale=1e4)[0])
    fused = torch.empty(rows, device="cuda")
    ops.q4k_matvec_act(w, ops.act_f32(x), k, fused)
    two = ops.q4_k_q8_1_matvec(w, ops.quantize_q8_1(x))
    assert torch.equal(fused, two)


def test_gate_up_act_against_oracle(orc):
    rows, k = 9728, 2560
    up_w = fx.seeded_q4k_matrix(rows, k, seed=1)
    gate_w = fx.seeded_q4k_matrix(rows, k, seed=2)
    x, d, g = vectors(k, seed=5, scale=3.0)
    x_out = torch.empty(k, device="cuda")
    up, gate, prod = (torch.empty(rows, device="cuda") for _ in range(3))
    ops.q4k_gate_up_act(dev(up_w), dev(gate_w), ops.act_f32(dev(x), dev(d), dev(g), x_out), k, up, gate, prod)
    h_ref, q8 = orc.rmsnorm_q8_1(x, d, g)
    assert np.array_equal(x_out.cpu().numpy(), h_ref)
    ru, rg, rp = orc.q4k_gate_up(up_w, gate_w, q8, rows, k)
    assert_within_tolerance(up.cpu().numpy(), ru, "up")
    assert_within_tolerance(gate.cpu().numpy(), rg, "gate")
    assert_within_tolerance(prod.cpu().numpy(), rp, "prod")


@pytest.mark.parametrize("rows,k", [(151936, 2560), (1000, 2048), (64, 4096)])
def test_q6k_act_with_state_advance(orc, rows, k):
    w = fx.seeded_q6k_matrix(rows, k, seed=rows)
    x, d, g = vectors(k, seed=6, scale=1e3)
    state = torch.frombuffer(bytearray(D.state_bytes(9, 4096, 3)), dtype=torch.uint8).cuda()
    out = torch.empty(rows, device="cuda")
    ops.q6k_matvec_act(dev(w), ops.act_f32(dev(x), dev(d), dev(g), advance=state), k, out)
    _, q8 = orc.rmsnorm_q8_1(x, d, g)
    assert_within_tolerance(out.cpu().numpy(), orc.q6k_matvec(w, q8, rows, k), "q6k act")
    st = D.parse_state(bytes(state.cpu().numpy().tobytes()))
    assert st["pos"] == 4097 and st["steps"] == 4 and st["next_token"] == -1


def test_act_rejects_bad_sources():
    k = 2560
    w = torch.zeros(16 * k // 256 * 144, dtype=torch.uint8, device="cuda")
    x = torch.zeros(k + 64, device="cuda")
    out = torch.empty(16, device="cuda")
    with pytest.raises(Exception):  # x_out overlaps x
        ops.q4k_matvec_act(w, ops.act_f32(x[:k], x_out=x[64:]), k, out)
    w2 = torch.zeros(16 * 512 // 256 * 144, dtype=torch.uint8, device="cuda")
    with pytest.raises(Exception):  # K=512: no streaming configuration
        ops.q4k_matvec_act(w2, ops.act_f32(torch.zeros(512, device="cuda")), 512, out)
