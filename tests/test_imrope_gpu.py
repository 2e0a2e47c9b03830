"""Fused RMSNorm + gamma + IMROPE on the GPU.

Oracle: reference_head (tests/reference_math.py:22-35) in float64.  The
kernel takes the theta scale as a runtime fp32 input (bits 0x3f492c27, as the
reference's harness passes it); the oracle is evaluated at that same scale.
Against the reference's exact-base goldens the runtime fp32 scale itself
differs by 2.4e-8 relative, which moves outputs at position 32768 far beyond
1e-5 -- an input difference, so those goldens are checked through the entry
that takes the scale in float64."""
import hashlib

import numpy as np
import pytest
import torch

from gpu_util import assert_within_tolerance, dev
from mojo_llm_lab_b200 import fixtures as fx
import ref_fixtures as rfx
from mojo_llm_lab_b200 import formats as F
from mojo_llm_lab_b200 import ops

pytestmark = pytest.mark.gpu


def _run_ref_abi(q, gamma, pos):
    theta = torch.tensor([F.theta_scale_f32()], dtype=torch.float32, device="cuda")
    out = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    ops.fused_q_imrope_runtime_fastpow(dev(q), dev(gamma), dev(np.asarray(pos, dtype=np.int32)), out, theta)
    return out.cpu().numpy()


@pytest.mark.parametrize("name", list(rfx.IMROPE_CASES))
def test_reference_fixtures_at_runtime_theta(orc, name):
    q, gamma, pos = fx.parse_imrope(fx.serialize_imrope(rfx.imrope_reference_inputs(rfx.IMROPE_CASES[name])))
    got = _run_ref_abi(q, gamma, pos)
    ref = orc.imrope(q, gamma, pos, orc.runtime_theta_scale())
    assert_within_tolerance(got.reshape(-1), ref.reshape(-1), name)


@pytest.mark.parametrize("name", list(fx.SEEDED_IMROPE_CASES))
def test_seeded_inputs_at_runtime_theta(orc, name):
    inp = fx.imrope_seeded_inputs(fx.SEEDED_IMROPE_CASES[name], seed=2024)
    got = _run_ref_abi(inp["q"], inp["gamma"], inp["positions_axis_major"])
    ref = orc.imrope(inp["q"], inp["gamma"], inp["positions_axis_major"], orc.runtime_theta_scale())
    assert_within_tolerance(got.reshape(-1), ref.reshape(-1), name)


@pytest.mark.parametrize("name", list(rfx.IMROPE_CASES))
def test_reference_goldens_at_exact_theta(golden, name):
    g = golden["imrope_reference_fixtures"][name]
    q, gamma, pos = fx.parse_imrope(fx.serialize_imrope(rfx.imrope_reference_inputs(g["positions"])))
    out = ops.rmsnorm_imrope_q(dev(q), dev(gamma), dev(pos), theta_scale=golden["reference_theta_scale"])
    got = out.cpu().numpy()
    assert_within_tolerance(got[0], g["head0"], name + " head0")
    assert_within_tolerance(got[31], g["head31"], name + " head31")


def test_reference_goldens_need_float64_theta_only_at_long_positions(golden, orc):
    # distinct/fallback: the fp32 runtime scale stays inside tolerance of the
    # exact-base reference; long_position does not (documented input effect).
    for name in ("distinct_axes", "fallback_only"):
        g = golden["imrope_reference_fixtures"][name]
        q, gamma, pos = fx.parse_imrope(fx.serialize_imrope(rfx.imrope_reference_inputs(g["positions"])))
        got = _run_ref_abi(q, gamma, pos)
        assert_within_tolerance(got[0], g["head0"], name)


def test_throughput_mode_many_tokens(orc):
    tokens = 64
    rng = np.random.default_rng(8)
    q = rng.standard_normal((tokens * 32, 128)).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    pos = rng.integers(0, 40000, (tokens, 4)).astype(np.int32)
    theta = torch.tensor([F.theta_scale_f32()], dtype=torch.float32, device="cuda")
    out = ops.rmsnorm_imrope_q(dev(q), dev(gamma), dev(pos), theta_scale=theta).cpu().numpy()
    for t in (0, 17, 63):
        ref = orc.imrope(q[t * 32:(t + 1) * 32], gamma, pos[t], orc.runtime_theta_scale())
        assert_within_tolerance(out[t * 32:(t + 1) * 32].reshape(-1), ref.reshape(-1), f"token {t}")


def test_zero_input_gives_zero():
    out = _run_ref_abi(np.zeros((32, 128), np.float32), np.ones(128, np.float32), [3, 5, 11, 17])
    assert not out.any()


def test_input_fixture_hashes_unchanged(golden):
    for name, g in golden["imrope_reference_fixtures"].items():
        payload = fx.serialize_imrope(rfx.imrope_reference_inputs(g["positions"]))
        assert hashlib.sha256(payload).hexdigest() == g["input_sha256"]


@pytest.mark.parametrize("const_aux", [False, True])
@pytest.mark.parametrize("tokens", [1, 5])
def test_pdl_chain_feeds_each_output_into_the_next(orc, const_aux, tokens):
    """out_i = IMROPE(out_{i-1}), every launch PDL-chained on the previous one.
    With const_aux the rotation table is built before the dependency wait;
    q (the previous launch's output) must still be read after it."""
    rng = np.random.default_rng(31 + tokens)
    q0 = rng.standard_normal((tokens * 32, 128)).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    pos = rng.integers(0, 40000, (tokens, 4)).astype(np.int32)
    theta = torch.tensor([F.theta_scale_f32()], dtype=torch.float32, device="cuda")
    g_d, p_d = dev(gamma), dev(pos)
    bufs = [dev(q0)] + [torch.empty(tokens * 32, 128, dtype=torch.float32, device="cuda") for _ in range(4)]
    for i in range(4):
        ops.rmsnorm_imrope_q(bufs[i], g_d, p_d, theta, out=bufs[i + 1], pdl=True, const_aux=const_aux)
    prev = q0
    for i in range(4):
        got = bufs[i + 1].cpu().numpy()
        for t in range(tokens):
            ref = orc.imrope(prev[t * 32:(t + 1) * 32], gamma, pos[t], orc.runtime_theta_scale())
            assert_within_tolerance(got[t * 32:(t + 1) * 32].reshape(-1), ref.reshape(-1), f"step {i} token {t}")
        prev = got  # the next step starts from the GPU's fp32 values, as the chain did
    assert ops.device_error() == 0
