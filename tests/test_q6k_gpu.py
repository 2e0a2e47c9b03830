"""Q6_K x Q8_1 vocabulary projection on the GPU against the oracle.

Parity for Q6_K is against this repository's float64 oracle of the public GGML
layout: the reference has no Q6_K oracle or fixture (parity unpinned)."""
import numpy as np
import pytest

from gpu_util import assert_within_tolerance, canaries_intact, dev, dev_bytes, with_canaries
from mojo_llm_lab_b200 import fixtures as fx
from mojo_llm_lab_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,k", [(151936, 2560), (1, 2560), (7, 2560), (16, 2560), (23, 2560),
                                    (18992, 2560), (1000, 2048), (100, 4096), (9, 9728)])
def test_seeded_q6k_against_oracle(orc, rows, k):
    w = fx.seeded_q6k_matrix(rows, k, seed=rows + k)
    a = orc.quantize_q8_1(fx.seeded_activation(k, seed=77))
    ref = orc.q6k_matvec(w, a, rows, k)
    buf, out = with_canaries(rows)
    ops.q6_k_q8_1_matvec(dev(w), dev_bytes(a), out)
    ratio = assert_within_tolerance(out.cpu().numpy(), ref, f"q6k {rows}x{k}")
    assert canaries_intact(buf)
    assert ratio < 0.1
    assert ops.device_error() == 0


def test_q6k_extreme_scales(orc):
    rows, k = 64, 2560
    w = fx.seeded_q6k_matrix(rows, k, seed=1).reshape(-1, 210).copy()
    w[::4, 192:208] = np.uint8(0x80)   # scales -128
    w[1::4, 192:208] = np.uint8(0x7F)  # scales 127
    w[2::4, 208:210] = 0               # d = 0
    w[3::4, 0:192] = 0xFF              # q6 = 63 everywhere
    w = w.reshape(-1)
    a = orc.quantize_q8_1(fx.seeded_activation(k, seed=2) * 50)
    ref = orc.q6k_matvec(w, a, rows, k)
    out = ops.q6_k_q8_1_matvec(dev(w), dev_bytes(a))
    assert_within_tolerance(out.cpu().numpy(), ref, "q6k extremes")
