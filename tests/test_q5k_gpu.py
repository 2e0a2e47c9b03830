"""Q5_K x Q8_1 streaming matvec on the GPU against the oracle (public GGML
layout restated in oracle.c; parity unpinned: no reference Q5_K code)."""
import numpy as np
import pytest
import torch

from gpu_util import assert_within_tolerance, canaries_intact, dev, dev_bytes, with_canaries
from mojo_llm_lab_b200 import fixtures as fx
from mojo_llm_lab_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,k", [(4096, 2560), (1, 2560), (17, 2048), (333, 4096), (9728, 2560), (5000, 2048)])
def test_seeded_q5k_against_oracle(orc, rows, k):
    w = fx.seeded_q5k_matrix(rows, k, seed=rows + k)
    a = orc.quantize_q8_1(fx.seeded_activation(k, seed=3) * 7)
    ref = orc.q5k_matvec(w, a, rows, k)
    buf, out = with_canaries(rows)
    ops.q5_k_q8_1_matvec(dev(w), dev_bytes(a), out)
    assert_within_tolerance(out.cpu().numpy(), ref, f"q5k {rows}x{k}")
    assert canaries_intact(buf)
    assert ops.device_error() == 0


def test_q5k_pdl_chain_and_unsupported_k(orc):
    rows, k = 256, 2560
    w = dev(fx.seeded_q5k_matrix(rows, k, seed=1))
    a = dev_bytes(orc.quantize_q8_1(fx.seeded_activation(k, seed=2)))
    plain = ops.q5_k_q8_1_matvec(w, a)
    for _ in range(3):
        chained = ops.q5_k_q8_1_matvec(w, a, pdl=True)
    assert torch.equal(plain, chained)
    w2 = torch.zeros(4 * 3 * 176, dtype=torch.uint8, device="cuda")
    a2 = torch.zeros(768 // 32 * 36, dtype=torch.uint8, device="cuda")
    with pytest.raises(Exception):
        ops.q5_k_q8_1_matvec(w2, a2)   # K = 768: no streaming configuration
