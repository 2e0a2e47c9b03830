"""Batched-token Q4_K x Q8_1 (prompt processing) on the tensor cores against
the oracle: every token's output row within 1e-5 + 1e-5 |ref| of the oracle's
matvec of that token, for single-split and K-split grids, token counts that
are not whole 32-token tiles, and the shapes of the decode stack."""
import numpy as np
import pytest
import torch

from gpu_util import assert_within_tolerance, dev
from mojo_llm_lab_b200 import fixtures as fx
from mojo_llm_lab_b200 import formats as F
from mojo_llm_lab_b200 import ops

pytestmark = pytest.mark.gpu


def tokens_q8(orc, k, tokens, seed):
    rows = [orc.quantize_q8_1(fx.seeded_activation(k, seed=seed + t)) for t in range(tokens)]
    return np.frombuffer(b"".join(rows), dtype=np.uint8).reshape(tokens, -1)


@pytest.mark.parametrize("rows,k,tokens", [(128, 256, 8), (128, 2560, 32), (256, 2560, 45), (4096, 2560, 64),
                                           (2560, 9728, 32), (9728, 2560, 32), (1024, 4096, 100)])
def test_matmul_tokens_against_oracle(orc, rows, k, tokens):
    w = fx.seeded_q4k_matrix(rows, k, seed=rows + k)
    a = tokens_q8(orc, k, tokens, seed=tokens)
    out = ops.q4k_matmul_tokens(dev(w), dev(a))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    check = range(tokens) if tokens <= 8 else sorted({0, 1, tokens // 2, tokens - 1})
    for t in check:
        ref = orc.q4k_matvec(w, a[t].tobytes(), rows, k)
        assert_within_tolerance(got[t], ref, f"token {t}")
    assert ops.device_error() == 0


def test_matmul_tokens_matches_the_matvec():
    rows, k, tokens = 4096, 2560, 33
    w = dev(fx.seeded_q4k_matrix(rows, k, seed=3))
    xs = torch.stack([torch.from_numpy(fx.seeded_activation(k, seed=50 + t)) for t in range(tokens)]).cuda()
    a = torch.stack([ops.quantize_q8_1(xs[t]) for t in range(tokens)])
    out = ops.q4k_matmul_tokens(w, a)
    for t in (0, 17, 32):
        ref = ops.q4_k_q8_1_matvec(w, a[t]).cpu().numpy()
        assert_within_tolerance(out[t].cpu().numpy(), ref, f"token {t}")


def test_matmul_tokens_rejects_bad_shapes():
    from mojo_llm_lab_b200._lib import MLLB_EINVAL, lib
    L = lib()
    assert L.mllb_q4k_matmul_tokens_workspace(100, 2560, 4) == MLLB_EINVAL   # rows not a multiple of 128
    assert L.mllb_q4k_matmul_tokens_workspace(128, 2500, 4) == MLLB_EINVAL   # K not a multiple of 256
    assert L.mllb_q4k_matmul_tokens_workspace(128, 2560, 0) == MLLB_EINVAL
    w = torch.zeros(4096 * F.q4k_row_bytes(2560), dtype=torch.uint8, device="cuda")
    a = torch.zeros(64, F.q8_1_bytes(2560), dtype=torch.uint8, device="cuda")
    out = torch.zeros(64, 4096, device="cuda")
    need = L.mllb_q4k_matmul_tokens_workspace(4096, 2560, 64)
    assert need > 0
    # a K-split plan without its workspace is refused before any launch
    assert L.mllb_q4k_matmul_tokens(w.data_ptr(), a.data_ptr(), out.data_ptr(), 4096, 2560, 64, None, 0, 0,
                                    None) == MLLB_EINVAL
