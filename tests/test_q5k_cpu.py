"""Q5_K oracle (oracle.c) against a numpy restatement of GGML's published
dequantisation (block_q5_K; the j / is / u1 / u2 loop of dequantize_row_q5_K).
The reference has no Q5_K code, so this pins the oracle to the format, not to
reference outputs (parity unpinned)."""
import numpy as np
import pytest

from mojo_llm_lab_b200 import fixtures as fx
from mojo_llm_lab_b200 import formats as F


def ggml_style_dequant(block: np.ndarray) -> np.ndarray:
    d = float(block[0:2].view(np.float16)[0])
    dmin = float(block[2:4].view(np.float16)[0])
    sc = block[4:16]
    qh, ql = block[16:48], block[48:176]

    def scale_min(j):
        if j < 4:
            return sc[j] & 63, sc[j + 4] & 63
        return (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4), (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4)

    y = np.empty(256)
    u1, u2, is_, q = 1, 2, 0, 0
    for j in range(0, 256, 64):
        s1, m1 = scale_min(is_)
        s2, m2 = scale_min(is_ + 1)
        for l in range(32):
            y[j + l] = d * s1 * ((ql[q + l] & 0xF) + (16 if qh[l] & u1 else 0)) - dmin * m1
        for l in range(32):
            y[j + 32 + l] = d * s2 * ((ql[q + l] >> 4) + (16 if qh[l] & u2 else 0)) - dmin * m2
        q += 32
        is_ += 2
        u1 <<= 2
        u2 <<= 2
    return y


@pytest.mark.parametrize("seed", range(6))
def test_q5k_decode_matches_ggml_restatement(orc, seed):
    blocks = fx.seeded_q5k_matrix(4, 256, seed=seed).reshape(-1, F.Q5K_BLOCK_BYTES)
    for b in blocks:
        assert np.array_equal(np.array(orc.q5k_decode_block(b.tobytes())), ggml_style_dequant(b))


def test_q5k_extremes(orc):
    b = np.zeros(176, dtype=np.uint8)
    b[0:2] = np.array([-0.5], dtype=np.float16).view(np.uint8)   # negative d
    b[2:4] = np.array([0.25], dtype=np.float16).view(np.uint8)
    b[4:16] = 0xFF                                                # every scale / min = 63
    b[16:48] = 0xFF                                               # every fifth bit set
    b[48:176] = 0xFF                                              # every nibble 15
    got = np.array(orc.q5k_decode_block(b.tobytes()))
    assert np.array_equal(got, ggml_style_dequant(b))
    assert np.allclose(got, -0.5 * 63 * 31 - 0.25 * 63)


def test_q5k_matvec_matches_decoded_dot(orc):
    rows, k = 3, 512
    w = fx.seeded_q5k_matrix(rows, k, seed=9)
    x = fx.seeded_activation(k, seed=10)
    a = orc.quantize_q8_1(x)
    got = orc.q5k_matvec(w, a, rows, k)
    act = np.concatenate([orc.decode_q8_1(a[i * 36:(i + 1) * 36]) for i in range(k // 32)])
    for r in range(rows):
        vals = np.concatenate([orc.q5k_decode_block(w[(r * 2 + b) * 176:(r * 2 + b + 1) * 176]) for b in range(2)])
        assert got[r] == pytest.approx(float(np.sum(vals * act)), rel=1e-12)
