"""Q4_0 KV-cache oracle on the CPU.

No reference test or fixture touches Q4_0 arithmetic (the reference selects
GGML_TYPE_Q4_0 for its KV cache, integration/resident_decode.cpp:70, and
llama.cpp does the rest), so the oracle's quantiser is checked here against
a second, independent restatement of GGML's quantize_row_q4_0 written with
numpy float32 scalars (every operation rounded to fp32), on random blocks
and on the cases the rule singles out: ties in magnitude, zeros and negative
zeros, the clamp at 15, tiny (fp16 d underflows to 0) and huge values.
"""
import numpy as np
import pytest

F32 = np.float32


def q4_0_block_scalar(xb):
    """GGML quantize_row_q4_0 of one block, numpy-scalar restatement."""
    amax, vmax = F32(0.0), F32(0.0)
    for v in xb:
        if amax < abs(v):
            amax, vmax = abs(v), v
    d = F32(vmax / F32(-8.0))
    inv = F32(F32(1.0) / d) if d != 0 else F32(0.0)
    out = bytearray(np.array([d], dtype=np.float16).tobytes())
    for j in range(16):
        q0 = min(15, int(F32(F32(xb[j] * inv) + F32(8.5))))
        q1 = min(15, int(F32(F32(xb[j + 16] * inv) + F32(8.5))))
        out.append(q0 | (q1 << 4))
    return bytes(out)


def edge_blocks():
    rng = np.random.default_rng(3)
    # (Down to 1e-30: below ~1e-37 1 / d overflows to inf and GGML's
    # float-to-int conversion of x * inf is undefined in C.)
    blocks = [rng.standard_normal(32).astype(F32) * F32(s) for s in (1.0, 1e-3, 1e4, 1e-30)]
    zeros = np.zeros(32, dtype=F32)
    neg_zero = zeros.copy()
    neg_zero[0] = F32(-0.0)
    tie = rng.standard_normal(32).astype(F32) * F32(0.1)
    tie[5], tie[9] = F32(-2.0), F32(2.0)      # equal magnitude: the first (-2) wins
    tie_pos = tie.copy()
    tie_pos[5], tie_pos[9] = F32(2.0), F32(-2.0)
    ramp = (np.arange(32, dtype=F32) - F32(8.0))
    clamp = np.full(32, F32(-1.0))
    clamp[0] = F32(1.0)                         # vmax = +1: every -1 maps past 15
    halves = (np.arange(32, dtype=F32) * F32(0.25)) - F32(4.0)
    single = zeros.copy()
    single[31] = F32(-7.5)
    blocks += [zeros, neg_zero, tie, tie_pos, ramp, clamp, halves, single]
    return blocks


@pytest.mark.parametrize("i", range(12))
def test_quantizer_matches_scalar_restatement(orc, i):
    xb = edge_blocks()[i]
    assert bytes(orc.quantize_q4_0(xb)) == q4_0_block_scalar(xb)


def test_quantizer_random_blocks(orc):
    rng = np.random.default_rng(11)
    x = (rng.standard_normal(32 * 400) * rng.choice([1e-4, 1.0, 50.0], 32 * 400)).astype(F32)
    got = orc.quantize_q4_0(x)
    want = b"".join(q4_0_block_scalar(x[b * 32:(b + 1) * 32]) for b in range(400))
    assert bytes(got) == want


def test_zero_block_and_ties(orc):
    z = orc.quantize_q4_0(np.zeros(32, dtype=F32))
    assert z[:2].view(np.uint16)[0] == 0x8000      # d = +0 / -8 = -0
    assert set(z[2:]) == {0x88}                     # id = 0: every q is 8
    tie = np.zeros(32, dtype=F32)
    tie[3], tie[4] = F32(-4.0), F32(4.0)
    b = orc.quantize_q4_0(tie)
    assert b[:2].view(np.float16)[0] == np.float16(0.5)   # vmax = -4 (first): d = 0.5
    vals = orc.dequantize_q4_0(b)
    assert vals[3] == -4.0 and vals[4] == 3.5             # +4 -> q 16, clamped to 15


def test_round_trip_error_bound(orc):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(32 * 256).astype(F32)
    blocks = orc.quantize_q4_0(x).reshape(-1, 18)
    d = np.abs(blocks[:, :2].copy().view(np.float16).astype(np.float64)).repeat(32)
    err = np.abs(orc.dequantize_q4_0(blocks) - x.astype(np.float64))
    # Within half a step, except the clamp at 15 (the value -vmax), within one.
    assert np.all(err <= d * 1.001 + 1e-12)
    assert np.mean(err <= d * 0.5 * 1.001 + 1e-12) > 0.99


def test_cache_planes_split_the_blocks(orc):
    rng = np.random.default_rng(6)
    rows = rng.standard_normal((3, 5, 128)).astype(F32)
    qs, d = orc.kv_q4_0_rows(rows)
    assert qs.shape == (3, 5, 64) and d.shape == (3, 5, 4)
    blocks = orc.quantize_q4_0(rows).reshape(3, 5, 4, 18)
    assert np.array_equal(qs.reshape(3, 5, 4, 16), blocks[..., 2:])
    assert np.array_equal(d, blocks[..., :2].copy().view(np.uint16)[..., 0])


def dequant_planes(qs, d):
    """float64 rows [..., 128] of Q4_0 planes (qs [..., 64], d [..., 4] fp16 bits)."""
    lead = qs.shape[:-1]
    nib = qs.reshape(*lead, 4, 16)
    vals = np.concatenate([(nib & 15), (nib >> 4)], axis=-1).astype(np.float64) - 8.0
    scale = d.view(np.float16).astype(np.float64)[..., None]
    return (vals * scale).reshape(*lead, 128)


@pytest.mark.parametrize("hq,hkv,ctx,n", [(8, 2, 40, 40), (4, 4, 17, 9), (16, 2, 64, 1)])
def test_attention_q4_0_equals_float64_on_dequantised_rows(orc, hq, hkv, ctx, n):
    rng = np.random.default_rng(ctx + n)
    k, v = (rng.standard_normal((hkv, ctx, 128)).astype(F32) for _ in range(2))
    kq, kd = orc.kv_q4_0_rows(k)
    vq, vd = orc.kv_q4_0_rows(v)
    d = np.ascontiguousarray(np.concatenate([kd, vd], axis=-1))
    q = rng.standard_normal(hq * 128).astype(F32)
    got = orc.attention_q4_0(q, kq, vq, d, n, hq, hkv)
    kf, vf = dequant_planes(kq, kd), dequant_planes(vq, vd)
    want = np.empty(hq * 128)
    for h in range(hq):
        j = h // (hq // hkv)
        s = kf[j, :n] @ q[h * 128:(h + 1) * 128].astype(np.float64) / np.sqrt(128.0)
        p = np.exp(s - s.max())
        want[h * 128:(h + 1) * 128] = p @ vf[j, :n] / p.sum()
    np.testing.assert_allclose(got, want.astype(F32), rtol=1e-6, atol=1e-7)


def test_qk_rope_f32_rounds_to_the_fp16_rows(orc):
    rng = np.random.default_rng(8)
    hq, hkv = 8, 2
    qkv = (rng.standard_normal((hq + 2 * hkv) * 128) * 20).astype(F32)
    qg, kg = (rng.uniform(0.5, 1.5, 128).astype(F32) for _ in range(2))
    q1, k16, v16 = orc.qk_rope_append(qkv, hq, hkv, qg, kg, 77, 0.7)
    q2, k32, v32 = orc.qk_rope_f32(qkv, hq, hkv, qg, kg, 77, 0.7)
    assert np.array_equal(q1, q2)
    assert np.array_equal(k32.astype(np.float16).view(np.uint16), k16)
    assert np.array_equal(v32.astype(np.float16).view(np.uint16), v16)
