"""The CPU oracle against golden vectors produced by the reference's own code.

Every comparison here is exact (==): the oracle restates the reference's
float64 arithmetic in the same operation order, so it must reproduce it bit
for bit.  tests/golden/make_golden.py documents how golden.json was made.
"""
import hashlib
import struct

import numpy as np
import pytest

from mojo_llm_lab_b200 import fixtures as fx
import ref_fixtures as rfx


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def test_position_axis_matches_reference(orc, golden):
    assert [orc.position_axis(p) for p in range(64)] == golden["position_axis"]
    # tests/test_reference_math.py:39-43 known axes, fallback pairs 61/62 -> axis 3
    wanted = {0: 0, 1: 1, 2: 2, 23: 2, 24: 0, 43: 1, 44: 2, 59: 2, 60: 0, 61: 3, 62: 3, 63: 0}
    assert {p: orc.position_axis(p) for p in wanted} == wanted


def test_reference_theta_scale_bits(orc, golden):
    assert orc.reference_theta_scale() == golden["reference_theta_scale"]
    # the runtime fp32 value is the fp32 nearest to the exact scale
    assert np.float32(golden["reference_theta_scale"]).view(np.uint32) == orc.THETA_SCALE_BITS


@pytest.mark.parametrize("name", ["distinct_axes", "long_position", "fallback_only"])
def test_imrope_reference_fixtures_bit_exact(orc, golden, name):
    g = golden["imrope_reference_fixtures"][name]
    payload = fx.serialize_imrope(rfx.imrope_reference_inputs(g["positions"]))
    assert sha(payload) == g["input_sha256"]
    q, gamma, positions = fx.parse_imrope(payload)
    out = orc.imrope(q, gamma, positions, orc.reference_theta_scale())
    assert out[0].tolist() == g["head0"]
    assert out[31].tolist() == g["head31"]
    assert sha(out.tobytes()) == g["output_sha256"]


@pytest.mark.parametrize("name", ["distinct_axes", "long_position", "fallback_only"])
def test_imrope_seeded_bit_exact(orc, golden, name):
    g = golden["imrope_seeded"][name]
    inputs = fx.imrope_seeded_inputs(g["positions"], seed=g["seed"])
    assert sha(inputs["q"].tobytes() + inputs["gamma"].tobytes()) == g["input_sha256"]
    out = orc.imrope(inputs["q"], inputs["gamma"], g["positions"], orc.reference_theta_scale())
    assert out[0].tolist() == g["head0"]
    assert sha(out.tobytes()) == g["output_sha256"]


def test_imrope_contract_cases(orc):
    # zero in -> zero out (tests/test_reference_math.py:45-47)
    assert orc.reference_head([0.0] * 128, [1.0] * 128, [3, 5, 11, 17]) == [0.0] * 128
    # RMS is per head, gamma shared (tests/test_reference_math.py:93-102)
    gamma = [1 + i / 128 for i in range(128)]
    for magnitude in (1, 7, 32):
        out = orc.reference_head([float(magnitude)] * 128, gamma, [0] * 4)
        factor = magnitude / np.sqrt(magnitude * magnitude + 1e-6)
        assert np.allclose(out, factor * np.array(gamma), atol=1e-14, rtol=0)
    with pytest.raises(ValueError):
        orc.reference_head([1.0] * 128, [1.0] * 4096, [0] * 4)


@pytest.mark.parametrize("case", ["default", "random_quants", "gate_up", "gate_up_rows128",
                                  "varied_factors", "varied_activations",
                                  "default_activation_scales", "width2048"])
def test_q4_dot_bit_exact_on_reference_fixtures(orc, golden, case):
    g = golden["q4_reference_fixtures"][case]
    files = rfx.q4_matvec_fixtures(**g["options"])
    assert {k: sha(v) for k, v in files.items()} == g["sha256"]
    width = g["options"].get("input_width", 2560)
    for key in ("weights", "gate"):
        if "dot_" + key in g:
            w = files[key + ".bin"]
            rows = len(w) // (width // 256 * 144)
            got = orc.q4k_matvec(w, files["activations.bin"], rows, width)
            assert got.tolist() == g["dot_" + key]


def test_q4_dot_bit_exact_on_seeded_rows(orc, golden):
    g = golden["q4_seeded"]
    w = fx.seeded_q4k_matrix(g["rows"], g["k"], seed=g["weight_seed"]).tobytes()
    x = fx.seeded_activation(g["k"], seed=g["activation_seed"])
    assert sha(w) == g["weights_sha256"] and sha(x.tobytes()) == g["x_sha256"]
    a = orc.quantize_q8_1(x)
    assert sha(a) == g["q8_1_sha256"]
    assert orc.q4k_matvec(w, a, g["rows"], g["k"]).tolist() == g["dot"]


def test_q8_1_known_answer_reproduces_reference_activations(orc, golden):
    g = golden["q8_1_known_answer"]
    x = np.array(g["x"], dtype=np.float32)
    assert np.array_equal(x.astype(np.float64), np.array(g["x"]))  # exact in fp32
    for mode in (orc.S_D_TIMES_SUMQ, orc.S_SUM_X):
        assert sha(orc.quantize_q8_1(x, mode)) == g["bytes_sha256"]


def test_q8_1_rules(orc):
    # amax / 127 == d, round(x / d) == q, zero block -> zeros, ties away from zero
    x = np.zeros(64, dtype=np.float32)
    x[0] = 2.54
    x[1] = -1.27  # exactly -0.5 * amax -> q = -63.5 -> rounds away from zero to -64
    out = orc.quantize_q8_1(x)
    d = struct.unpack_from("<e", out, 0)[0]
    q = struct.unpack_from("<32b", out, 4)
    d32 = np.float32(2.54) / np.float32(127)
    assert d == float(np.float16(d32))
    assert q[0] == 127 and q[1] == int(np.sign(x[1] / d32) * np.floor(abs(x[1] / d32) + 0.5))
    assert out[36:] == bytes(36)  # all-zero block


def test_half_conversions_match_numpy(orc):
    rng = np.random.default_rng(5)
    vals = np.concatenate([rng.standard_normal(4000) * 10.0 ** rng.integers(-9, 5, 4000),
                           np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e-8, 2.9802322e-08, 5.96e-8,
                                     6.1035156e-05, 6.1e-05, -3.0e-7], dtype=np.float32)]).astype(np.float32)
    ours = np.array([orc.float_to_half(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(ours, vals.astype(np.float16).view(np.uint16))
    for bits in list(range(0, 65536, 97)) + [0x0001, 0x03ff, 0x0400, 0x7bff, 0x7c00, 0x8001]:
        want = float(np.uint16(bits).view(np.float16))
        got = orc.half_to_double(bits)
        assert (np.isnan(got) and np.isnan(want)) or got == want


def test_fsum_matches_python_fsum(orc):
    import math
    rng = np.random.default_rng(7)
    for _ in range(50):
        v = rng.standard_normal(rng.integers(1, 3000)) * 10.0 ** rng.integers(-20, 20, 1)
        v[::7] *= 1e12
        assert orc.fsum(v) == math.fsum(v.tolist())
    assert orc.fsum([1e308, 1.0, -1e308]) == math.fsum([1e308, 1.0, -1e308])
    assert orc.fsum([0.1] * 10) == math.fsum([0.1] * 10)


def test_q4_decoder_all_six_bit_values(orc):
    # tests/test_q4_reference.py:17-24 restated: every 6-bit scale/min, both nibbles
    from mojo_llm_lab_b200 import formats as F
    for value in range(64):
        scales = [(value + j * 7) % 64 for j in range(8)]
        minima = [(63 - value + j * 11) % 64 for j in range(8)]
        got = orc.decode_block(F.q4k_block(scales, minima, 0.5, 0.25, rfx.DEMO_QUANTS))
        want = [0.5 * scales[g] * (lane % 16 if g % 2 == 0 else 15 - lane % 16) - 0.25 * minima[g]
                for g in range(8) for lane in range(32)]
        assert got == want


def test_q4_dot_reference_contract_cases(orc):
    # tests/test_q4_dot.py:13-23 restated
    from mojo_llm_lab_b200 import formats as F
    weights = F.q4k_block([1] * 8, [0] * 8, 1, 0, rfx.DEMO_QUANTS) * 10
    groups = [struct.pack("<ee32b", (g + 1) / 8, 0, *([1] * 32)) for g in range(8)]
    assert orc.dot_q4_q8(weights, b"".join(groups) * 10) == 10 * 240 * sum((g + 1) / 8 for g in range(8))
    weights = F.q4k_block([0] * 8, [1] * 8, 0, 0.5, rfx.DEMO_QUANTS)
    assert orc.dot_q4_q8(weights, struct.pack("<ee32b", 1, 0, *([1, -1] * 16)) * 8) == 0
    assert orc.dot_q4_q8(weights, struct.pack("<ee32b", 1, 32, *([1] * 32)) * 8) == -128
    for w, a in [(b"", b""), (bytes(144), bytes(36)), (bytes(145), bytes(288))]:
        with pytest.raises(ValueError):
            orc.dot_q4_q8(w, a)


def test_q6k_decoder_layout(orc):
    # q6 = low nibble | high 2 bits << 4, minus 32; element order of the public layout
    blk = bytearray(210)
    blk[0] = 0x21          # ql[0]: element 0 low nibble 1, element 64 high nibble 2
    blk[32] = 0x43         # ql[32]: element 32 low 3, element 96 high 4
    blk[128] = 0b11100100  # qh[0]: e0 +0<<4, e32 +1<<4, e64 +2<<4, e96 +3<<4
    for j in range(16):
        blk[192 + j] = (j + 1) & 0xFF
    blk[208:210] = struct.pack("<e", 0.5)
    v = orc.q6k_decode_block(bytes(blk))
    assert v[0] == 0.5 * 1 * (1 - 32)
    assert v[32] == 0.5 * 3 * ((3 | 16) - 32)
    assert v[64] == 0.5 * 5 * ((2 | 32) - 32)
    assert v[96] == 0.5 * 7 * ((4 | 48) - 32)
    assert v[16] == 0.5 * 2 * (0 - 32)   # second sub-block scale for l >= 16
    assert v[128] == 0.5 * 9 * (0 - 32)  # second half uses scales 8..15


# ------------------------------------------------ pure-Python port (CPU baseline)

def test_python_port_dot_bit_exact_on_golden(golden):
    from oracle import pyport
    g = golden["q4_reference_fixtures"]["varied_factors"]
    files = rfx.q4_matvec_fixtures(**g["options"])
    w, a = files["weights.bin"], files["activations.bin"]
    row = 10 * 144
    got = [pyport.dot_q4_q8(w[r * row:(r + 1) * row], a) for r in range(8)]
    assert got == g["dot_weights"][:8]
    s = golden["q4_seeded"]
    w = fx.seeded_q4k_matrix(s["rows"], s["k"], seed=s["weight_seed"])
    import oracle
    a = oracle.quantize_q8_1(fx.seeded_activation(s["k"], seed=s["activation_seed"]))
    row = s["k"] // 256 * 144
    assert [pyport.dot_q4_q8(w[r * row:(r + 1) * row].tobytes(), a) for r in range(4)] == s["dot"][:4]


def test_python_port_head_bit_exact_on_golden(golden):
    from oracle import pyport
    g = golden["imrope_reference_fixtures"]["long_position"]
    q, gamma, positions = fx.parse_imrope(fx.serialize_imrope(rfx.imrope_reference_inputs(g["positions"])))
    q64, g64 = q.astype(np.float64), gamma.astype(np.float64).tolist()
    assert pyport.reference_head(q64[0].tolist(), g64, positions.tolist()) == g["head0"]
    assert pyport.reference_head(q64[31].tolist(), g64, positions.tolist()) == g["head31"]
