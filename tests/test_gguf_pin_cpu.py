"""Parity pins for the formats the reference leaves to GGML: Q6_K (the vocab
projection, GGML's `mul_mat_vec_q<Q6_K>` in docs/q6k-vocab-roofline.md:7-14),
Q5_K (docs/qwen35-2b-profile.md:9-14), the Q4_0 KV cache
(integration/resident_decode.cpp:70) and the GGUF container.

The algorithm lives in llama.cpp/GGML (b12110, un-vendored).  Its own Python
restatement ships here as the `gguf` package (gguf-py 0.19.0:
`gguf.quants.{Q4_K,Q5_K,Q6_K}.dequantize_blocks`, `Q4_0.quantize_blocks`,
`GGUFReader` / `GGUFWriter`), so these tests hold the oracle's decoders,
quantiser and our GGUF reader/writer to it.  The GPU tests compare the kernels
with the oracle, so they inherit the pin.

Exactness: gguf-py dequantises in fp32.  With the block scale d = 1 (Q4_K /
Q5_K also d = 1, dmin = 0, and d = 0, dmin = 1) every dequantised value is a
small integer (scale * (q - 32), sc * q, -m), exact in fp32, so the comparison
is bit-exact and tests the index map itself.  With seeded d / dmin, values
match to fp32 rounding, and whole-row dot products through gguf-py's weights
match the oracle's matvec.  gguf-py is test infrastructure only: nothing in
mojo_llm_lab_b200/ or bench.py imports it.
"""
import math

import numpy as np
import pytest

import oracle
from mojo_llm_lab_b200 import fixtures as fx
from mojo_llm_lab_b200 import gguf as ours

gguf = pytest.importorskip("gguf")
from gguf.constants import GGMLQuantizationType as QT  # noqa: E402
import gguf.quants as gq  # noqa: E402

F16_ONE = np.frombuffer(np.float16(1.0).tobytes(), dtype=np.uint8)


def _gguf_values(blocks: np.ndarray, qtype) -> np.ndarray:
    return gq.dequantize(np.ascontiguousarray(blocks).reshape(-1), qtype).reshape(blocks.shape[0], 256)


def _oracle_values(blocks: np.ndarray, decode) -> np.ndarray:
    return np.array([decode(b.tobytes()) for b in blocks], dtype=np.float64)


# ------------------------------------------------------------------ Q6_K

def _q6k_blocks(n: int, seed: int) -> np.ndarray:
    """Seeded blocks plus the edge cases of every field: int8 scales -128 / 127 /
    +-32 / 0, 6-bit quants all 0 and all 63 (ql = 0x00 / 0xff, qh = 0x00 / 0xff)."""
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (n, 210), dtype=np.uint8)
    edge_scales = np.array([-128, 127, -32, 32, 0, -1, 1, 31, -128, 127, 64, -64, 5, -5, 100, -100], dtype=np.int8)
    b[0, 192:208] = edge_scales.view(np.uint8)
    b[1, 0:192] = 0x00            # q6 = 0 everywhere
    b[2, 0:192] = 0xFF            # q6 = 63 everywhere
    b[3, 192:208] = np.int8(-128).view(np.uint8)
    b[3, 0:192] = 0xFF
    b[4, 192:208] = np.int8(127).view(np.uint8)
    b[4, 0:192] = 0x00
    return b


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_q6k_index_map_exact_with_unit_scale(seed):
    b = _q6k_blocks(256, seed)
    b[:, 208:210] = F16_ONE
    got = _oracle_values(b, oracle.q6k_decode_block)
    ref = _gguf_values(b, QT.Q6_K).astype(np.float64)
    assert np.array_equal(got, ref)


def test_q6k_field_edges_with_extreme_d():
    """d = 0, the smallest subnormal, 1 and 65504 (fp16 max) on the edge blocks."""
    b = np.repeat(_q6k_blocks(5, 7), 4, axis=0)
    for i, dv in enumerate([0.0, 2.0 ** -24, 1.0, 65504.0]):
        b[i::4, 208:210] = np.frombuffer(np.float16(dv).tobytes(), dtype=np.uint8)
    got = _oracle_values(b, oracle.q6k_decode_block)
    ref = _gguf_values(b, QT.Q6_K).astype(np.float64)
    # d * scale * (q - 32): at most 11 + 8 + 6 significant bits, exact in fp32
    # except where fp32 overflows (65504 * 128 * 32 < 2^31 * ... stays finite).
    assert np.array_equal(got, ref)


def test_q6k_seeded_values_match_to_fp32():
    b = fx.seeded_q6k_matrix(64, 2560, seed=4).reshape(-1, 210)
    got = _oracle_values(b, oracle.q6k_decode_block)
    ref = _gguf_values(b, QT.Q6_K).astype(np.float64)
    assert np.array_equal(got.astype(np.float32).astype(np.float64), ref)


def _q8_values(act: bytes) -> np.ndarray:
    """fp64 values d * q of Q8_1 blocks (fp16 d, fp16 s, 32 x int8)."""
    b = np.frombuffer(act, dtype=np.uint8).reshape(-1, 36)
    d = np.ascontiguousarray(b[:, 0:2]).view(np.float16).astype(np.float64)
    q = np.ascontiguousarray(b[:, 4:36]).view(np.int8).astype(np.float64)
    return (d * q).reshape(-1)


def _rows_dot(values: np.ndarray, x: np.ndarray) -> np.ndarray:
    return np.array([math.fsum(v * x) for v in values])


def test_q6k_matvec_through_gguf_weights_is_bit_exact():
    """Every product of a Q6_K weight (d * scale * (q - 32): <= 24 significant
    bits) and a Q8_1 value (<= 19 bits) is exact in fp64, so the correctly
    rounded row sum through gguf-py's weights equals the oracle's bit for bit."""
    rows, k = 48, 2560
    w = fx.seeded_q6k_matrix(rows, k, seed=11)
    act = oracle.quantize_q8_1(fx.seeded_activation(k, seed=12))
    vals = _gguf_values(w.reshape(-1, 210), QT.Q6_K).astype(np.float64).reshape(rows, k)
    ref = _rows_dot(vals, _q8_values(act))
    assert np.array_equal(oracle.q6k_matvec(w, act, rows, k), ref)


# ------------------------------------------------------------ Q4_K / Q5_K

def _k_blocks(size: int, n: int, seed: int) -> np.ndarray:
    """Seeded blocks with 6-bit scale/min edge patterns (all 0, all 63, mixed)."""
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (n, size), dtype=np.uint8)
    b[0, 4:16] = 0x00
    b[1, 4:16] = 0xFF
    b[2, 4:16] = np.array([0x3F, 0x00, 0xC0, 0x3F, 0xFF, 0x00, 0x80, 0x40, 0x0F, 0xF0, 0xAA, 0x55], dtype=np.uint8)
    b[3, size - 128:] = 0xFF      # nibbles all 15 (and, for Q5_K, the fifth bits below)
    b[4, size - 128:] = 0x00
    if size == 176:
        b[3, 16:48] = 0xFF
        b[4, 16:48] = 0x00
    return b


@pytest.mark.parametrize("size,qtype,decode", [(144, QT.Q4_K, oracle.decode_block),
                                               (176, QT.Q5_K, oracle.q5k_decode_block)])
@pytest.mark.parametrize("mode", ["scales", "mins"])
def test_k_quant_index_map_exact(size, qtype, decode, mode):
    """d = 1, dmin = 0 isolates sc * q; d = 0, dmin = 1 isolates -m."""
    b = _k_blocks(size, 256, seed=3 if mode == "scales" else 4)
    zero = np.zeros(2, dtype=np.uint8)
    b[:, 0:2], b[:, 2:4] = (F16_ONE, zero) if mode == "scales" else (zero, F16_ONE)
    got = _oracle_values(b, decode)
    ref = _gguf_values(b, qtype).astype(np.float64)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("kind", ["q4k", "q5k"])
def test_k_quant_seeded_values_and_matvec(kind):
    rows, k = 32, 2560
    size, qtype, decode, make, matvec = {
        "q4k": (144, QT.Q4_K, oracle.decode_block, fx.seeded_q4k_matrix, oracle.q4k_matvec),
        "q5k": (176, QT.Q5_K, oracle.q5k_decode_block, fx.seeded_q5k_matrix, oracle.q5k_matvec)}[kind]
    w = make(rows, k, seed=21)
    got = _oracle_values(w.reshape(-1, size), decode)
    ref = _gguf_values(w.reshape(-1, size), qtype).astype(np.float64)
    # gguf-py forms d*sc*q - dmin*m in fp32: one value may round once.
    assert np.all(np.abs(got - ref) <= 2.0 ** -23 * np.maximum(np.abs(got), 1e-30) + 1e-12)
    act = oracle.quantize_q8_1(fx.seeded_activation(k, seed=22))
    exact = _rows_dot(got.reshape(rows, k), _q8_values(act))
    assert np.array_equal(matvec(w, act, rows, k), exact)
    via_gguf = _rows_dot(ref.reshape(rows, k), _q8_values(act))
    assert np.all(np.abs(via_gguf - exact) <= 1e-5 + 1e-5 * np.abs(exact))


# ------------------------------------------------------------------ Q4_0

def _q4_0_inputs() -> np.ndarray:
    rng = np.random.default_rng(5)
    x = rng.standard_normal((96, 32)).astype(np.float32)
    x[0] = 0.0                                     # amax = 0: d = 0, all quants 8
    x[1] = np.linspace(-8, 7, 32, dtype=np.float32)   # exact grid, max at a negative value
    x[2] = -x[1]                                   # max at a positive value: q clamps at 15
    x[3, :] = 1.0
    x[3, 0] = -8.0                                 # the value -8 maps to 0, +1 to 7 (tie at 7.5 + 0.5)
    x[4] = np.float32(1e-30) * rng.standard_normal(32).astype(np.float32)  # tiny: d near fp16 underflow
    x[5] = np.float32(6e4) * np.sign(rng.standard_normal(32)).astype(np.float32)  # large: d = 7500
    # ties of x / d + 8.5 at integer boundaries: values k * d / 2 for odd k
    d = np.float32(-0.25)
    x[6] = np.float32(2.0)                         # amax first, negative sign -> d = -2 / 8
    x[6, 0] = np.float32(-2.0)
    x[6, 1:] = (np.arange(1, 32, dtype=np.float32) % 15 - 7) * np.float32(0.5) * -d
    x[7] = np.float32(3.0) * rng.integers(-2, 3, 32).astype(np.float32)
    return x


def test_q4_0_quantiser_bytes_match_gguf():
    x = _q4_0_inputs()
    got = oracle.quantize_q4_0(x.reshape(-1))
    ref = gq.quantize(x, QT.Q4_0).reshape(-1)
    assert np.array_equal(got, ref)


def test_q4_0_decode_matches_gguf():
    blocks = gq.quantize(_q4_0_inputs(), QT.Q4_0)
    got = oracle.dequantize_q4_0(blocks.reshape(-1))
    ref = gq.dequantize(blocks.reshape(-1), QT.Q4_0).astype(np.float64)
    assert np.array_equal(got.astype(np.float32).astype(np.float64), ref)


def test_q4_0_kv_planes_match_gguf_blocks():
    """The cache's split planes (nibbles, fp16 scales) hold GGML's 18-byte blocks."""
    rows = np.random.default_rng(9).standard_normal((6, 128)).astype(np.float32)
    qs, d = oracle.kv_q4_0_rows(rows)
    blocks = gq.quantize(rows.reshape(-1, 32), QT.Q4_0).reshape(6, 4, 18)
    assert np.array_equal(d, np.ascontiguousarray(blocks[:, :, :2]).view(np.uint16).reshape(6, 4))
    assert np.array_equal(qs, blocks[:, :, 2:].reshape(6, 64))


# ------------------------------------------------------------------ GGUF

def _tensors():
    rng = np.random.default_rng(31)
    return [("blk.0.ffn_gate.weight", QT.Q4_K, 3, 2560, fx.seeded_q4k_matrix(3, 2560, seed=1)),
            ("blk.0.ffn_down.weight", QT.Q5_K, 2, 512, fx.seeded_q5k_matrix(2, 512, seed=2)),
            ("output.weight", QT.Q6_K, 4, 512, fx.seeded_q6k_matrix(4, 512, seed=3)),
            ("blk.0.attn_norm.weight", QT.F32, 1, 96, rng.standard_normal(96).astype(np.float32).view(np.uint8))]


def test_gguf_writer_file_loads_through_our_reader(tmp_path):
    path = tmp_path / "w.gguf"
    w = gguf.GGUFWriter(str(path), arch="qwen3")
    w.add_block_count(36)
    w.add_uint32("x.u32", 7)
    w.add_string("x.s", "tokenizer ü")
    w.add_float32("x.f", 0.5)
    w.add_bool("x.b", True)
    for name, qt, rows, k, data in _tensors():
        if qt == QT.F32:
            w.add_tensor(name, data.view(np.float32))
        else:
            w.add_tensor(name, data.reshape(rows, -1), raw_dtype=qt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    g = ours.GgufFile(path)
    assert g.metadata["general.architecture"] == "qwen3" and g.metadata["qwen3.block_count"] == 36
    assert g.metadata["x.u32"] == 7 and g.metadata["x.s"] == "tokenizer ü"
    assert g.metadata["x.f"] == 0.5 and g.metadata["x.b"] is True
    for name, qt, rows, k, data in _tensors():
        t = g.tensors[name]
        assert t.ggml_type == int(qt)
        assert t.dims == ((k, rows) if rows > 1 else (k,))
        assert np.array_equal(g.raw(name), data)


def test_our_writer_file_loads_through_gguf_reader(tmp_path):
    path = tmp_path / "o.gguf"
    meta = {"general.architecture": "qwen3", "qwen3.block_count": np.uint32(36), "x.i64": -5,
            "x.name": "tokenizer ü", "x.arr": np.arange(7, dtype=np.int32)}
    ours.write_gguf(path, meta, [(name, int(qt), (k, rows) if rows > 1 else (k,), data.tobytes())
                                 for name, qt, rows, k, data in _tensors()], alignment=64)
    r = gguf.GGUFReader(str(path))
    fields = r.fields
    assert int(fields["qwen3.block_count"].contents()) == 36
    assert int(fields["x.i64"].contents()) == -5
    assert fields["x.name"].contents() == "tokenizer ü"
    assert list(fields["x.arr"].contents()) == list(range(7))
    by_name = {t.name: t for t in r.tensors}
    for name, qt, rows, k, data in _tensors():
        t = by_name[name]
        assert t.tensor_type == qt
        assert list(t.shape) == ([k, rows] if rows > 1 else [k])
        assert np.array_equal(np.asarray(t.data).reshape(-1).view(np.uint8), data)
