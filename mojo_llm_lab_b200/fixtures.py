"""Synthetic inputs of the benchmark configurations, in the reference's binary
layouts.

* Layouts: the IMROPE input file ('<4224f4i', 16,912 bytes: head-major
  Q[32,128], gamma[128], int32 positions[4]; tools/generate_fixtures.py:32)
  and weight files repeated to more rows (benchmark/q4_compare.c:148-163).
* Seeded distributions (numpy PCG64): Q4_K / Q5_K with fp16 d ~ U(1e-3, 1e-2),
  dmin ~ U(0, 5e-3), 6-bit scales/mins and nibbles uniform; Q6_K with
  d ~ U(1e-3, 1e-2), int8 scales ~ U{-32..31}, uniform ql/qh; activations
  x ~ N(0, 1); IMROPE q ~ N(0, 1), gamma ~ U(0.5, 1.5).

The byte-identical reproduction of the reference's own fixture generators
(its Mersenne Twister draw order, for the reference's SHA-256 pins) is test
infrastructure and lives in tests/ref_fixtures.py.
"""
from __future__ import annotations

import math
import struct

import numpy as np

from . import formats as F

# ===================================================================== IMROPE

SEEDED_IMROPE_CASES = {
    "distinct_axes": (7, 13, 29, 0),
    "long_position": (32768, 32768, 32768, 32768),
    "fallback_only": (0, 0, 0, 32768),
}


def imrope_seeded_inputs(positions, seed: int = 0, heads: int = F.HEADS):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((heads, F.HEAD_DIM), dtype=np.float32)
    gamma = rng.uniform(0.5, 1.5, F.HEAD_DIM).astype(np.float32)
    return {"q": q, "gamma": gamma, "positions_axis_major": list(positions)}


def serialize_imrope(fixture) -> bytes:
    """'<4224f4i': head-major Q[32,128], gamma[128], int32 positions[4]."""
    q, gamma, positions = (fixture[k] for k in ("q", "gamma", "positions_axis_major"))
    q = [list(map(float, row)) for row in q]
    gamma = list(map(float, gamma))
    if (len(q) != F.HEADS or any(len(row) != F.HEAD_DIM for row in q)
            or len(gamma) != F.HEAD_DIM or len(positions) != 4):
        raise ValueError("an IMROPE input holds q[32][128], gamma[128] and 4 positions")
    values = [v for row in q for v in row] + gamma
    if not all(math.isfinite(v) for v in values):
        raise ValueError("IMROPE inputs must all be finite")
    return struct.pack("<4224f4i", *values, *positions)


def parse_imrope(payload: bytes):
    if len(payload) != F.IMROPE_FIXTURE_BYTES:
        raise ValueError("IMROPE fixture must be 16,912 bytes")
    q = np.frombuffer(payload, dtype="<f4", count=4096).reshape(F.HEADS, F.HEAD_DIM).copy()
    gamma = np.frombuffer(payload, dtype="<f4", count=128, offset=4096 * 4).copy()
    positions = np.frombuffer(payload, dtype="<i4", count=4, offset=4224 * 4).copy()
    return q, gamma, positions


def tile_rows(payload: bytes, row_bytes: int, rows: int) -> bytes:
    """Repeat a 64-row weight file up to `rows` rows, as benchmark/q4_compare.c:148-163 does."""
    src_rows = len(payload) // row_bytes
    if src_rows * row_bytes != len(payload) or rows % src_rows:
        raise ValueError("rows must be a multiple of the source rows")
    return payload * (rows // src_rows)


# ===================================================================== seeded

def seeded_q4k_matrix(rows: int, k: int, seed: int) -> np.ndarray:
    """rows x (k/256) Q4_K blocks: d ~ U(1e-3,1e-2), dmin ~ U(0,5e-3), uniform 6-bit
    scales/mins and nibbles.  Returns a flat uint8 array."""
    nb = rows * (k // F.QK_K)
    rng = np.random.default_rng(seed)
    d = F.f16_bits(rng.uniform(1e-3, 1e-2, nb))
    dmin = F.f16_bits(rng.uniform(0.0, 5e-3, nb))
    scales = rng.integers(0, 64, (nb, 8), dtype=np.uint8)
    minima = rng.integers(0, 64, (nb, 8), dtype=np.uint8)
    quants = rng.integers(0, 256, (nb, 128), dtype=np.uint8)
    out = np.empty((nb, F.Q4K_BLOCK_BYTES), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = F.pack_q4k_scale_array(scales, minima)
    out[:, 16:] = quants
    return out.reshape(-1)


def seeded_q5k_matrix(rows: int, k: int, seed: int) -> np.ndarray:
    """rows x (k/256) Q5_K blocks with Q4_K's distributions (d ~ U(1e-3,1e-2),
    dmin ~ U(0,5e-3), uniform 6-bit scales/mins) and uniform qh / qs bytes."""
    nb = rows * (k // F.QK_K)
    rng = np.random.default_rng(seed)
    d = F.f16_bits(rng.uniform(1e-3, 1e-2, nb))
    dmin = F.f16_bits(rng.uniform(0.0, 5e-3, nb))
    scales = rng.integers(0, 64, (nb, 8), dtype=np.uint8)
    minima = rng.integers(0, 64, (nb, 8), dtype=np.uint8)
    out = np.empty((nb, F.Q5K_BLOCK_BYTES), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = F.pack_q4k_scale_array(scales, minima)
    out[:, 16:] = rng.integers(0, 256, (nb, 160), dtype=np.uint8)
    return out.reshape(-1)


def seeded_q6k_matrix(rows: int, k: int, seed: int) -> np.ndarray:
    """rows x (k/256) Q6_K blocks: d ~ U(1e-3,1e-2), int8 scales ~ U{-32..31},
    uniform ql/qh bytes.  Returns a flat uint8 array."""
    nb = rows * (k // F.QK_K)
    rng = np.random.default_rng(seed)
    d = F.f16_bits(rng.uniform(1e-3, 1e-2, nb))
    scales = rng.integers(-32, 32, (nb, 16), dtype=np.int8)
    bits = rng.integers(0, 256, (nb, 192), dtype=np.uint8)
    out = np.empty((nb, F.Q6K_BLOCK_BYTES), dtype=np.uint8)
    out[:, 0:192] = bits
    out[:, 192:208] = scales.view(np.uint8)
    out[:, 208:210] = d.view(np.uint8).reshape(nb, 2)
    return out.reshape(-1)


def seeded_activation(k: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal(k, dtype=np.float32)
