"""Binary block formats of the decode hot path (GGML layouts, byte-exact).

Q4_K super-block, 144 bytes per 256 weights (tests/q4_reference.py:6-24 of the
reference; GGML block_q4_K):
    [0:2]   fp16 d        [2:4] fp16 dmin
    [4:16]  12 bytes of packed 6-bit sub-block scales and mins
    [16:144] 128 bytes of 4-bit quants; group g of 32 weights uses the low
             (g even) or high (g odd) nibble of bytes 16 + (g // 2) * 32 + l.
    weight(g, l) = d * scale_g * q - dmin * min_g

Q8_1 activation block, 36 bytes per 32 values (tests/q4_reference.py:27-33):
    [0:2] fp16 d   [2:4] fp16 s   [4:36] 32 x int8 q;   value = d * q

Q6_K super-block, 210 bytes per 256 weights (public GGML block_q6_K):
    [0:128] ql low nibbles  [128:192] qh 2-bit pairs  [192:208] int8 scales
    [208:210] fp16 d;       weight = d * scale_j * (q6 - 32)

Everything here is plain numpy/struct on the host: encoders used by the
fixture generators and the byte sizes the C-ABI checks against.
"""
from __future__ import annotations

import struct

import numpy as np

QK_K = 256
Q4K_BLOCK_BYTES = 144
Q6K_BLOCK_BYTES = 210
Q5K_BLOCK_BYTES = 176
Q8_1_BLOCK_BYTES = 36
Q8_1_GROUP = 32

HEAD_DIM = 128
HEADS = 32
IMROPE_SECTIONS = (24, 20, 20, 0)
IMROPE_EPSILON = 1e-6
IMROPE_FREQ_BASE = 5_000_000.0
# The runtime fp32 theta scale the reference's harness writes to device
# memory (benchmark/bench.c:245): fp32 nearest to 5e6 ** (-2 / 128).
THETA_SCALE_BITS = 0x3F492C27
IMROPE_FIXTURE_BYTES = 16_912  # '<4224f4i': q[32*128], gamma[128], positions[4]


def q4k_row_bytes(k: int) -> int:
    if k <= 0 or k % QK_K:
        raise ValueError("Q4_K rows need a positive multiple of 256 weights")
    return k // QK_K * Q4K_BLOCK_BYTES


def q5k_row_bytes(k: int) -> int:
    if k <= 0 or k % QK_K:
        raise ValueError("Q5_K rows need a positive multiple of 256 weights")
    return k // QK_K * Q5K_BLOCK_BYTES


def q6k_row_bytes(k: int) -> int:
    if k <= 0 or k % QK_K:
        raise ValueError("Q6_K rows need a positive multiple of 256 weights")
    return k // QK_K * Q6K_BLOCK_BYTES


def q8_1_bytes(k: int) -> int:
    if k <= 0 or k % Q8_1_GROUP:
        raise ValueError("Q8_1 needs a positive multiple of 32 values")
    return k // Q8_1_GROUP * Q8_1_BLOCK_BYTES


def theta_scale_f32() -> float:
    return float(np.array([THETA_SCALE_BITS], dtype=np.uint32).view(np.float32)[0])


# ------------------------------------------------------------------ Q4_K packing

def pack_q4k_scale_bytes(scales, minima) -> bytes:
    """8 six-bit scales and 8 six-bit mins -> the 12 packed bytes of a Q4_K block.

    Groups 0-3 keep their low 6 bits in bytes 0-3 (scales) and 4-7 (mins);
    groups 4-7 split into a low nibble (bytes 8-11) and the two high bits of
    bytes 0-7.  This is the inverse of the decode rule of
    tests/q4_reference.py:57-62.
    """
    meta = bytearray(12)
    for j in range(4):
        meta[j] = (scales[j] & 63) | ((scales[j + 4] >> 4) << 6)
        meta[j + 4] = (minima[j] & 63) | ((minima[j + 4] >> 4) << 6)
        meta[j + 8] = (scales[j + 4] & 15) | ((minima[j + 4] & 15) << 4)
    return bytes(meta)


def pack_q4k_scale_array(scales: np.ndarray, minima: np.ndarray) -> np.ndarray:
    """Vectorised pack_q4k_scale_bytes over [blocks, 8] uint8 arrays -> [blocks, 12]."""
    sc = scales.astype(np.uint8)
    mn = minima.astype(np.uint8)
    meta = np.empty((sc.shape[0], 12), dtype=np.uint8)
    meta[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    meta[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    meta[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return meta


def q4k_block(scales, minima, d: float, dmin: float, quants: bytes) -> bytes:
    if len(quants) != 128:
        raise ValueError("Q4_K quants are 128 bytes")
    return struct.pack("<ee", d, dmin) + pack_q4k_scale_bytes(scales, minima) + bytes(quants)


def q8_1_block(d: float, s: float, quants) -> bytes:
    return struct.pack("<ee32b", d, s, *quants)


def f16_bits(values) -> np.ndarray:
    """float -> fp16 bit patterns (round to nearest even), as uint16."""
    return np.asarray(values, dtype=np.float64).astype(np.float16).view(np.uint16)


def unpack_q8_1(payload: bytes):
    """Q8_1 bytes -> (d fp16->float32 [G], s [G], q int8 [G, 32])."""
    a = np.frombuffer(payload, dtype=np.uint8).reshape(-1, Q8_1_BLOCK_BYTES)
    d = a[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
    s = a[:, 2:4].copy().view(np.float16).astype(np.float32).reshape(-1)
    q = a[:, 4:].view(np.int8)
    return d, s, q
