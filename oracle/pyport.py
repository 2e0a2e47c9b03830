"""Pure-Python restatement of the reference's Python oracles -- TEST
INFRASTRUCTURE ONLY (the single-thread Python CPU baseline of bench.py and
its CPU test; never part of the product).

The reference's CPU path for the matvec and IMROPE is plain Python over byte
strings.  Its checkout does not travel to the GPU host, so this module
restates the same arithmetic, in the same floating-point order, to time that
path on the GPU host's cores:

* ``dot_q4_q8``       tests/q4_reference.py:36-47 (weights from
                      decode_block :6-24, activations from decode_q8_1
                      :27-33; one float64 product per element, math.fsum)
* ``reference_head``  tests/reference_math.py:22-35 (float64 RMSNorm, gamma,
                      exact theta scale 5e6^(-2/128), split-half rotation)

Results are bit-identical to the reference's functions (checked against the
golden vectors in tests/test_oracle_golden.py).
"""
from __future__ import annotations

import math
import struct

_HEAD_DIM = 128
_PAIRS = _HEAD_DIM // 2


def _scale_min(packed: bytes, group: int) -> tuple[int, int]:
    """6-bit (scale, min) of sub-block `group` from the 12 packed bytes."""
    if group < 4:
        return packed[group] & 0x3F, packed[group + 4] & 0x3F
    lo, hi_s, hi_m = packed[group + 4], packed[group - 4] >> 6, packed[group] >> 6
    return (lo & 0x0F) | (hi_s << 4), (lo >> 4) | (hi_m << 4)


def _block_values(block: bytes) -> list[float]:
    d, dmin = struct.unpack_from("<ee", block)
    packed = block[4:16]
    out = []
    for group in range(8):
        sc, mn = _scale_min(packed, group)
        ds, dm = d * sc, dmin * mn
        shift = 4 * (group & 1)
        base = 16 + (group >> 1) * 32
        out.extend(ds * ((block[base + i] >> shift) & 0x0F) - dm for i in range(32))
    return out


def _q8_values(block: bytes) -> list[float]:
    delta = struct.unpack_from("<e", block)[0]
    return [delta * q for q in struct.unpack_from("<32b", block, 4)]


def dot_q4_q8(weights: bytes, activations: bytes) -> float:
    nb = len(weights) // 144
    if not weights or len(weights) % 144 or len(activations) != nb * 288:
        raise ValueError("weights must be whole Q4_K blocks with 8 Q8_1 blocks each")
    terms = []
    for b in range(nb):
        w = _block_values(weights[b * 144:(b + 1) * 144])
        a = []
        for g in range(8):
            off = (b * 8 + g) * 36
            a.extend(_q8_values(activations[off:off + 36]))
        terms.extend(map(float.__mul__, w, a))
    return math.fsum(terms)


def _axis(pair: int) -> int:
    """IMROPE sections (24, 20, 20, 0): pairs cycle t, h, w inside their section."""
    r = pair % 64
    if r % 3 == 1 and r < 60:
        return 1
    if r % 3 == 2 and r < 60:
        return 2
    if r % 3 == 0 and r < 72:
        return 0
    return 3


def reference_head(q, gamma, positions) -> list[float]:
    if len(q) != _HEAD_DIM or len(gamma) != _HEAD_DIM or len(positions) != 4:
        raise ValueError("one head: q[128], gamma[128], positions[4]")
    r = 1.0 / math.sqrt(sum(v * v for v in q) / _HEAD_DIM + 1e-6)
    y = [q[i] * r * gamma[i] for i in range(_HEAD_DIM)]
    step = 5_000_000.0 ** (-2.0 / _HEAD_DIM)
    out = [0.0] * _HEAD_DIM
    for p in range(_PAIRS):
        ang = positions[_axis(p)] * (step ** p)
        c, s = math.cos(ang), math.sin(ang)
        a, b = y[p], y[p + _PAIRS]
        out[p] = a * c - b * s
        out[p + _PAIRS] = a * s + b * c
    return out
