"""Synthetic inputs in the reference's binary fixture layouts.

Two families:

1. Reference-compatible fixtures.  Byte-identical to what the reference's
   generators write, so a harness built for the reference reads them
   unchanged and the reference's own SHA-256 pins apply:
   * IMROPE inputs ('<4224f4i', 16,912 bytes): tools/generate_fixtures.py:10-46
   * Q4_K matvec / gate-up inputs (weights.bin, gate.bin, activations.bin):
     tools/generate_q4_matvec_fixtures.py:16-84
   The random draws happen in the same order as there (Python's Mersenne
   Twister seeded 42 / 12345 / 54321 / per-variation seeds) because the byte
   layout and the pinned hashes require it.

2. Seeded distributions of the benchmark configurations (numpy PCG64):
   Q4_K with fp16 d ~ U(1e-3, 1e-2), dmin ~ U(0, 5e-3), 6-bit scales/mins and
   nibbles uniform; Q6_K with d ~ U(1e-3, 1e-2), int8 scales ~ U{-32..31},
   uniform ql/qh; activations x ~ N(0, 1); IMROPE q ~ N(0, 1),
   gamma ~ U(0.5, 1.5).
"""
from __future__ import annotations

import hashlib
import json
import math
import random
import struct
from pathlib import Path

import numpy as np

from . import formats as F

# ===================================================================== IMROPE

IMROPE_CASES = {
    "distinct_axes": (3, 5, 11, 17),
    "long_position": (32768, 32768, 32768, 32768),
    "fallback_only": (0, 0, 0, 32768),
}

# Position fixtures of the benchmark configuration (distinct axes, all axes
# at 32768, fourth-axis fallback).
SEEDED_IMROPE_CASES = {
    "distinct_axes": (7, 13, 29, 0),
    "long_position": (32768, 32768, 32768, 32768),
    "fallback_only": (0, 0, 0, 32768),
}


def imrope_reference_inputs(positions):
    """The reference's deterministic Q / gamma pattern (tools/generate_fixtures.py:18-22)."""
    gamma = [1 + i / 128 for i in range(F.HEAD_DIM)]
    q = [[(-1 if (i + h) % 2 else 1) * (1 + ((i + 3 * h) % 8) / 8) * (1 + h / 8)
          for i in range(F.HEAD_DIM)] for h in range(F.HEADS)]
    return {"q": q, "gamma": gamma, "positions_axis_major": list(positions)}


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
        raise ValueError("Expected Q[32,128], gamma[128], positions[4]")
    values = [v for row in q for v in row] + gamma
    if not all(math.isfinite(v) for v in values):
        raise ValueError("Nonfinite fixture input")
    return struct.pack("<4224f4i", *values, *positions)


def parse_imrope(payload: bytes):
    if len(payload) != F.IMROPE_FIXTURE_BYTES:
        raise ValueError("IMROPE fixture must be 16,912 bytes")
    q = np.frombuffer(payload, dtype="<f4", count=4096).reshape(F.HEADS, F.HEAD_DIM).copy()
    gamma = np.frombuffer(payload, dtype="<f4", count=128, offset=4096 * 4).copy()
    positions = np.frombuffer(payload, dtype="<i4", count=4, offset=4224 * 4).copy()
    return q, gamma, positions


def write_imrope_fixtures(output_dir) -> dict:
    """Same files and manifest as tools/generate_fixtures.py:write_fixtures."""
    output_dir = Path(output_dir)
    output_dir.mkdir(parents=True, exist_ok=True)
    manifest = {}
    for name, positions in IMROPE_CASES.items():
        payload = serialize_imrope(imrope_reference_inputs(positions))
        filename = name + ".input.bin"
        (output_dir / filename).write_bytes(payload)
        manifest[name] = {"filename": filename, "bytes": len(payload),
                          "sha256": hashlib.sha256(payload).hexdigest()}
    (output_dir / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


# ===================================================================== Q4 matvec

# Per-row gate factor cycle of the reference's gate fixture: covers zero,
# small, negative and large SwiGLU inputs.
_GATE_FACTORS = (0, 1, -1, 1 / 16, -1 / 16, 8, -8, 1)
# The fixed nibble pattern of a reference Q4_K block.
DEMO_QUANTS = bytes((i % 16) | (((15 - i) % 16) << 4) for i in range(128))


def _draw_six_bit_block(rng: random.Random, d: float, dmin: float) -> bytes:
    scales = [rng.randrange(64) for _ in range(8)]
    minima = [rng.randrange(64) for _ in range(8)]
    return F.q4k_block(scales, minima, d, dmin, DEMO_QUANTS)


def vary_factors(payload: bytes, seed: int) -> bytes:
    """Scale each block's fp16 d and dmin by U(0.75, 1.25) (re-rounded to fp16)."""
    if not payload or len(payload) % F.Q4K_BLOCK_BYTES:
        raise ValueError("Require whole Q4_K blocks")
    rng = random.Random(seed)
    result = bytearray(payload)
    for offset in range(0, len(payload), F.Q4K_BLOCK_BYTES):
        factors = struct.unpack_from("<ee", payload, offset)
        if not all(math.isfinite(v) for v in factors):
            raise ValueError("Require finite Q4_K factors")
        scaled = [v * rng.uniform(0.75, 1.25) for v in factors]
        struct.pack_into("<ee", result, offset, *scaled)
    return bytes(result)


def vary_activation_scales(payload: bytes, seed: int) -> bytes:
    """Scale each Q8_1 block's d by 2**U{-3..3}; s is regenerated as d * sum(q)."""
    if not payload or len(payload) % F.Q8_1_BLOCK_BYTES:
        raise ValueError("Require whole Q8_1 blocks")
    rng = random.Random(seed)
    out = bytearray()
    for offset in range(0, len(payload), F.Q8_1_BLOCK_BYTES):
        delta, _, *values = struct.unpack_from("<ee32b", payload, offset)
        if not math.isfinite(delta) or delta <= 0 or max(map(abs, values)) != 127:
            raise ValueError("Require positive finite scale and matching quantization range")
        delta *= 2 ** rng.randrange(-3, 4)
        out.extend(F.q8_1_block(delta, delta * sum(values), values))
    return bytes(out)


def q4_matvec_fixtures(random_quants=False, gate_up=False, rows=64, factor_seed=None,
                       activation_scale_seed=None, input_width=2560) -> dict:
    """weights.bin / activations.bin (/ gate.bin) exactly as the reference writes them."""
    if rows < 64 or rows > 9728 or rows % 64:
        raise ValueError("rows must be a multiple of 64 between 64 and 9728")
    if input_width not in (2048, 2560):
        raise ValueError("input_width must be 2048 or 2560")
    blocks = input_width // F.QK_K
    base_blocks = 64 * blocks
    rng = random.Random(42)
    weights = [_draw_six_bit_block(rng, 1 / 512, 1 / 1024) for _ in range(base_blocks)]
    activations = []
    for _ in range(input_width // F.Q8_1_GROUP):
        values = [rng.randrange(-127, 128) for _ in range(32)]
        values[0] = 127
        activations.append(F.q8_1_block(1 / 128, sum(values) / 128, values))
    weights += [_draw_six_bit_block(rng, 1 / 512, 1 / 1024) for _ in range((rows - 64) * blocks)]

    def fresh_quants(stream: random.Random, index: int) -> bytes:
        # The first 64 rows draw byte by byte, the extension rows in one call.
        if index < base_blocks:
            return bytes(stream.randrange(256) for _ in range(128))
        return stream.randbytes(128)

    if random_quants:
        quant_rng = random.Random(12345)
        weights = [blk[:16] + fresh_quants(quant_rng, i) for i, blk in enumerate(weights)]
    result = {"weights.bin": b"".join(weights), "activations.bin": b"".join(activations)}
    if gate_up:
        gate_rng = random.Random(54321)
        gate = []
        for i, blk in enumerate(weights):
            factor = _GATE_FACTORS[(i // blocks) % 8]
            gate.append(struct.pack("<ee", factor / 8192, factor / 16384) + blk[4:16]
                        + fresh_quants(gate_rng, i))
        result["gate.bin"] = b"".join(gate)
    if factor_seed is not None:
        result["weights.bin"] = vary_factors(result["weights.bin"], factor_seed)
        if gate_up:
            result["gate.bin"] = vary_factors(result["gate.bin"], factor_seed + 1)
    if activation_scale_seed is not None:
        result["activations.bin"] = vary_activation_scales(result["activations.bin"],
                                                           activation_scale_seed)
    return result


def write_q4_matvec_fixtures(directory, **options) -> dict:
    """Same files and fixtures.json as tools/generate_q4_matvec_fixtures.py:main."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    manifest = {"activation_scale_seed": options.get("activation_scale_seed"),
                "factor_seed": options.get("factor_seed"), "rows": options.get("rows", 64),
                "input_width": options.get("input_width", 2560), "seed": 42,
                "random_quants": options.get("random_quants", False),
                "gate_up": options.get("gate_up", False),
                "gate_seed": 54321 if options.get("gate_up") else None,
                "quant_seed": 12345 if options.get("random_quants") else None, "files": {}}
    for name, payload in q4_matvec_fixtures(**options).items():
        (directory / name).write_bytes(payload)
        manifest["files"][name] = {"bytes": len(payload), "sha256": hashlib.sha256(payload).hexdigest()}
    (directory / "fixtures.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


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
