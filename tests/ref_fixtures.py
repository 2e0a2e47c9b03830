"""The reference's own fixture generators, reproduced byte for byte (test
infrastructure: the parity tests and the driver-API compatibility tests use
them; nothing in mojo_llm_lab_b200/ does).

* IMROPE inputs ('<4224f4i', 16,912 bytes): tools/generate_fixtures.py:10-46
* Q4_K matvec / gate-up inputs (weights.bin, gate.bin, activations.bin):
  tools/generate_q4_matvec_fixtures.py:16-84

The random draws happen in the same order as there (Python's Mersenne Twister
seeded 42 / 12345 / 54321 / per-variation seeds) because the files' bytes,
and so the reference's SHA-256 pins (tests/test_fixtures.py:10-14,
tests/test_q4_matvec_fixtures.py:12-15), depend on that order.
"""
from __future__ import annotations

import hashlib
import json
import math
import random
import struct
from pathlib import Path

from mojo_llm_lab_b200 import formats as F
from mojo_llm_lab_b200.fixtures import serialize_imrope

IMROPE_CASES = {
    "distinct_axes": (3, 5, 11, 17),
    "long_position": (32768, 32768, 32768, 32768),
    "fallback_only": (0, 0, 0, 32768),
}

def imrope_reference_inputs(positions):
    """The reference's deterministic Q / gamma pattern (tools/generate_fixtures.py:18-22)."""
    gamma = [1 + i / 128 for i in range(F.HEAD_DIM)]
    q = [[(-1 if (i + h) % 2 else 1) * (1 + ((i + 3 * h) % 8) / 8) * (1 + h / 8)
          for i in range(F.HEAD_DIM)] for h in range(F.HEADS)]
    return {"q": q, "gamma": gamma, "positions_axis_major": list(positions)}


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
        raise ValueError("the payload must be whole 144-byte Q4_K blocks")
    rng = random.Random(seed)
    result = bytearray(payload)
    for offset in range(0, len(payload), F.Q4K_BLOCK_BYTES):
        factors = struct.unpack_from("<ee", payload, offset)
        if not all(math.isfinite(v) for v in factors):
            raise ValueError("a Q4_K block has a non-finite d or dmin")
        scaled = [v * rng.uniform(0.75, 1.25) for v in factors]
        struct.pack_into("<ee", result, offset, *scaled)
    return bytes(result)


def vary_activation_scales(payload: bytes, seed: int) -> bytes:
    """Scale each Q8_1 block's d by 2**U{-3..3}; s is regenerated as d * sum(q)."""
    if not payload or len(payload) % F.Q8_1_BLOCK_BYTES:
        raise ValueError("the payload must be whole 36-byte Q8_1 blocks")
    rng = random.Random(seed)
    out = bytearray()
    for offset in range(0, len(payload), F.Q8_1_BLOCK_BYTES):
        delta, _, *values = struct.unpack_from("<ee32b", payload, offset)
        if not math.isfinite(delta) or delta <= 0 or max(map(abs, values)) != 127:
            raise ValueError("each Q8_1 block needs a positive finite d and a quant of magnitude 127")
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
