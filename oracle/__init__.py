"""CPU oracle for the decode hot path -- TEST INFRASTRUCTURE ONLY.

This package is the checker.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``) may import it;
the product package ``mojo_llm_lab_b200`` never does, and fails loudly when its
CUDA library is missing instead of falling back to anything here.

The arithmetic lives in ``oracle.c`` (a plain-C restatement of the reference's
Python oracles, bit-identical to them on the golden vectors in
``tests/golden/``); this module loads it with ctypes and exposes numpy-facing
wrappers whose names follow the reference:

* ``dot_q4_q8`` / ``q4k_matvec``      tests/q4_reference.py:36-47
* ``decode_block``                     tests/q4_reference.py:6-24
* ``decode_q8_1``                      tests/q4_reference.py:27-33
* ``reference_head`` / ``imrope``      tests/reference_math.py:22-35
* ``position_axis``                    tests/reference_math.py:11-19
* ``quantize_q8_1``                    GGML quantize_q8_1 semantics captured at
                                       benchmark/q4_compare.c:328-357
* ``q6k_matvec``                       public GGML Q6_K layout (the reference has
                                       no Q6_K oracle; pinned to llama.cpp's
                                       gguf-py 0.19.0 Q6_K.dequantize_blocks in
                                       tests/test_gguf_pin_cpu.py)
* ``q5k_matvec``                       public GGML Q5_K layout (no reference
                                       code; pinned to gguf-py Q5_K likewise)
* ``quantize_q4_0`` / ``kv_q4_0_rows`` GGML quantize_row_q4_0 for the Q4_0 KV
                                       cache the reference's contexts use
                                       (integration/resident_decode.cpp:70);
                                       pinned to gguf-py Q4_0.quantize_blocks
* ``pyport``                           pure-Python restatement of the reference's
                                       Python oracles, for the single-thread
                                       Python CPU baseline only
* ``attention`` / ``attention_q4_0``   float64 softmax attention over an fp16 or
                                       a Q4_0 cache
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

HEAD_DIM = 128
HEADS = 32
SECTIONS = (24, 20, 20, 0)
BASE = 5_000_000.0
EPSILON = 1e-6
THETA_SCALE_BITS = 0x3F492C27  # the runtime fp32 theta scale of benchmark/bench.c:245

S_D_TIMES_SUMQ = 0
S_SUM_X = 1

_lib = None


def build(force: bool = False) -> Path:
    """Compile oracle.c with its Makefile (gcc, OpenMP, -ffp-contract=off)."""
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
        env = dict(os.environ)
        env.pop("CC", None)
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True, env=env)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        handle = C.CDLL(str(LIB_PATH))
        P = C.c_void_p
        i64 = C.c_int64
        sigs = {
            "orc_half_to_double": (C.c_double, [C.c_uint16]),
            "orc_float_to_half": (C.c_uint16, [C.c_float]),
            "orc_fsum": (C.c_double, [P, i64]),
            "orc_q8_1_quantize": (C.c_int, [P, i64, P, C.c_int]),
            "orc_q8_1_decode": (None, [P, P]),
            "orc_q4k_decode_block": (None, [P, P]),
            "orc_q4k_subdots": (C.c_int, [P, P, i64, i64, P, P]),
            "orc_q4k_matvec": (C.c_int, [P, P, i64, i64, P, C.c_int]),
            "orc_q4k_gate_up": (C.c_int, [P, P, P, i64, i64, P, P, P, C.c_int]),
            "orc_swiglu": (C.c_double, [C.c_double, C.c_double]),
            "orc_q6k_decode_block": (None, [P, P]),
            "orc_q6k_matvec": (C.c_int, [P, P, i64, i64, P, C.c_int]),
            "orc_position_axis": (C.c_int, [C.c_int]),
            "orc_imrope": (C.c_int, [P, P, P, C.c_double, C.c_int, P]),
            "orc_reference_theta_scale": (C.c_double, []),
            "orc_rmsnorm": (C.c_int, [P, P, i64, C.c_double, P]),
            "orc_q5k_decode_block": (None, [P, P]),
            "orc_q5k_matvec": (C.c_int, [P, P, i64, i64, P, C.c_int]),
            "orc_embed_q6k": (C.c_int, [P, i64, i64, P]),
            "orc_rmsnorm_q8_1": (C.c_int, [P, P, i64, P, C.c_double, P, P]),
            "orc_qk_rope_append": (C.c_int, [P, C.c_int, C.c_int, P, P, C.c_int32, C.c_double, P, P, P, P]),
            "orc_attention": (C.c_int, [P, P, P, i64, i64, C.c_int, C.c_int, P, C.c_int]),
            "orc_q4_0_quantize": (C.c_int, [P, i64, P]),
            "orc_q4_0_decode": (None, [P, P]),
            "orc_attention_q4_0": (C.c_int, [P, P, P, P, i64, i64, C.c_int, C.c_int, P, C.c_int]),
            "orc_argmax": (i64, [P, i64]),
            "orc_version": (C.c_int, []),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _bytes(data) -> np.ndarray:
    if isinstance(data, np.ndarray):
        return np.ascontiguousarray(data.view(np.uint8).reshape(-1))
    return np.frombuffer(bytes(data), dtype=np.uint8)


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise ValueError(f"oracle {what} rejected its input (rc={rc})")


# ----------------------------------------------------------------- scalars

def half_to_double(bits: int) -> float:
    return lib().orc_half_to_double(bits)


def float_to_half(value: float) -> int:
    return lib().orc_float_to_half(value)


def fsum(values) -> float:
    v = np.ascontiguousarray(values, dtype=np.float64)
    return lib().orc_fsum(_ptr(v), v.size)


def position_axis(pair: int) -> int:
    return lib().orc_position_axis(pair)


def reference_theta_scale() -> float:
    return lib().orc_reference_theta_scale()


def runtime_theta_scale() -> float:
    return float(np.array([THETA_SCALE_BITS], dtype=np.uint32).view(np.float32)[0])


# ----------------------------------------------------------------- Q8_1

def quantize_q8_1(x, s_mode: int = S_D_TIMES_SUMQ) -> bytes:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if x.size == 0 or x.size % 32:
        raise ValueError("Q8_1 needs a multiple of 32 values")
    out = np.zeros(x.size // 32 * 36, dtype=np.uint8)
    _check(lib().orc_q8_1_quantize(_ptr(x), x.size, _ptr(out), s_mode), "quantize_q8_1")
    return out.tobytes()


def decode_q8_1(payload) -> list:
    p = _bytes(payload)
    if p.size != 36:
        raise ValueError("Q8_1 block must have exactly 36 bytes")
    out = np.zeros(32, dtype=np.float64)
    lib().orc_q8_1_decode(_ptr(p), _ptr(out))
    return out.tolist()


# ----------------------------------------------------------------- Q4_K

def decode_block(payload) -> list:
    p = _bytes(payload)
    if p.size != 144:
        raise ValueError("Q4_K block must have exactly 144 bytes")
    out = np.zeros(256, dtype=np.float64)
    lib().orc_q4k_decode_block(_ptr(p), _ptr(out))
    return out.tolist()


def q4k_matvec(weights, activations, rows: int, k: int, threads: int = 0) -> np.ndarray:
    w, a = _bytes(weights), _bytes(activations)
    if w.size != rows * (k // 256) * 144 or a.size != k // 32 * 36 or k % 256:
        raise ValueError("Mismatched Q4_K/Q8_1 block counts")
    out = np.zeros(rows, dtype=np.float64)
    _check(lib().orc_q4k_matvec(_ptr(w), _ptr(a), rows, k, _ptr(out), threads), "q4k_matvec")
    return out


def dot_q4_q8(weights, activations) -> float:
    """One-row dot product with the reference's signature (tests/q4_reference.py:36)."""
    w, a = _bytes(weights), _bytes(activations)
    if w.size == 0 or w.size % 144 or a.size != w.size // 144 * 288:
        raise ValueError("Mismatched Q4_K/Q8_1 block counts")
    return float(q4k_matvec(w, a, 1, w.size // 144 * 256)[0])


def q4k_subdots(weights, activations, rows: int, k: int):
    w, a = _bytes(weights), _bytes(activations)
    dots = np.zeros(rows * (k // 32), dtype=np.int32)
    sums = np.zeros(k // 32, dtype=np.int32)
    _check(lib().orc_q4k_subdots(_ptr(w), _ptr(a), rows, k, _ptr(dots), _ptr(sums)), "q4k_subdots")
    return dots.reshape(rows, k // 32), sums


def q4k_gate_up(up_weights, gate_weights, activations, rows: int, k: int, threads: int = 0):
    u, g, a = _bytes(up_weights), _bytes(gate_weights), _bytes(activations)
    up = np.zeros(rows, dtype=np.float64)
    gate = np.zeros(rows, dtype=np.float64)
    prod = np.zeros(rows, dtype=np.float64)
    _check(lib().orc_q4k_gate_up(_ptr(u), _ptr(g), _ptr(a), rows, k, _ptr(up), _ptr(gate), _ptr(prod),
                                 threads), "q4k_gate_up")
    return up, gate, prod


def swiglu(up: float, gate: float) -> float:
    return lib().orc_swiglu(up, gate)


# ----------------------------------------------------------------- Q5_K

def q5k_decode_block(payload) -> list:
    """Public GGML Q5_K layout (parity unpinned: the reference has no Q5_K code)."""
    p = _bytes(payload)
    if p.size != 176:
        raise ValueError("Q5_K block must have exactly 176 bytes")
    out = np.zeros(256, dtype=np.float64)
    lib().orc_q5k_decode_block(_ptr(p), _ptr(out))
    return out.tolist()


def q5k_matvec(weights, activations, rows: int, k: int, threads: int = 0) -> np.ndarray:
    w, a = _bytes(weights), _bytes(activations)
    if w.size != rows * (k // 256) * 176 or a.size != k // 32 * 36 or k % 256:
        raise ValueError("Mismatched Q5_K/Q8_1 block counts")
    out = np.zeros(rows, dtype=np.float64)
    _check(lib().orc_q5k_matvec(_ptr(w), _ptr(a), rows, k, _ptr(out), threads), "q5k_matvec")
    return out


# ----------------------------------------------------------------- Q6_K

def q6k_decode_block(payload) -> list:
    p = _bytes(payload)
    if p.size != 210:
        raise ValueError("Q6_K block must have exactly 210 bytes")
    out = np.zeros(256, dtype=np.float64)
    lib().orc_q6k_decode_block(_ptr(p), _ptr(out))
    return out.tolist()


def q6k_matvec(weights, activations, rows: int, k: int, threads: int = 0) -> np.ndarray:
    w, a = _bytes(weights), _bytes(activations)
    if w.size != rows * (k // 256) * 210 or a.size != k // 32 * 36 or k % 256:
        raise ValueError("Mismatched Q6_K/Q8_1 block counts")
    out = np.zeros(rows, dtype=np.float64)
    _check(lib().orc_q6k_matvec(_ptr(w), _ptr(a), rows, k, _ptr(out), threads), "q6k_matvec")
    return out


# ----------------------------------------------------------------- IMROPE

def imrope(q, gamma, positions, theta_scale: float) -> np.ndarray:
    """reference_head over every head of q[heads, 128] at the given theta scale."""
    q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1)
    gamma = np.ascontiguousarray(gamma, dtype=np.float32).reshape(-1)
    positions = np.ascontiguousarray(positions, dtype=np.int32).reshape(-1)
    if q.size % HEAD_DIM or q.size == 0 or gamma.size != HEAD_DIM or positions.size != 4:
        raise ValueError("wrong reference shape")
    heads = q.size // HEAD_DIM
    out = np.zeros(q.size, dtype=np.float64)
    _check(lib().orc_imrope(_ptr(q), _ptr(gamma), _ptr(positions), float(theta_scale), heads, _ptr(out)),
           "imrope")
    return out.reshape(heads, HEAD_DIM)


def reference_head(q, gamma, positions) -> list:
    """tests/reference_math.py:22 with the exact theta scale, one head."""
    if len(q) != HEAD_DIM or len(gamma) != HEAD_DIM or len(positions) != 4:
        raise ValueError("wrong reference shape")
    return imrope(q, gamma, positions, reference_theta_scale())[0].tolist()


def rmsnorm(x, gamma, eps: float = 1e-6) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    gamma = np.ascontiguousarray(gamma, dtype=np.float32).reshape(-1)
    out = np.zeros(x.size, dtype=np.float64)
    _check(lib().orc_rmsnorm(_ptr(x), _ptr(gamma), x.size, eps, _ptr(out)), "rmsnorm")
    return out


# ------------------------------------------------------------ decode step

def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).reshape(-1))


def embed_q6k(weights, k: int, token: int) -> np.ndarray:
    """Row ``token`` of a Q6_K matrix, dequantised to fp32."""
    w = _bytes(weights)
    out = np.empty(k, dtype=np.float32)
    _check(lib().orc_embed_q6k(_ptr(w), k, token, _ptr(out)), "embed_q6k")
    return out


def rmsnorm_q8_1(x, delta, gamma, eps: float = 1e-6):
    """(h, q8): h = x + delta in fp32, q8 = Q8_1(fp32(h * rsqrt(mean h^2 + eps) * gamma))."""
    x = _f32(x)
    g = _f32(gamma)
    d = None if delta is None else _f32(delta)
    h = np.empty_like(x)
    q8 = np.empty(x.size // 32 * 36, dtype=np.uint8)
    _check(lib().orc_rmsnorm_q8_1(_ptr(x), None if d is None else _ptr(d), x.size, _ptr(g), eps, _ptr(h), _ptr(q8)),
           "rmsnorm_q8_1")
    return h, q8


def qk_rope_append(qkv, q_heads: int, kv_heads: int, q_gamma, k_gamma, pos: int, theta_scale: float):
    """(q_out fp32, k_row fp16 bits, v_row fp16 bits) of one token's fused QKV output."""
    qkv = _f32(qkv)
    q_out = np.empty(q_heads * HEAD_DIM, dtype=np.float32)
    k_row = np.empty(kv_heads * HEAD_DIM, dtype=np.uint16)
    v_row = np.empty(kv_heads * HEAD_DIM, dtype=np.uint16)
    qg, kg = _f32(q_gamma), _f32(k_gamma)
    _check(lib().orc_qk_rope_append(_ptr(qkv), q_heads, kv_heads, _ptr(qg), _ptr(kg), pos, theta_scale,
                                    _ptr(q_out), _ptr(k_row), _ptr(v_row), None), "qk_rope_append")
    return q_out, k_row, v_row


def qk_rope_f32(qkv, q_heads: int, kv_heads: int, q_gamma, k_gamma, pos: int, theta_scale: float):
    """(q_out, k rows, v rows), all fp32: the values a Q4_0 cache append quantises."""
    qkv = _f32(qkv)
    q_out = np.empty(q_heads * HEAD_DIM, dtype=np.float32)
    k_f32 = np.empty(kv_heads * HEAD_DIM, dtype=np.float32)
    qg, kg = _f32(q_gamma), _f32(k_gamma)
    _check(lib().orc_qk_rope_append(_ptr(qkv), q_heads, kv_heads, _ptr(qg), _ptr(kg), pos, theta_scale,
                                    _ptr(q_out), None, None, _ptr(k_f32)), "qk_rope_f32")
    v = qkv[(q_heads + kv_heads) * HEAD_DIM:(q_heads + 2 * kv_heads) * HEAD_DIM].copy()
    return q_out, k_f32, v


def attention(q, k_cache: np.ndarray, v_cache: np.ndarray, n: int, q_heads: int, kv_heads: int,
              threads: int = 0) -> np.ndarray:
    """Grouped-query softmax attention over cache rows [0, n); caches fp16 bits [kv][ctx][128]."""
    q = _f32(q)
    assert k_cache.dtype == np.uint16 and v_cache.dtype == np.uint16
    assert k_cache.flags.c_contiguous and v_cache.flags.c_contiguous
    ctx = k_cache.shape[-2]
    out = np.empty(q_heads * HEAD_DIM, dtype=np.float32)
    _check(lib().orc_attention(_ptr(q), _ptr(k_cache), _ptr(v_cache), ctx, n, q_heads, kv_heads, _ptr(out),
                               threads), "attention")
    return out


Q4_0_BLOCK_BYTES = 18


def quantize_q4_0(x) -> np.ndarray:
    """GGML Q4_0 blocks (18 bytes per 32 values) of fp32 x."""
    x = _f32(x)
    out = np.empty(x.size // 32 * Q4_0_BLOCK_BYTES, dtype=np.uint8)
    _check(lib().orc_q4_0_quantize(_ptr(x), x.size, _ptr(out)), "q4_0_quantize")
    return out


def dequantize_q4_0(blocks: np.ndarray) -> np.ndarray:
    """float64 values of Q4_0 blocks."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, Q4_0_BLOCK_BYTES)
    out = np.empty(blocks.shape[0] * 32, dtype=np.float64)
    for i in range(blocks.shape[0]):
        lib().orc_q4_0_decode(_ptr(blocks[i]), _ptr(out[i * 32:]))
    return out


def kv_q4_0_rows(rows) -> tuple[np.ndarray, np.ndarray]:
    """Q4_0 cache planes of fp32 rows [..., 128]: (nibbles [..., 64] uint8,
    block scales [..., 4] fp16 bits), the split of GGML's 18-byte blocks."""
    lead = np.shape(rows)[:-1]
    assert np.shape(rows)[-1] == HEAD_DIM
    blocks = quantize_q4_0(rows).reshape(-1, 4, Q4_0_BLOCK_BYTES)
    d = np.ascontiguousarray(blocks[:, :, :2]).view(np.uint16).reshape(*lead, 4)
    qs = np.ascontiguousarray(blocks[:, :, 2:]).reshape(*lead, 64)
    return qs, d


def attention_q4_0(q, k_qs: np.ndarray, v_qs: np.ndarray, kv_d: np.ndarray, n: int, q_heads: int, kv_heads: int,
                   threads: int = 0) -> np.ndarray:
    """attention over the Q4_0 cache planes: k_qs / v_qs uint8 [kv][ctx][64],
    kv_d fp16 bits [kv][ctx][8] (K block scales, then V)."""
    q = _f32(q)
    assert k_qs.dtype == np.uint8 and v_qs.dtype == np.uint8 and kv_d.dtype == np.uint16
    for a in (k_qs, v_qs, kv_d):
        assert a.flags.c_contiguous
    ctx = k_qs.shape[-2]
    out = np.empty(q_heads * HEAD_DIM, dtype=np.float32)
    _check(lib().orc_attention_q4_0(_ptr(q), _ptr(k_qs), _ptr(v_qs), _ptr(kv_d), ctx, n, q_heads, kv_heads,
                                    _ptr(out), threads), "attention_q4_0")
    return out


def argmax(x) -> int:
    """Index of the first maximum."""
    x = _f32(x)
    return int(lib().orc_argmax(_ptr(x), x.size))
