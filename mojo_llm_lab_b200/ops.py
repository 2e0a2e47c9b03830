"""PyTorch-facing host API of the decode hot path.

Thin wrappers over the C ABI (include/mllb200.h): they validate tensors,
derive shapes from the byte layouts, pick the current CUDA stream and call the
library.  Function names and argument order follow the reference's kernel
entries, so code written against those reads the same:

    fused_q_imrope_runtime_fastpow(q, gamma, positions, output, theta_scale)
                                   kernels/fused_q_imrope_runtime_fastpow.mojo:8-14
    q4_k_q8_1_matvec(weights, activations, output)
                                   kernels/q4_k_q8_1_matvec_dp4a_128.mojo:8-13
    q4_k_q8_1_gate_order(weights, gate_weights, activations, output)
                                   kernels/q4_k_q8_1_gate_order.mojo:55-60
    quantize_q8_1(x, out)          GGML quantize_q8_1 (benchmark/q4_compare.c:328)
    q6_k_q8_1_matvec(weights, activations, output)    GGML mul_mat_vec_q<Q6_K>

Errors: ValueError for shapes/dtypes/alignment (the reference's oracles raise
ValueError for wrong layouts), MllbError for CUDA failures.  All tensors must
live on the same CUDA device; nothing here copies to or from the host.
"""
from __future__ import annotations

import torch

from . import formats as F
from ._lib import LAUNCH_CONST_AUX, LAUNCH_PDL, S_D_SUMQ, S_SUM_X, ActF32, check, device_error, lib  # noqa: F401

__all__ = [
    "quantize_q8_1", "q4_k_q8_1_matvec", "q4_k_q8_1_gate_order", "q4k_gate_up", "q6_k_q8_1_matvec",
    "fused_q_imrope_runtime_fastpow", "rmsnorm_imrope_q", "q4k_subdots", "stream_read", "device_error",
    "rmsnorm_q8_1", "decode_embed", "decode_final_norm", "decode_qk_rope_append", "decode_attention",
    "decode_attention_qkv", "kv_q4_0_store", "decode_attention_q4_0", "decode_attention_qkv_q4_0",
    "q4k_matvec_act", "q4k_gate_up_act", "q6k_matvec_act", "act_f32", "q5_k_q8_1_matvec", "q4k_matvec_norm",
    "q4k_matvec_norm_workspace",
    "argmax_key", "token_key", "key_token", "S_D_SUMQ", "S_SUM_X",
]


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _need(t: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _same_device(*ts: torch.Tensor) -> None:
    devs = {t.device for t in ts if t is not None}
    if len(devs) > 1:
        raise ValueError(f"tensors on different devices: {sorted(map(str, devs))}")


def _k_from_q8(act: torch.Tensor) -> int:
    n = act.numel()
    if n == 0 or n % F.Q8_1_BLOCK_BYTES:
        raise ValueError("Q8_1 activations must be whole 36-byte blocks")
    return n // F.Q8_1_BLOCK_BYTES * F.Q8_1_GROUP


def _rows(weights: torch.Tensor, row_bytes: int, what: str) -> int:
    n = weights.numel()
    if n == 0 or n % row_bytes:
        raise ValueError(f"Mismatched {what}/Q8_1 block counts")
    return n // row_bytes


# ------------------------------------------------------------------- Q8_1

def quantize_q8_1(x: torch.Tensor, out: torch.Tensor | None = None, s_mode: int = S_D_SUMQ) -> torch.Tensor:
    """fp32 x[k] -> Q8_1 bytes (uint8[k/32*36])."""
    _need(x, "x", torch.float32)
    k = x.numel()
    if k == 0 or k % F.Q8_1_GROUP:
        raise ValueError("Q8_1 needs a positive multiple of 32 values")
    if out is None:
        out = torch.empty(k // 32 * 36, dtype=torch.uint8, device=x.device)
    _need(out, "out", torch.uint8)
    if out.numel() != k // 32 * 36:
        raise ValueError("out has the wrong size")
    _same_device(x, out)
    check(lib().mllb_q8_1_quantize(x.data_ptr(), out.data_ptr(), k, s_mode, _stream(x)), "quantize_q8_1")
    return out


# ------------------------------------------------------------------- Q4_K

def q4_k_q8_1_matvec(weights: torch.Tensor, activations: torch.Tensor,
                     output: torch.Tensor | None = None, pdl: bool = False) -> torch.Tensor:
    """out = W @ a.  pdl=True: programmatic dependent launch (MLLB_LAUNCH_PDL) --
    only when no preceding kernel in the stream writes `weights`."""
    _need(weights, "weights", torch.uint8)
    _need(activations, "activations", torch.uint8)
    k = _k_from_q8(activations)
    rows = _rows(weights, F.q4k_row_bytes(k), "Q4_K")
    if output is None:
        output = torch.empty(rows, dtype=torch.float32, device=weights.device)
    _need(output, "output", torch.float32)
    if output.numel() != rows:
        raise ValueError("output has the wrong size")
    _same_device(weights, activations, output)
    check(lib().mllb_q4k_matvec_ex(weights.data_ptr(), activations.data_ptr(), output.data_ptr(), rows, k,
                                   LAUNCH_PDL if pdl else 0, _stream(weights)), "q4_k_q8_1_matvec")
    return output


def q4k_gate_up(up_weights: torch.Tensor, gate_weights: torch.Tensor, activations: torch.Tensor,
                up: torch.Tensor | None = None, gate: torch.Tensor | None = None,
                prod: torch.Tensor | None = None, want=("up", "gate", "prod"), pdl: bool = False):
    """Fused gate/up: returns (up, gate, prod) with prod = up * silu(gate)."""
    _need(up_weights, "up_weights", torch.uint8)
    _need(gate_weights, "gate_weights", torch.uint8)
    _need(activations, "activations", torch.uint8)
    k = _k_from_q8(activations)
    rows = _rows(up_weights, F.q4k_row_bytes(k), "Q4_K")
    if gate_weights.numel() != up_weights.numel():
        raise ValueError("up and gate matrices differ in size")
    dev = up_weights.device
    outs = {"up": up, "gate": gate, "prod": prod}
    for name in ("up", "gate", "prod"):
        if outs[name] is None and name in want:
            outs[name] = torch.empty(rows, dtype=torch.float32, device=dev)
        if outs[name] is not None:
            _need(outs[name], name, torch.float32)
            if outs[name].numel() != rows:
                raise ValueError(f"{name} has the wrong size")
    _same_device(up_weights, gate_weights, activations, *outs.values())
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    check(lib().mllb_q4k_gate_up_ex(up_weights.data_ptr(), gate_weights.data_ptr(), activations.data_ptr(),
                                    ptr(outs["up"]), ptr(outs["gate"]), ptr(outs["prod"]), rows, k,
                                    LAUNCH_PDL if pdl else 0, _stream(up_weights)), "q4k_gate_up")
    return outs["up"], outs["gate"], outs["prod"]


def q4_k_q8_1_gate_order(weights: torch.Tensor, gate_weights: torch.Tensor, activations: torch.Tensor,
                         output: torch.Tensor | None = None) -> torch.Tensor:
    """The reference's fused entry: output = up * silu(gate), up weights first."""
    return q4k_gate_up(weights, gate_weights, activations, prod=output, want=("prod",))[2]


def q4k_subdots(weights: torch.Tensor, activations: torch.Tensor):
    """Exact int32 sub-block dots [rows, k/32] and activation quant sums [k/32]."""
    _need(weights, "weights", torch.uint8)
    _need(activations, "activations", torch.uint8)
    k = _k_from_q8(activations)
    rows = _rows(weights, F.q4k_row_bytes(k), "Q4_K")
    dots = torch.empty(rows, k // 32, dtype=torch.int32, device=weights.device)
    sums = torch.empty(k // 32, dtype=torch.int32, device=weights.device)
    check(lib().mllb_q4k_subdots(weights.data_ptr(), activations.data_ptr(), dots.data_ptr(), sums.data_ptr(),
                                 rows, k, _stream(weights)), "q4k_subdots")
    return dots, sums


# ------------------------------------------------------------------- Q6_K

def q6_k_q8_1_matvec(weights: torch.Tensor, activations: torch.Tensor,
                     output: torch.Tensor | None = None, pdl: bool = False) -> torch.Tensor:
    _need(weights, "weights", torch.uint8)
    _need(activations, "activations", torch.uint8)
    k = _k_from_q8(activations)
    rows = _rows(weights, F.q6k_row_bytes(k), "Q6_K")
    if output is None:
        output = torch.empty(rows, dtype=torch.float32, device=weights.device)
    _need(output, "output", torch.float32)
    if output.numel() != rows:
        raise ValueError("output has the wrong size")
    _same_device(weights, activations, output)
    check(lib().mllb_q6k_matvec_ex(weights.data_ptr(), activations.data_ptr(), output.data_ptr(), rows, k,
                                   LAUNCH_PDL if pdl else 0, _stream(weights)), "q6_k_q8_1_matvec")
    return output


# ------------------------------------------------------------------- IMROPE

def fused_q_imrope_runtime_fastpow(q: torch.Tensor, gamma: torch.Tensor, positions: torch.Tensor,
                                   output: torch.Tensor, theta_scale: torch.Tensor) -> torch.Tensor:
    """Reference pointer list: q[heads,128], gamma[128], positions int32[4], output, theta_scale fp32[1]."""
    _need(q, "q", torch.float32)
    _need(gamma, "gamma", torch.float32)
    _need(positions, "positions", torch.int32)
    _need(output, "output", torch.float32)
    _need(theta_scale, "theta_scale", torch.float32)
    if q.numel() == 0 or q.numel() % F.HEAD_DIM or gamma.numel() != F.HEAD_DIM or positions.numel() != 4 \
            or output.numel() != q.numel() or theta_scale.numel() != 1:
        raise ValueError("wrong reference shape")
    _same_device(q, gamma, positions, output, theta_scale)
    check(lib().mllb_rmsnorm_imrope_q(q.data_ptr(), gamma.data_ptr(), positions.data_ptr(), theta_scale.data_ptr(),
                                      output.data_ptr(), q.numel() // F.HEAD_DIM, _stream(q)),
          "fused_q_imrope_runtime_fastpow")
    return output


def rmsnorm_imrope_q(q: torch.Tensor, gamma: torch.Tensor, positions: torch.Tensor,
                     theta_scale: torch.Tensor | float | None = None, out: torch.Tensor | None = None,
                     heads_per_token: int | None = None, pdl: bool = False,
                     const_aux: bool = False) -> torch.Tensor:
    """Batched form: q[tokens*heads_per_token, 128], positions int32[tokens, 4].

    theta_scale: a device fp32[1] tensor (reference ABI), a Python float used
    as the exact float64 scale, or None for pow(5e6, -2/128) in float64.
    pdl: programmatic dependent launch; with const_aux too, gamma, positions
    and theta_scale (not written by the preceding kernel) are read and the
    rotation table built before waiting for it (MLLB_LAUNCH_CONST_AUX).
    """
    _need(q, "q", torch.float32)
    _need(gamma, "gamma", torch.float32)
    _need(positions, "positions", torch.int32)
    if q.numel() == 0 or q.numel() % F.HEAD_DIM or gamma.numel() != F.HEAD_DIM or positions.numel() % 4:
        raise ValueError("wrong reference shape")
    heads = q.numel() // F.HEAD_DIM
    tokens = positions.numel() // 4
    if heads_per_token is None:
        if heads % tokens:
            raise ValueError("heads do not split evenly over the tokens")
        heads_per_token = heads // tokens
    if heads_per_token * tokens != heads:
        raise ValueError("heads_per_token * tokens != heads")
    if out is None:
        out = torch.empty_like(q)
    _need(out, "out", torch.float32)
    ptr, value = None, F.IMROPE_FREQ_BASE ** (-2.0 / F.HEAD_DIM)
    if isinstance(theta_scale, torch.Tensor):
        _need(theta_scale, "theta_scale", torch.float32)
        ptr = theta_scale.data_ptr()
    elif theta_scale is not None:
        value = float(theta_scale)
    _same_device(q, gamma, positions, out)
    check(lib().mllb_rmsnorm_imrope_q_batched_ex(q.data_ptr(), gamma.data_ptr(), positions.data_ptr(), ptr, value,
                                                 out.data_ptr(), tokens, heads_per_token,
                                                 (LAUNCH_PDL if pdl else 0) | (LAUNCH_CONST_AUX if const_aux else 0),
                                                 _stream(q)),
          "rmsnorm_imrope_q")
    return out


# ------------------------------------------------------------------- probe

def stream_read(data: torch.Tensor, out: torch.Tensor | None = None, blocks: int = 0) -> torch.Tensor:
    """XOR-stream `data` once with 16-byte loads (HBM read roofline)."""
    _need(data, "data", torch.uint8)
    if blocks <= 0:
        blocks = torch.cuda.get_device_properties(data.device).multi_processor_count * 8
    if out is None:
        out = torch.empty(blocks * 256 * 16, dtype=torch.uint8, device=data.device)
    check(lib().mllb_stream_read(data.data_ptr(), data.numel(), out.data_ptr(), blocks, _stream(data)),
          "stream_read")
    return out


# ------------------------------------------------------------------ decode
# The ops of one decode step around the matvecs (mojo_llm_lab_b200.decode
# chains them).  `state` is the 32-byte mllb_decode_state as a uint8 tensor.

def _flags(pdl: bool) -> int:
    return LAUNCH_PDL if pdl else 0


def _ptr(t):
    return None if t is None else t.data_ptr()


def token_key(token: int) -> int:
    """Packed next-token key that selects `token`."""
    return int(lib().mllb_token_key(token))


def key_token(key: int) -> int:
    """Token index of a packed key (-1 for the empty key INT64_MIN)."""
    return int(lib().mllb_key_token(key))


def _need_state(state: torch.Tensor) -> None:
    _need(state, "state", torch.uint8)
    if state.numel() != 32:
        raise ValueError("state must be the 32-byte mllb_decode_state")


def rmsnorm_q8_1(x: torch.Tensor, gamma: torch.Tensor, delta: torch.Tensor | None = None,
                 x_out: torch.Tensor | None = None, q8: torch.Tensor | None = None, eps: float = 1e-6,
                 s_mode: int = S_D_SUMQ, pdl: bool = False) -> torch.Tensor:
    """q8 = Q8_1(fp32(h * rsqrt(mean(h^2) + eps) * gamma)), h = x + delta (stored to x_out)."""
    for name, t in (("x", x), ("gamma", gamma), ("delta", delta), ("x_out", x_out)):
        if t is not None:
            _need(t, name, torch.float32)
            if t.numel() != x.numel():
                raise ValueError(f"{name} must have {x.numel()} values")
    k = x.numel()
    if q8 is None:
        q8 = torch.empty(F.q8_1_bytes(k), dtype=torch.uint8, device=x.device)
    _need(q8, "q8", torch.uint8)
    _same_device(x, gamma, delta, x_out, q8)
    check(lib().mllb_rmsnorm_q8_1(x.data_ptr(), _ptr(delta), _ptr(x_out), gamma.data_ptr(), eps, q8.data_ptr(), k,
                                  s_mode, _flags(pdl), _stream(x)), "rmsnorm_q8_1")
    return q8


def decode_final_norm(x: torch.Tensor, gamma: torch.Tensor, state: torch.Tensor, delta: torch.Tensor | None = None,
                      x_out: torch.Tensor | None = None, q8: torch.Tensor | None = None, eps: float = 1e-6,
                      pdl: bool = False) -> torch.Tensor:
    """rmsnorm_q8_1 that also resets the next-token key and advances pos / steps."""
    _need_state(state)
    k = x.numel()
    if q8 is None:
        q8 = torch.empty(F.q8_1_bytes(k), dtype=torch.uint8, device=x.device)
    _same_device(x, gamma, delta, x_out, q8, state)
    check(lib().mllb_decode_final_norm(x.data_ptr(), _ptr(delta), _ptr(x_out), gamma.data_ptr(), eps, q8.data_ptr(),
                                       k, state.data_ptr(), _flags(pdl), _stream(x)), "decode_final_norm")
    return q8


def decode_embed(q6k_weights: torch.Tensor, vocab: int, state: torch.Tensor, hidden: torch.Tensor,
                 tokens: torch.Tensor | None = None, pdl: bool = False) -> torch.Tensor:
    """hidden = dequantised row (token of the state's key) of the Q6_K matrix."""
    _need(q6k_weights, "q6k_weights", torch.uint8)
    _need(hidden, "hidden", torch.float32)
    _need_state(state)
    k = hidden.numel()
    if q6k_weights.numel() != vocab * F.q6k_row_bytes(k):
        raise ValueError("Q6_K matrix size does not match vocab x hidden")
    if tokens is not None:
        _need(tokens, "tokens", torch.int32)
    _same_device(q6k_weights, state, hidden, tokens)
    check(lib().mllb_decode_embed(q6k_weights.data_ptr(), vocab, k, state.data_ptr(), _ptr(tokens),
                                  0 if tokens is None else tokens.numel(), hidden.data_ptr(), _flags(pdl),
                                  _stream(hidden)), "decode_embed")
    return hidden


def decode_qk_rope_append(qkv: torch.Tensor, q_gamma: torch.Tensor, k_gamma: torch.Tensor, state: torch.Tensor,
                          k_cache: torch.Tensor, v_cache: torch.Tensor, q_heads: int, kv_heads: int,
                          theta_scale: float | None = None, q_out: torch.Tensor | None = None,
                          pdl: bool = False) -> torch.Tensor:
    """q/k RMSNorm + gamma + IMROPE at state.pos; K, V appended to the fp16 caches [kv_heads, ctx, 128]."""
    _need(qkv, "qkv", torch.float32)
    _need(q_gamma, "q_gamma", torch.float32)
    _need(k_gamma, "k_gamma", torch.float32)
    _need(k_cache, "k_cache", torch.float16)
    _need(v_cache, "v_cache", torch.float16)
    _need_state(state)
    if qkv.numel() != (q_heads + 2 * kv_heads) * F.HEAD_DIM:
        raise ValueError("qkv must hold (q_heads + 2 kv_heads) x 128 values")
    if k_cache.dim() != 3 or k_cache.shape[0] != kv_heads or k_cache.shape[2] != F.HEAD_DIM:
        raise ValueError("caches must be [kv_heads, ctx, 128]")
    if v_cache.shape != k_cache.shape:
        raise ValueError("v_cache must match k_cache")
    if q_out is None:
        q_out = torch.empty(q_heads * F.HEAD_DIM, dtype=torch.float32, device=qkv.device)
    theta = F.theta_scale_f32() if theta_scale is None else float(theta_scale)
    _same_device(qkv, q_gamma, k_gamma, state, k_cache, v_cache, q_out)
    check(lib().mllb_decode_qk_rope_append(qkv.data_ptr(), q_gamma.data_ptr(), k_gamma.data_ptr(), state.data_ptr(),
                                           theta, q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), q_heads,
                                           kv_heads, k_cache.shape[1], _flags(pdl), _stream(qkv)),
          "decode_qk_rope_append")
    return q_out


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, state: torch.Tensor,
                     out: torch.Tensor | None = None, q8: torch.Tensor | None = None,
                     scratch: torch.Tensor | None = None, pdl: bool = False):
    """Attention of the token at state.pos over cache rows 0..pos -> (out fp32, Q8_1 of out)."""
    _need(q, "q", torch.float32)
    _need(k_cache, "k_cache", torch.float16)
    _need(v_cache, "v_cache", torch.float16)
    _need_state(state)
    kv_heads, ctx = k_cache.shape[0], k_cache.shape[1]
    q_heads = q.numel() // F.HEAD_DIM
    with torch.cuda.device(q.device):
        need = int(lib().mllb_decode_attention_scratch(q_heads, kv_heads, ctx))
    if need < 0:
        check(int(need), "decode_attention_scratch")
    if scratch is None:
        scratch = torch.empty(need, dtype=torch.float64, device=q.device)
    _need(scratch, "scratch", torch.float64)
    if out is None:
        out = torch.empty(q.numel(), dtype=torch.float32, device=q.device)
    if q8 is None:
        q8 = torch.empty(F.q8_1_bytes(q.numel()), dtype=torch.uint8, device=q.device)
    _same_device(q, k_cache, v_cache, state, out, q8, scratch)
    check(lib().mllb_decode_attention(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), state.data_ptr(),
                                      scratch.data_ptr(), scratch.numel(), out.data_ptr(), q8.data_ptr(), q_heads,
                                      kv_heads, ctx, _flags(pdl), _stream(q)), "decode_attention")
    return out, q8


def decode_attention_qkv(qkv: torch.Tensor, q_gamma: torch.Tensor, k_gamma: torch.Tensor, state: torch.Tensor,
                         k_cache: torch.Tensor, v_cache: torch.Tensor, q_heads: int,
                         theta_scale: float | None = None, out: torch.Tensor | None = None,
                         q8: torch.Tensor | None = None, scratch: torch.Tensor | None = None, pdl: bool = False):
    """Fused q/k RMSNorm + IMROPE, KV append at state.pos and attention -> (out fp32, Q8_1 of out)."""
    _need(qkv, "qkv", torch.float32)
    _need(q_gamma, "q_gamma", torch.float32)
    _need(k_gamma, "k_gamma", torch.float32)
    _need(k_cache, "k_cache", torch.float16)
    _need(v_cache, "v_cache", torch.float16)
    _need_state(state)
    kv_heads, ctx = k_cache.shape[0], k_cache.shape[1]
    if qkv.numel() != (q_heads + 2 * kv_heads) * F.HEAD_DIM:
        raise ValueError("qkv must hold (q_heads + 2 kv_heads) x 128 values")
    if v_cache.shape != k_cache.shape or k_cache.dim() != 3 or k_cache.shape[2] != F.HEAD_DIM:
        raise ValueError("caches must both be [kv_heads, ctx, 128]")
    with torch.cuda.device(qkv.device):
        need = int(lib().mllb_decode_attention_scratch(q_heads, kv_heads, ctx))
    if need < 0:
        check(int(need), "decode_attention_scratch")
    if scratch is None:
        scratch = torch.empty(need, dtype=torch.float64, device=qkv.device)
    _need(scratch, "scratch", torch.float64)
    width = q_heads * F.HEAD_DIM
    if out is None:
        out = torch.empty(width, dtype=torch.float32, device=qkv.device)
    if q8 is None:
        q8 = torch.empty(F.q8_1_bytes(width), dtype=torch.uint8, device=qkv.device)
    theta = F.theta_scale_f32() if theta_scale is None else float(theta_scale)
    _same_device(qkv, q_gamma, k_gamma, state, k_cache, v_cache, out, q8, scratch)
    check(lib().mllb_decode_attention_qkv(qkv.data_ptr(), q_gamma.data_ptr(), k_gamma.data_ptr(), theta,
                                          state.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), scratch.data_ptr(),
                                          scratch.numel(), out.data_ptr(), q8.data_ptr(), q_heads, kv_heads, ctx,
                                          _flags(pdl), _stream(qkv)), "decode_attention_qkv")
    return out, q8


def _need_q4_0_cache(k_qs: torch.Tensor, v_qs: torch.Tensor, kv_d: torch.Tensor) -> tuple[int, int]:
    _need(k_qs, "k_qs", torch.uint8)
    _need(v_qs, "v_qs", torch.uint8)
    _need(kv_d, "kv_d", torch.float16)
    if k_qs.dim() != 3 or k_qs.shape[2] != F.HEAD_DIM // 2 or v_qs.shape != k_qs.shape:
        raise ValueError("k_qs and v_qs must both be uint8 [kv_heads, ctx, 64]")
    if kv_d.shape != (k_qs.shape[0], k_qs.shape[1], 8):
        raise ValueError("kv_d must be fp16 [kv_heads, ctx, 8]")
    return k_qs.shape[0], k_qs.shape[1]


def kv_q4_0_store(k: torch.Tensor, v: torch.Tensor, k_qs: torch.Tensor, v_qs: torch.Tensor, kv_d: torch.Tensor,
                  row0: int = 0, pdl: bool = False) -> None:
    """Quantise fp32 K and V rows [kv_heads, rows, 128] into rows row0.. of
    the Q4_0 cache planes (GGML quantize_row_q4_0 rule)."""
    _need(k, "k", torch.float32)
    _need(v, "v", torch.float32)
    kv_heads, ctx = _need_q4_0_cache(k_qs, v_qs, kv_d)
    if k.dim() != 3 or k.shape[0] != kv_heads or k.shape[2] != F.HEAD_DIM or v.shape != k.shape:
        raise ValueError("k and v must both be fp32 [kv_heads, rows, 128]")
    _same_device(k, v, k_qs, v_qs, kv_d)
    check(lib().mllb_kv_q4_0_store(k.data_ptr(), v.data_ptr(), k_qs.data_ptr(), v_qs.data_ptr(), kv_d.data_ptr(),
                                   kv_heads, ctx, row0, k.shape[1], _flags(pdl), _stream(k)), "kv_q4_0_store")


def _attention_buffers(dev, q_heads: int, kv_heads: int, ctx: int, out, q8, scratch):
    with torch.cuda.device(dev):
        need = int(lib().mllb_decode_attention_scratch(q_heads, kv_heads, ctx))
    if need < 0:
        check(int(need), "decode_attention_scratch")
    if scratch is None:
        scratch = torch.empty(need, dtype=torch.float64, device=dev)
    _need(scratch, "scratch", torch.float64)
    width = q_heads * F.HEAD_DIM
    if out is None:
        out = torch.empty(width, dtype=torch.float32, device=dev)
    if q8 is None:
        q8 = torch.empty(F.q8_1_bytes(width), dtype=torch.uint8, device=dev)
    return out, q8, scratch


def decode_attention_q4_0(q: torch.Tensor, k_qs: torch.Tensor, v_qs: torch.Tensor, kv_d: torch.Tensor,
                          state: torch.Tensor, out: torch.Tensor | None = None, q8: torch.Tensor | None = None,
                          scratch: torch.Tensor | None = None, pdl: bool = False):
    """decode_attention over the Q4_0 cache planes -> (out fp32, Q8_1 of out)."""
    _need(q, "q", torch.float32)
    _need_state(state)
    kv_heads, ctx = _need_q4_0_cache(k_qs, v_qs, kv_d)
    q_heads = q.numel() // F.HEAD_DIM
    out, q8, scratch = _attention_buffers(q.device, q_heads, kv_heads, ctx, out, q8, scratch)
    _same_device(q, k_qs, v_qs, kv_d, state, out, q8, scratch)
    check(lib().mllb_decode_attention_q4_0(q.data_ptr(), k_qs.data_ptr(), v_qs.data_ptr(), kv_d.data_ptr(),
                                           state.data_ptr(), scratch.data_ptr(), scratch.numel(), out.data_ptr(),
                                           q8.data_ptr(), q_heads, kv_heads, ctx, _flags(pdl), _stream(q)),
          "decode_attention_q4_0")
    return out, q8


def decode_attention_qkv_q4_0(qkv: torch.Tensor, q_gamma: torch.Tensor, k_gamma: torch.Tensor, state: torch.Tensor,
                              k_qs: torch.Tensor, v_qs: torch.Tensor, kv_d: torch.Tensor, q_heads: int,
                              theta_scale: float | None = None, out: torch.Tensor | None = None,
                              q8: torch.Tensor | None = None, scratch: torch.Tensor | None = None,
                              pdl: bool = False):
    """decode_attention_qkv with the K/V rows appended to the Q4_0 cache planes."""
    _need(qkv, "qkv", torch.float32)
    _need(q_gamma, "q_gamma", torch.float32)
    _need(k_gamma, "k_gamma", torch.float32)
    _need_state(state)
    kv_heads, ctx = _need_q4_0_cache(k_qs, v_qs, kv_d)
    if qkv.numel() != (q_heads + 2 * kv_heads) * F.HEAD_DIM:
        raise ValueError("qkv must hold (q_heads + 2 kv_heads) x 128 values")
    out, q8, scratch = _attention_buffers(qkv.device, q_heads, kv_heads, ctx, out, q8, scratch)
    theta = F.theta_scale_f32() if theta_scale is None else float(theta_scale)
    _same_device(qkv, q_gamma, k_gamma, state, k_qs, v_qs, kv_d, out, q8, scratch)
    check(lib().mllb_decode_attention_qkv_q4_0(qkv.data_ptr(), q_gamma.data_ptr(), k_gamma.data_ptr(), theta,
                                               state.data_ptr(), k_qs.data_ptr(), v_qs.data_ptr(), kv_d.data_ptr(),
                                               scratch.data_ptr(), scratch.numel(), out.data_ptr(), q8.data_ptr(),
                                               q_heads, kv_heads, ctx, _flags(pdl), _stream(qkv)),
          "decode_attention_qkv_q4_0")
    return out, q8


def argmax_key(x: torch.Tensor, key: torch.Tensor, index_offset: int = 0, pdl: bool = False) -> torch.Tensor:
    """key[0] = max(key[0], packed (x[i], index_offset + i) over i); key: int64[1]."""
    _need(x, "x", torch.float32)
    _need(key, "key", torch.int64)
    _same_device(x, key)
    check(lib().mllb_argmax_f32(x.data_ptr(), x.numel(), index_offset, key.data_ptr(), _flags(pdl), _stream(x)),
          "argmax")
    return key


# --------------------------------------------- matvecs with an fp32 activation

def act_f32(x: torch.Tensor, delta: torch.Tensor | None = None, gamma: torch.Tensor | None = None,
            x_out: torch.Tensor | None = None, eps: float = 1e-6, advance: torch.Tensor | None = None) -> ActF32:
    """Describe an activation built inside the matvec: Q8_1(rmsnorm(x + delta) * gamma), or
    Q8_1(x + delta) without gamma; x + delta is stored to x_out; advance is a decode state."""
    for name, t in (("x", x), ("delta", delta), ("gamma", gamma), ("x_out", x_out)):
        if t is not None:
            _need(t, name, torch.float32)
            if t.numel() != x.numel():
                raise ValueError(f"{name} must have {x.numel()} values")
    if advance is not None:
        _need_state(advance)
    _same_device(x, delta, gamma, x_out, advance)
    return ActF32(x.data_ptr(), _ptr(delta), _ptr(gamma), _ptr(x_out), eps, _ptr(advance))


def q4k_matvec_act(weights: torch.Tensor, act: ActF32, k: int, output: torch.Tensor, pdl: bool = False):
    _need(weights, "weights", torch.uint8)
    _need(output, "output", torch.float32)
    rows = _rows(weights, F.q4k_row_bytes(k), "Q4_K")
    check(lib().mllb_q4k_matvec_act(weights.data_ptr(), act, output.data_ptr(), rows, k, _flags(pdl),
                                    _stream(weights)), "q4k_matvec_act")
    return output


def q4k_gate_up_act(up_weights: torch.Tensor, gate_weights: torch.Tensor, act: ActF32, k: int,
                    up: torch.Tensor | None = None, gate: torch.Tensor | None = None,
                    prod: torch.Tensor | None = None, pdl: bool = False):
    _need(up_weights, "up_weights", torch.uint8)
    _need(gate_weights, "gate_weights", torch.uint8)
    rows = _rows(up_weights, F.q4k_row_bytes(k), "Q4_K")
    check(lib().mllb_q4k_gate_up_act(up_weights.data_ptr(), gate_weights.data_ptr(), act, _ptr(up), _ptr(gate),
                                     _ptr(prod), rows, k, _flags(pdl), _stream(up_weights)), "q4k_gate_up_act")
    return up, gate, prod


def q6k_matvec_act(weights: torch.Tensor, act: ActF32, k: int, output: torch.Tensor, pdl: bool = False):
    _need(weights, "weights", torch.uint8)
    _need(output, "output", torch.float32)
    rows = _rows(weights, F.q6k_row_bytes(k), "Q6_K")
    check(lib().mllb_q6k_matvec_act(weights.data_ptr(), act, output.data_ptr(), rows, k, _flags(pdl),
                                    _stream(weights)), "q6k_matvec_act")
    return output



# ------------------------------------- gate/up with the Q8_1 of its product

def q4k_gate_up_q8(up_weights: torch.Tensor, gate_weights: torch.Tensor, activations: torch.Tensor,
                   prod: torch.Tensor, q8_out: torch.Tensor, counters: torch.Tensor,
                   up: torch.Tensor | None = None, gate: torch.Tensor | None = None, pdl: bool = False):
    """Fused gate/up that also writes the Q8_1 of prod = up * silu(gate) (counters: rows / 32 zeroed int32,
    left zero by every call)."""
    _need(up_weights, "up_weights", torch.uint8)
    _need(gate_weights, "gate_weights", torch.uint8)
    _need(activations, "activations", torch.uint8)
    k = _k_from_q8(activations)
    rows = _rows(up_weights, F.q4k_row_bytes(k), "Q4_K")
    if gate_weights.numel() != up_weights.numel():
        raise ValueError("up and gate matrices differ in size")
    for name, t in (("prod", prod), ("up", up), ("gate", gate)):
        if t is not None:
            _need(t, name, torch.float32)
            if t.numel() != rows:
                raise ValueError(f"{name} has the wrong size")
    _need(q8_out, "q8_out", torch.uint8)
    if q8_out.numel() != F.q8_1_bytes(rows):
        raise ValueError("q8_out has the wrong size")
    _need(counters, "counters", torch.int32)
    if counters.numel() < rows // 32:
        raise ValueError("counters needs rows / 32 entries")
    _same_device(up_weights, gate_weights, activations, prod, q8_out, counters, up, gate)
    check(lib().mllb_q4k_gate_up_q8(up_weights.data_ptr(), gate_weights.data_ptr(), activations.data_ptr(),
                                    _ptr(up), _ptr(gate), prod.data_ptr(), q8_out.data_ptr(), counters.data_ptr(),
                                    rows, k, _flags(pdl), _stream(up_weights)), "q4k_gate_up_q8")
    return q8_out


def q4k_matvec_norm_workspace(rows: int, k: int, device) -> torch.Tensor:
    """Zeroed workspace for q4k_matvec_norm (reusable by calls that do not overlap on the GPU)."""
    need = int(lib().mllb_q4k_matvec_norm_workspace(rows, k))
    if need < 0:
        check(need, "q4k_matvec_norm_workspace")
    return torch.zeros(need, dtype=torch.uint8, device=device)


def q4k_matvec_norm(weights: torch.Tensor, activations: torch.Tensor, x: torch.Tensor, gamma: torch.Tensor,
                    eps: float = 1e-6, x_out: torch.Tensor | None = None, q8_out: torch.Tensor | None = None,
                    out: torch.Tensor | None = None, workspace: torch.Tensor | None = None, pdl: bool = False):
    """Q4_K matvec whose output is a residual delta, with the next RMSNorm + Q8_1 built in:
    h = x + W a -> x_out, q8_out = Q8_1(rmsnorm(h) * gamma).  Returns (x_out, q8_out, out)."""
    _need(weights, "weights", torch.uint8)
    _need(activations, "activations", torch.uint8)
    k = _k_from_q8(activations)
    rows = _rows(weights, F.q4k_row_bytes(k), "Q4_K")
    _need(x, "x", torch.float32)
    _need(gamma, "gamma", torch.float32)
    if x.numel() != rows or gamma.numel() != rows:
        raise ValueError("x and gamma need one value per row")
    if x_out is None:
        x_out = torch.empty_like(x)
    if q8_out is None:
        q8_out = torch.empty(F.q8_1_bytes(rows), dtype=torch.uint8, device=x.device)
    if workspace is None:
        workspace = q4k_matvec_norm_workspace(rows, k, x.device)
    for name, t in (("x_out", x_out), ("out", out)):
        if t is not None:
            _need(t, name, torch.float32)
            if t.numel() != rows:
                raise ValueError(f"{name} has the wrong size")
    _need(q8_out, "q8_out", torch.uint8)
    if q8_out.numel() != F.q8_1_bytes(rows):
        raise ValueError("q8_out has the wrong size")
    _need(workspace, "workspace", torch.uint8)
    _same_device(weights, activations, x, gamma, x_out, q8_out, out, workspace)
    check(lib().mllb_q4k_matvec_norm(weights.data_ptr(), activations.data_ptr(), _ptr(out), rows, k, x.data_ptr(),
                                     x_out.data_ptr(), gamma.data_ptr(), float(eps), q8_out.data_ptr(),
                                     workspace.data_ptr(), workspace.numel(), _flags(pdl), _stream(weights)),
          "q4k_matvec_norm")
    return x_out, q8_out, out


# ------------------------------------------------------- batched tokens (prefill)

def q4k_matmul_tokens(weights: torch.Tensor, activations: torch.Tensor, output: torch.Tensor | None = None,
                      k: int | None = None) -> torch.Tensor:
    """out[t] = W @ x_t for T tokens at once (tensor-core int8 group dots, fp64 scaling).

    weights: Q4_K bytes of `rows` (a multiple of 128) rows; activations: T consecutive Q8_1
    rows ([T, K/32*36] or flat, then `k` gives K); output: fp32 [T, rows]."""
    _need(weights, "weights", torch.uint8)
    _need(activations, "activations", torch.uint8)
    if activations.dim() == 2:
        k = activations.shape[1] // F.Q8_1_BLOCK_BYTES * F.Q8_1_GROUP
    elif k is None:
        raise ValueError("flat activations need k")
    q8_row = k // F.Q8_1_GROUP * F.Q8_1_BLOCK_BYTES
    if k <= 0 or k % 256 or activations.numel() % q8_row:
        raise ValueError("activations are not whole Q8_1 rows of K = a multiple of 256")
    tokens = activations.numel() // q8_row
    rows = _rows(weights, F.q4k_row_bytes(k), "Q4_K")
    if output is None:
        output = torch.empty(tokens, rows, dtype=torch.float32, device=weights.device)
    _need(output, "output", torch.float32)
    if output.numel() != tokens * rows:
        raise ValueError("output must hold tokens x rows values")
    _same_device(weights, activations, output)
    L = lib()
    with torch.cuda.device(weights.device):
        need = int(L.mllb_q4k_matmul_tokens_workspace(rows, k, tokens))
    if need < 0:
        check(need, "q4k_matmul_tokens_workspace")
    work = torch.empty(max(need, 8), dtype=torch.uint8, device=weights.device) if need > 0 else None
    check(L.mllb_q4k_matmul_tokens(weights.data_ptr(), activations.data_ptr(), output.data_ptr(), rows, k, tokens,
                                   _ptr(work), need, 0, _stream(weights)), "q4k_matmul_tokens")
    return output


def q5_k_q8_1_matvec(weights: torch.Tensor, activations: torch.Tensor, output: torch.Tensor | None = None,
                     pdl: bool = False) -> torch.Tensor:
    """Q5_K x Q8_1 matvec (K = 2048, 2560 or 4096)."""
    _need(weights, "weights", torch.uint8)
    _need(activations, "activations", torch.uint8)
    k = _k_from_q8(activations)
    rows = _rows(weights, F.q5k_row_bytes(k), "Q5_K")
    if output is None:
        output = torch.empty(rows, dtype=torch.float32, device=weights.device)
    _need(output, "output", torch.float32)
    if output.numel() != rows:
        raise ValueError(f"output must have {rows} values")
    _same_device(weights, activations, output)
    check(lib().mllb_q5k_matvec_ex(weights.data_ptr(), activations.data_ptr(), output.data_ptr(), rows, k,
                                   _flags(pdl), _stream(weights)), "q5_k_q8_1_matvec")
    return output
