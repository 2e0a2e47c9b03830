"""Float64 restatement of one synthetic decode step -- TEST INFRASTRUCTURE ONLY.

Composes the oracle's per-op restatements (``oracle.c``) into the step that
``mojo_llm_lab_b200.decode.Decoder`` runs on the GPU: embedding, then per
layer residual + RMSNorm -> Q8_1, the fused QKV matvec, q/k RMSNorm + IMROPE
with the fp16 KV append, attention, the O matvec, residual + RMSNorm, the
gate/up SwiGLU, Q8_1 of the product, the down matvec; final norm, Q6_K
logits, first-maximum argmax.  The KV cache is fp16 rows or the Q4_0 planes
(GGML quantize_row_q4_0 of the fp32 K / V rows).  Every value handed from one op to the next is
rounded to fp32 (fp16 in the cache, Q8_1 bytes for matvec inputs) exactly
where the GPU rounds it, so the two agree bit for bit barring rounding ties.

The reference has no whole-model CPU path (it decodes through llama.cpp,
integration/resident_decode.cpp); its acceptance test for a decode is
full-logit agreement with atol 1e-4, rtol 1e-5 and the same top-1 token
(integration/logit_validation.h:14,76-80), which ``logit_agreement`` restates.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import (argmax, attention, attention_q4_0, embed_q6k, kv_q4_0_rows, q4k_gate_up, q4k_matvec, q6k_matvec,
               qk_rope_append, qk_rope_f32, quantize_q8_1, rmsnorm_q8_1)

ATOL = 1e-4
RTOL = 1e-5


@dataclass
class HostLayer:
    qkv: np.ndarray
    o: np.ndarray
    up: np.ndarray
    gate: np.ndarray
    down: np.ndarray
    attn_norm: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray
    ffn_norm: np.ndarray


@dataclass
class HostModel:
    hidden: int
    q_heads: int
    kv_heads: int
    ffn: int
    vocab: int
    eps: float
    theta_scale: float
    layers: list
    out_norm: np.ndarray
    output: np.ndarray        # full Q6_K matrix (also the embedding)


def host_model(weights) -> HostModel:
    """Host copy of an unsharded ``DecodeWeights``."""
    cfg = weights.cfg
    if weights.ffn_shard.world != 1:
        raise ValueError("the oracle takes the unsharded weights")
    np_ = lambda t: t.detach().cpu().numpy()  # noqa: E731
    layers = [HostLayer(**{name: np_(getattr(lw, name)) for name in HostLayer.__dataclass_fields__})
              for lw in weights.layers]
    return HostModel(hidden=cfg.hidden, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, ffn=cfg.ffn, vocab=cfg.vocab,
                     eps=cfg.eps, theta_scale=cfg.theta_scale, layers=layers, out_norm=np_(weights.out_norm),
                     output=np_(weights.embedding))


def reference_step(m: HostModel, k_cache: np.ndarray | None, v_cache: np.ndarray | None, token: int, pos: int,
                   threads: int = 0, q4_0: tuple | None = None) -> tuple[np.ndarray, int]:
    """One decode step of `token` at `pos`.  k_cache / v_cache: fp16 bit
    patterns (uint16) [layers, kv_heads, ctx, 128], updated in place at row
    `pos`; or, with q4_0 = (k_qs uint8 [layers, kv_heads, ctx, 64], v_qs,
    d fp16 bits [layers, kv_heads, ctx, 8]), the Q4_0 cache planes, updated
    in place.  Returns (fp32 logits, greedy next token)."""
    h = embed_q6k(m.output, m.hidden, token)
    delta = None
    for layer, lw in enumerate(m.layers):
        h, a = rmsnorm_q8_1(h, delta, lw.attn_norm, m.eps)
        qkv = q4k_matvec(lw.qkv, a, (m.q_heads + 2 * m.kv_heads) * 128, m.hidden, threads).astype(np.float32)
        if q4_0 is None:
            q, k_row, v_row = qk_rope_append(qkv, m.q_heads, m.kv_heads, lw.q_norm, lw.k_norm, pos, m.theta_scale)
            k_cache[layer, :, pos, :] = k_row.reshape(m.kv_heads, 128)
            v_cache[layer, :, pos, :] = v_row.reshape(m.kv_heads, 128)
            att = attention(q, k_cache[layer], v_cache[layer], pos + 1, m.q_heads, m.kv_heads, threads)
        else:
            k_qs, v_qs, kv_d = q4_0
            q, k_f32, v_f32 = qk_rope_f32(qkv, m.q_heads, m.kv_heads, lw.q_norm, lw.k_norm, pos, m.theta_scale)
            k_qs[layer, :, pos], kv_d[layer, :, pos, :4] = kv_q4_0_rows(k_f32.reshape(m.kv_heads, 128))
            v_qs[layer, :, pos], kv_d[layer, :, pos, 4:] = kv_q4_0_rows(v_f32.reshape(m.kv_heads, 128))
            att = attention_q4_0(q, k_qs[layer], v_qs[layer], kv_d[layer], pos + 1, m.q_heads, m.kv_heads, threads)
        o = q4k_matvec(lw.o, quantize_q8_1(att), m.hidden, m.q_heads * 128, threads).astype(np.float32)
        h, a = rmsnorm_q8_1(h, o, lw.ffn_norm, m.eps)
        _, _, prod = q4k_gate_up(lw.up, lw.gate, a, m.ffn, m.hidden, threads)
        delta = q4k_matvec(lw.down, quantize_q8_1(prod.astype(np.float32)), m.hidden, m.ffn,
                           threads).astype(np.float32)
    h, a = rmsnorm_q8_1(h, delta, m.out_norm, m.eps)
    logits = q6k_matvec(m.output, a, m.vocab, m.hidden, threads).astype(np.float32)
    return logits, argmax(logits)


def logit_agreement(ref: np.ndarray, got: np.ndarray) -> dict:
    """Violations of |got - ref| <= atol + rtol |ref|, the worst ratio, and top-1 equality."""
    ref64, got64 = ref.astype(np.float64), got.astype(np.float64)
    err = np.abs(got64 - ref64)
    ratio = err / (ATOL + RTOL * np.abs(ref64))
    # A non-finite logit on either side is a violation (the reference throws).
    bad = ~np.isfinite(ratio) | (ratio > 1)
    return {"violations": int(bad.sum()),
            "nonfinite": int((~np.isfinite(got64)).sum() + (~np.isfinite(ref64)).sum()),
            "max_abs": float(err.max()), "max_ratio": float(ratio.max()),
            "bit_exact": int((ref.view(np.uint32) == got.view(np.uint32)).sum()), "values": int(ref.size),
            "top_match": int(np.argmax(ref)) == int(np.argmax(got))}
