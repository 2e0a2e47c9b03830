"""Synthetic Qwen3-style single-token decode on the B200 kernels.

The whole-model context of the reference's hot path (its PRD shapes,
docs/PRDs/11-06-2026-quantized-matvec.md:7, and the llama.cpp decode it
profiles, docs/decode-profile.md:5-11): a stack of ``layers`` blocks

    h = embed(token)                                  tied Q6_K output rows
    per layer:
      a   = Q8_1(rmsnorm(h) * attn_gamma)
      qkv = Wqkv a                                    Q4_K, one fused matrix
      q, k = rmsnorm(head) * q/k_gamma + IMROPE;  k, v -> fp16 or Q4_0 KV cache
      o   = Wo Q8_1(attention(q, K, V))               Q4_K
      h  += o;  a = Q8_1(rmsnorm(h) * ffn_gamma)
      f   = up(a) * silu(gate(a))                     fused Q4_K gate/up
      h  += Wdown Q8_1(f)                             Q4_K
    logits = Wout Q8_1(rmsnorm(h) * out_gamma)        Q6_K
    next   = argmax(logits)                           greedy

Everything that changes from token to token (the token, its position, the
KV rows) lives in device memory, so one step is captured once as a CUDA
graph of PDL-chained launches and replayed per token.  On one GPU the
gate/up launch also writes Q8_1(f) (``mllb_q4k_gate_up_q8``), so a layer is
8 launches.  Weights and the
prefilled KV cache are random (seeded) in the distributions of the
reference's fixtures; there is no checkpoint.

Multi-GPU (one process per GPU, ``torch.distributed``): the gate/up and
vocabulary matvecs are row-sharded.  Each rank quantises its slice of the
SwiGLU product and stores the Q8_1 blocks straight into every rank's buffer
over NVLink (``mllb_q8_1_quantize_allgather`` on symmetric memory; NCCL
all-gather when symmetric memory is unavailable), which gives every rank the
down projection's input; each rank takes the argmax of its logit rows and an
NCCL all-reduce MAX of the packed (value, index) keys gives every rank the
next token.  Everything else is replicated.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np
import torch

from . import formats as F
from ._lib import LAUNCH_PDL, ActF32, PeerGather, check, lib
from .shard import RowShard

HEAD_DIM = 128
STATE_BYTES = 32


@dataclass(frozen=True)
class DecodeConfig:
    """Shapes of the synthetic stack (defaults: the 36-layer decode config)."""

    layers: int = 36
    hidden: int = 2560
    q_heads: int = 32
    kv_heads: int = 8
    ffn: int = 9728
    vocab: int = 151936
    context: int = 4096        # prefilled KV rows
    new_tokens: int = 128      # decode steps the KV cache has room for
    eps: float = 1e-6
    theta_bits: int = 0x3F492C27
    seed: int = 20260611

    def validate(self) -> None:
        if self.layers < 1:
            raise ValueError("layers must be >= 1")
        for name in ("hidden", "ffn"):
            if getattr(self, name) <= 0 or getattr(self, name) % 256:
                raise ValueError(f"{name} must be a positive multiple of 256")
        if self.q_heads <= 0 or self.kv_heads <= 0 or self.q_heads % self.kv_heads:
            raise ValueError("q_heads must be a positive multiple of kv_heads")
        if self.q_heads // self.kv_heads not in (1, 2, 4, 8):
            raise ValueError("q_heads / kv_heads must be 1, 2, 4 or 8")
        if (self.q_heads * HEAD_DIM) % 256:
            raise ValueError("q_heads * 128 must be a multiple of 256 (O projection width)")
        if self.vocab <= 0 or self.context < 0 or self.new_tokens <= 0:
            raise ValueError("vocab, new_tokens must be positive and context >= 0")

    @property
    def qkv_rows(self) -> int:
        return (self.q_heads + 2 * self.kv_heads) * HEAD_DIM

    @property
    def attn_width(self) -> int:
        return self.q_heads * HEAD_DIM

    @property
    def ctx_capacity(self) -> int:
        return self.context + self.new_tokens

    @property
    def theta_scale(self) -> float:
        return struct.unpack("<f", struct.pack("<I", self.theta_bits))[0]

    def q4k_bytes(self) -> int:
        """Q4_K weight bytes of the whole stack."""
        per_layer = (self.qkv_rows * self.hidden + self.hidden * self.attn_width + 2 * self.ffn * self.hidden +
                     self.hidden * self.ffn) // 256 * F.Q4K_BLOCK_BYTES
        return per_layer * self.layers

    def q6k_bytes(self) -> int:
        return self.vocab * self.hidden // 256 * F.Q6K_BLOCK_BYTES

    def kv_bytes_read(self, n_keys: int, kv: str = "f16") -> int:
        """K and V bytes one step reads over n_keys cache rows: fp16 rows, or
        the Q4_0 planes (64 + 64 nibble bytes and 16 scale bytes a row)."""
        per_row = 2 * HEAD_DIM * 2 if kv == "f16" else 2 * (HEAD_DIM // 2) + 16
        return self.layers * self.kv_heads * n_keys * per_row

    def bytes_per_token(self, n_keys: int, kv: str = "f16") -> int:
        """Algorithmic HBM bytes of one step: every weight once, the KV rows once."""
        return self.q4k_bytes() + self.q6k_bytes() + self.kv_bytes_read(n_keys, kv)


def _seed(cfg: DecodeConfig, layer: int, slot: int) -> int:
    return (cfg.seed * 1_000_003 + (layer + 1) * 1009 + slot) % (1 << 62)


def _generator(device: torch.device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _fp16_field(n: int, low: float, high: float, g: torch.Generator, device) -> torch.Tensor:
    v = torch.empty(n, dtype=torch.float32, device=device).uniform_(low, high, generator=g)
    return v.half().view(torch.uint8).view(n, 2)


def random_q4k(rows: int, k: int, seed: int, device, signed_scales: bool = True) -> torch.Tensor:
    """Q4_K rows: fp16 |d| ~ U(1e-3, 1e-2), |dmin| ~ U(0, 5e-3), uniform 6-bit
    scales / mins (every bit of the 12 packed bytes belongs to exactly one of
    them, so uniform bytes are uniform fields) and uniform nibbles.

    signed_scales gives each block's d and dmin independent random signs.
    With both positive every weight d*sc*q - dmin*m has mean ~ +1.2, each
    projection output carries a common mode of ~1.2 * sum(input) that RMSNorm
    turns into an all-positive input of the next layer, and within two layers
    the SwiGLU product passes 127 * 65504, the largest activation a Q8_1
    block's fp16 scale can hold: the scale becomes inf and the logits NaN (as
    in GGML).  A random sign of d alone still leaves the -dmin*m bias, whose
    common mode builds up along the residual stream until the same overflow
    (layer 32 of 36).  With both signs random the rows are zero-mean and the
    36-layer stack stays finite."""
    g = _generator(torch.device(device), seed)
    n = rows * (k // 256)
    blocks = torch.randint(0, 256, (n, F.Q4K_BLOCK_BYTES), dtype=torch.uint8, generator=g, device=device)
    blocks[:, 0:2] = _fp16_field(n, 1e-3, 1e-2, g, device)
    blocks[:, 2:4] = _fp16_field(n, 0.0, 5e-3, g, device)
    if signed_scales:
        signs = torch.randint(0, 4, (n,), dtype=torch.uint8, generator=g, device=device)
        blocks[:, 1] |= (signs & 1) << 7
        blocks[:, 3] |= (signs & 2) << 6
    return blocks.view(-1)


def random_q6k(rows: int, k: int, seed: int, device) -> torch.Tensor:
    """Q6_K rows: uniform ql / qh bytes, int8 scales ~ U{-32..31}, fp16 d ~ U(1e-3, 1e-2)."""
    g = _generator(torch.device(device), seed)
    n = rows * (k // 256)
    blocks = torch.randint(0, 256, (n, F.Q6K_BLOCK_BYTES), dtype=torch.uint8, generator=g, device=device)
    blocks[:, 192:208] = torch.randint(-32, 32, (n, 16), dtype=torch.int8, generator=g,
                                       device=device).view(torch.uint8)
    blocks[:, 208:210] = _fp16_field(n, 1e-3, 1e-2, g, device)
    return blocks.view(-1)


def random_gamma(n: int, seed: int, device) -> torch.Tensor:
    g = _generator(torch.device(device), seed)
    return torch.empty(n, dtype=torch.float32, device=device).uniform_(0.5, 1.5, generator=g)


@dataclass
class LayerWeights:
    qkv: torch.Tensor         # Q4_K [(q_heads + 2 kv_heads) * 128, hidden]
    o: torch.Tensor           # Q4_K [hidden, q_heads * 128]
    up: torch.Tensor          # Q4_K [ffn rows of this rank, hidden]
    gate: torch.Tensor        # Q4_K [ffn rows of this rank, hidden]
    down: torch.Tensor        # Q4_K [hidden, ffn]
    attn_norm: torch.Tensor   # fp32 [hidden]
    q_norm: torch.Tensor      # fp32 [128]
    k_norm: torch.Tensor      # fp32 [128]
    ffn_norm: torch.Tensor    # fp32 [hidden]


@dataclass
class DecodeWeights:
    cfg: DecodeConfig
    layers: list[LayerWeights]
    out_norm: torch.Tensor    # fp32 [hidden]
    output: torch.Tensor      # Q6_K [vocab rows of this rank, hidden]
    embedding: torch.Tensor   # Q6_K [vocab, hidden] (full; tied to the output projection)
    ffn_shard: RowShard
    vocab_shard: RowShard

    def nbytes(self) -> int:
        n = self.output.numel() + self.out_norm.numel() * 4
        if self.embedding.data_ptr() != self.output.data_ptr():
            n += self.embedding.numel()
        for lw in self.layers:
            n += sum(t.numel() * t.element_size() for t in vars(lw).values())
        return n


def generate_weights(cfg: DecodeConfig, device, world: int = 1, rank: int = 0) -> DecodeWeights:
    """Seeded random weights; with world > 1 only this rank's gate/up and
    output rows are kept (the same bytes every layout would give)."""
    cfg.validate()
    ffn_shard = RowShard(cfg.ffn, world, rank)
    vocab_shard = RowShard(cfg.vocab, world, rank)
    row_bytes = cfg.hidden // 256 * F.Q4K_BLOCK_BYTES
    layers = []
    for layer in range(cfg.layers):
        up = random_q4k(cfg.ffn, cfg.hidden, _seed(cfg, layer, 2), device)
        gate = random_q4k(cfg.ffn, cfg.hidden, _seed(cfg, layer, 3), device)
        if world > 1:
            up = up[ffn_shard.start * row_bytes:ffn_shard.stop * row_bytes].clone()
            gate = gate[ffn_shard.start * row_bytes:ffn_shard.stop * row_bytes].clone()
        layers.append(LayerWeights(
            qkv=random_q4k(cfg.qkv_rows, cfg.hidden, _seed(cfg, layer, 0), device),
            o=random_q4k(cfg.hidden, cfg.attn_width, _seed(cfg, layer, 1), device),
            up=up,
            gate=gate,
            down=random_q4k(cfg.hidden, cfg.ffn, _seed(cfg, layer, 4), device),
            attn_norm=random_gamma(cfg.hidden, _seed(cfg, layer, 5), device),
            q_norm=random_gamma(HEAD_DIM, _seed(cfg, layer, 6), device),
            k_norm=random_gamma(HEAD_DIM, _seed(cfg, layer, 7), device),
            ffn_norm=random_gamma(cfg.hidden, _seed(cfg, layer, 8), device),
        ))
    embedding = random_q6k(cfg.vocab, cfg.hidden, _seed(cfg, -1, 0), device)
    out_row = cfg.hidden // 256 * F.Q6K_BLOCK_BYTES
    output = embedding if world == 1 else \
        embedding[vocab_shard.start * out_row:vocab_shard.stop * out_row].clone()
    return DecodeWeights(cfg=cfg, layers=layers, out_norm=random_gamma(cfg.hidden, _seed(cfg, -1, 1), device),
                         output=output, embedding=embedding, ffn_shard=ffn_shard, vocab_shard=vocab_shard)


def _kv_values(cfg: DecodeConfig, layer: int, slot: int, device) -> torch.Tensor:
    g = _generator(torch.device(device), _seed(cfg, layer, slot))
    return torch.randn((cfg.kv_heads, cfg.context, HEAD_DIM), generator=g, device=device, dtype=torch.float32)


def generate_kv_cache(cfg: DecodeConfig, device) -> tuple[torch.Tensor, torch.Tensor]:
    """fp16 caches [layers, kv_heads, ctx_capacity, 128]: rows < context are
    N(0, 1) (seeded), the rest zero until decode appends them."""
    shape = (cfg.layers, cfg.kv_heads, cfg.ctx_capacity, HEAD_DIM)
    k = torch.zeros(shape, dtype=torch.float16, device=device)
    v = torch.zeros(shape, dtype=torch.float16, device=device)
    for layer in range(cfg.layers):
        for slot, cache in ((9, k), (10, v)):
            cache[layer, :, :cfg.context] = _kv_values(cfg, layer, slot, device).half()
    return k, v


@dataclass
class Q4_0Cache:
    """The Q4_0 KV cache of every layer as three planes (the layout of
    include/mllb200.h): GGML Q4_0 blocks, the KV type of the reference's
    llama.cpp contexts (integration/resident_decode.cpp:70)."""

    k_qs: torch.Tensor   # uint8 [layers, kv_heads, ctx, 64]: K nibbles
    v_qs: torch.Tensor   # uint8 [layers, kv_heads, ctx, 64]: V nibbles
    d: torch.Tensor      # fp16  [layers, kv_heads, ctx, 8]: K block scales, then V

    @classmethod
    def zeros(cls, layers: int, kv_heads: int, ctx: int, device) -> "Q4_0Cache":
        qs = (layers, kv_heads, ctx, HEAD_DIM // 2)
        return cls(torch.zeros(qs, dtype=torch.uint8, device=device), torch.zeros(qs, dtype=torch.uint8, device=device),
                   torch.zeros((layers, kv_heads, ctx, 8), dtype=torch.float16, device=device))

    @property
    def device(self) -> torch.device:
        return self.k_qs.device

    def layer(self, i: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        return self.k_qs[i], self.v_qs[i], self.d[i]

    def clone(self) -> "Q4_0Cache":
        return Q4_0Cache(self.k_qs.clone(), self.v_qs.clone(), self.d.clone())


def generate_kv_cache_q4_0(cfg: DecodeConfig, device) -> Q4_0Cache:
    """The Q4_0 cache of the same seeded N(0, 1) rows as generate_kv_cache
    (quantised on the device by mllb_kv_q4_0_store, as a prefill writes it)."""
    cache = Q4_0Cache.zeros(cfg.layers, cfg.kv_heads, cfg.ctx_capacity, device)
    if cfg.context == 0:
        return cache
    stream = torch.cuda.current_stream(torch.device(device)).cuda_stream
    for layer in range(cfg.layers):
        k, v = _kv_values(cfg, layer, 9, device), _kv_values(cfg, layer, 10, device)
        kq, vq, d = cache.layer(layer)
        check(lib().mllb_kv_q4_0_store(k.data_ptr(), v.data_ptr(), kq.data_ptr(), vq.data_ptr(), d.data_ptr(),
                                       cfg.kv_heads, cfg.ctx_capacity, 0, cfg.context, 0, stream), "kv_q4_0_store")
    return cache


def state_bytes(token: int, pos: int, steps: int = 0) -> bytes:
    """Host image of mllb_decode_state seeded to decode `token` at `pos`."""
    key = int(lib().mllb_token_key(token))
    return struct.pack("<qiii12x", key, pos, token, steps)


def parse_state(raw: bytes) -> dict:
    key, pos, token, steps = struct.unpack("<qiii12x", raw)
    return {"next_token": int(lib().mllb_key_token(key)), "pos": pos, "token": token, "steps": steps}


@dataclass
class _Buffers:
    hidden: torch.Tensor      # residual stream, two buffers (norms write the other one)
    q8_hidden: torch.Tensor
    qkv: torch.Tensor
    attn: torch.Tensor
    q8_attn: torch.Tensor
    o_out: torch.Tensor
    prod: torch.Tensor
    q8_prod: torch.Tensor
    down_out: torch.Tensor
    logits: torch.Tensor
    state: torch.Tensor
    tokens: torch.Tensor
    scratch: torch.Tensor
    extra: dict = field(default_factory=dict)


class Decoder:
    """One decode step as a chain of C-ABI launches on one stream.

    ``step()`` launches it eagerly; ``capture()`` records it once into a CUDA
    graph that ``generate()`` replays per token.  With ``group`` (a NCCL
    process group of ``world`` ranks) the gate/up and vocabulary matvecs are
    row-sharded as the module docstring describes.
    """

    def __init__(self, weights: DecodeWeights, k_cache, v_cache: torch.Tensor | None = None, *, pdl: bool = True,
                 fused: bool = False, group=None, gather: str = "peer", prefetch: bool = False, quant_tail: bool = True,
                 norm_tail: bool = False, gather_tail: bool = True):
        cfg = weights.cfg
        cfg.validate()
        self.cfg, self.w, self.k_cache, self.v_cache = cfg, weights, k_cache, v_cache
        # KV cache: fp16 K and V tensors, or one Q4_0Cache (v_cache None).
        self.kv = "q4_0" if isinstance(k_cache, Q4_0Cache) else "f16"
        self.device = k_cache.device
        self.flags = LAUNCH_PDL if pdl else 0
        self.group = group
        self.world = weights.ffn_shard.world
        if self.world > 1:
            if group is None:
                raise ValueError("a sharded decoder needs a process group")
            if weights.ffn_shard.per_rank % 32 or weights.ffn_shard.per_rank * self.world != cfg.ffn:
                raise ValueError("gate/up shards must be equal and a multiple of 32 rows")
        if self.kv == "q4_0":
            qs = (cfg.layers, cfg.kv_heads, cfg.ctx_capacity, HEAD_DIM // 2)
            if (v_cache is not None or k_cache.k_qs.shape != qs or k_cache.v_qs.shape != qs or
                    k_cache.d.shape != qs[:3] + (8,) or k_cache.d.dtype != torch.float16):
                raise ValueError("a Q4_0 cache comes alone, with planes [layers, kv_heads, ctx_capacity, 64 | 8]")
        else:
            if k_cache.shape != (cfg.layers, cfg.kv_heads, cfg.ctx_capacity, HEAD_DIM) or \
                    k_cache.dtype != torch.float16:
                raise ValueError("k_cache must be fp16 [layers, kv_heads, ctx_capacity, 128]")
            if v_cache is None or v_cache.shape != k_cache.shape or v_cache.dtype != torch.float16:
                raise ValueError("v_cache must match k_cache")
        dev = self.device
        f32 = lambda n: torch.zeros(n, dtype=torch.float32, device=dev)  # noqa: E731
        u8 = lambda n: torch.zeros(n, dtype=torch.uint8, device=dev)  # noqa: E731
        with torch.cuda.device(dev):
            scratch_n = int(lib().mllb_decode_attention_scratch(cfg.q_heads, cfg.kv_heads, cfg.ctx_capacity))
        if scratch_n < 0:
            raise ValueError(f"attention shape rejected: {lib().mllb_last_error().decode()}")
        ffn_local = weights.ffn_shard.local_rows
        self.b = _Buffers(
            hidden=torch.zeros((2, cfg.hidden), dtype=torch.float32, device=dev), q8_hidden=u8(cfg.hidden // 32 * 36), qkv=f32(cfg.qkv_rows),
            attn=f32(cfg.attn_width), q8_attn=u8(cfg.attn_width // 32 * 36),
            o_out=f32(cfg.hidden), prod=f32(ffn_local), q8_prod=u8(cfg.ffn // 32 * 36), down_out=f32(cfg.hidden),
            logits=f32(weights.vocab_shard.local_rows),
            state=u8(STATE_BYTES), tokens=torch.zeros(cfg.new_tokens, dtype=torch.int32, device=dev),
            scratch=torch.zeros(scratch_n, dtype=torch.float64, device=dev))
        if self.world > 1 and fused:
            self.b.extra["prod_full"] = torch.zeros(cfg.ffn, dtype=torch.float32, device=dev)
        # L2 prefetch of layer l + 1 (weights and KV rows) on a side stream
        # while layer l computes: the layers are latency-bound and leave most
        # of the HBM bandwidth idle, and one layer (57 MB + 17 MB) fits in L2.
        self.prefetch = prefetch
        self.side = torch.cuda.Stream(dev) if prefetch else None
        self.peer = None
        if self.world > 1 and not fused and gather == "peer":
            self.peer = self._setup_peer_gather()
        nb_h, nb_f = cfg.hidden // 256, cfg.ffn // 256
        # The in-kernel activations need streaming configurations for every
        # matvec they feed (otherwise the separate norm / quantise kernels run).
        self.fused = (fused and nb_h in (8, 10, 16) and nb_f in (8, 10, 16, 38)
                      and weights.vocab_shard.local_rows % 8 == 0)
        # On one GPU the gate/up writes the Q8_1 of its product itself (the
        # CTA that completes a 32-row group quantises it) instead of a
        # separate quantiser launch: 8 launches per layer instead of 9.
        self.quant_tail = (quant_tail and not self.fused and self.world == 1 and nb_h in (8, 10, 16)
                           and ffn_local % 32 == 0)
        # Sharded over GPUs with peer mappings: the gate/up launch also stores
        # the Q8_1 of its product slice into every rank's buffer and completes
        # once all ranks' slices have arrived (mllb_q4k_gate_up_q8_gather), in
        # place of the separate all-gather launch.
        self.gather_tail = (gather_tail and self.peer is not None and not self.fused and nb_h in (8, 10, 16)
                            and ffn_local % 32 == 0)
        if self.quant_tail or self.gather_tail:  # the groups (+ the CTAs' arrivals for the gather)
            self.b.extra["prod_counters"] = torch.zeros(ffn_local // 32 + 1, dtype=torch.int32, device=dev)
        # norm_tail: the O and down projections (hidden rows each) also do the
        # residual add + RMSNorm + Q8_1 that follows them (mllb_q4k_matvec_norm)
        # where a streaming configuration exists for their K: two launches
        # fewer per layer, but the grid-wide meeting in that epilogue costs
        # more than the separate 10-CTA norm launch, which the PDL chain
        # largely hides (36-layer A/B: 1779 vs 1680 us/token), so it is off by
        # default.  The first layer's norm and the final norm (which advances
        # the state) stay separate launches either way.
        team_k = (8, 10, 16, 38)
        self.norm_tail_o = norm_tail and not self.fused and cfg.attn_width // 256 in team_k
        self.norm_tail_down = norm_tail and not self.fused and cfg.ffn // 256 in team_k
        for name, on, k in (("norm_ws_o", self.norm_tail_o, cfg.attn_width),
                            ("norm_ws_down", self.norm_tail_down, cfg.ffn)):
            if on:
                need = int(lib().mllb_q4k_matvec_norm_workspace(cfg.hidden, k))
                if need < 0:
                    raise ValueError(f"norm epilogue rejected: {lib().mllb_last_error().decode()}")
                self.b.extra[name] = torch.zeros(need, dtype=torch.uint8, device=dev)
        self.graph = None

    # -- state ------------------------------------------------------------
    def reset(self, token: int, pos: int | None = None, stream=None) -> None:
        """Seed the state to decode `token` at `pos` (default: the first free KV row)."""
        pos = self.cfg.context if pos is None else pos
        host = torch.frombuffer(bytearray(state_bytes(token, pos)), dtype=torch.uint8)
        self.b.state.copy_(host, non_blocking=False)

    def read_state(self) -> dict:
        return parse_state(bytes(self.b.state.cpu().numpy().tobytes()))

    # -- one step -----------------------------------------------------------
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def step(self) -> None:
        """Launch one decode step on the current stream."""
        if self.fused:
            self._step_fused()
        else:
            self._step_unfused()

    def _step_fused(self) -> None:
        # Per layer: QKV (norm built in), attention (rope + append built in)
        # and its combine, O, gate/up (residual + norm built in), down (Q8_1
        # of the product built in): 6 launches.
        cfg, w, b, L = self.cfg, self.w, self.b, lib()
        s, fl = self._stream(), self.flags
        P = lambda t: t.data_ptr()  # noqa: E731
        state = P(b.state)
        h = [P(b.hidden[0]), P(b.hidden[1])]
        cur = 0
        check(L.mllb_decode_embed(P(w.embedding), cfg.vocab, cfg.hidden, state, P(b.tokens), cfg.new_tokens,
                                  h[cur], fl, s), "decode_embed")
        ffn_local = w.ffn_shard.local_rows
        for layer, lw in enumerate(w.layers):
            delta = None if layer == 0 else P(b.down_out)
            out = None if delta is None else h[1 - cur]
            act = ActF32(h[cur], delta, P(lw.attn_norm), out, cfg.eps, None)
            check(L.mllb_q4k_matvec_act(P(lw.qkv), act, P(b.qkv), cfg.qkv_rows, cfg.hidden, fl, s), "qkv")
            if out is not None:
                cur = 1 - cur
            self._attention(layer, lw, state, fl, s)
            check(L.mllb_q4k_matvec_ex(P(lw.o), P(b.q8_attn), P(b.o_out), cfg.hidden, cfg.attn_width, fl, s), "o")
            act = ActF32(h[cur], P(b.o_out), P(lw.ffn_norm), h[1 - cur], cfg.eps, None)
            check(L.mllb_q4k_gate_up_act(P(lw.up), P(lw.gate), act, None, None, P(b.prod), ffn_local, cfg.hidden,
                                         fl, s), "gate_up")
            cur = 1 - cur
            if self.world > 1:
                import torch.distributed as dist
                dist.all_gather_into_tensor(b.extra["prod_full"], b.prod, group=self.group)
                prod = P(b.extra["prod_full"])
            else:
                prod = P(b.prod)
            check(L.mllb_q4k_matvec_act(P(lw.down), ActF32(prod, None, None, None, 0.0, None), P(b.down_out),
                                        cfg.hidden, cfg.ffn, fl, s), "down")
        act = ActF32(h[cur], P(b.down_out), P(w.out_norm), h[1 - cur], cfg.eps, state)
        check(L.mllb_q6k_matvec_act(P(w.output), act, P(b.logits), w.vocab_shard.local_rows, cfg.hidden, fl, s),
              "logits")
        if self.world == 1:
            check(L.mllb_argmax_f32(P(b.logits), cfg.vocab, 0, state, fl, s), "argmax")
        else:
            self._reduce_argmax(s, fl)

    def _attention(self, layer: int, lw: LayerWeights, state: int, fl: int, s: int) -> None:
        """q/k norm + IMROPE, KV append at the state's position, attention and
        its combine (-> b.attn, b.q8_attn): two launches."""
        cfg, b, L = self.cfg, self.b, lib()
        P = lambda t: t.data_ptr()  # noqa: E731
        if self.kv == "q4_0":
            kq, vq, d = self.k_cache.layer(layer)
            check(L.mllb_decode_attention_qkv_q4_0(P(b.qkv), P(lw.q_norm), P(lw.k_norm), cfg.theta_scale, state,
                                                   P(kq), P(vq), P(d), P(b.scratch), b.scratch.numel(), P(b.attn),
                                                   P(b.q8_attn), cfg.q_heads, cfg.kv_heads, cfg.ctx_capacity, fl, s),
                  "attention (Q4_0 cache)")
        else:
            check(L.mllb_decode_attention_qkv(P(b.qkv), P(lw.q_norm), P(lw.k_norm), cfg.theta_scale, state,
                                              P(self.k_cache[layer]), P(self.v_cache[layer]), P(b.scratch),
                                              b.scratch.numel(), P(b.attn), P(b.q8_attn), cfg.q_heads, cfg.kv_heads,
                                              cfg.ctx_capacity, fl, s), "attention")

    def _prefetch_layer(self, layer: int) -> None:
        """Issue the L2 prefetch of `layer` on the side stream once the main
        stream's work so far has completed."""
        if not self.prefetch or layer >= self.cfg.layers:
            return
        main = torch.cuda.current_stream(self.device)
        self.side.wait_stream(main)
        lw, L, sp = self.w.layers[layer], lib(), self.side.cuda_stream
        kv = self.k_cache.layer(layer) if self.kv == "q4_0" else (self.k_cache[layer], self.v_cache[layer])
        for t in (lw.qkv, lw.o, lw.up, lw.gate, lw.down, *kv):
            check(L.mllb_prefetch_l2(t.data_ptr(), t.numel() * t.element_size(), sp), "prefetch")

    def _join_side(self) -> None:
        if self.prefetch:
            torch.cuda.current_stream(self.device).wait_stream(self.side)

    def _step_unfused(self) -> None:
        cfg, w, b, L = self.cfg, self.w, self.b, lib()
        s, fl = self._stream(), self.flags
        P = lambda t: t.data_ptr()  # noqa: E731
        state = P(b.state)
        h = [P(b.hidden[0]), P(b.hidden[1])]
        cur = 0
        check(L.mllb_decode_embed(P(w.embedding), cfg.vocab, cfg.hidden, state, P(b.tokens), cfg.new_tokens,
                                  h[cur], fl, s), "decode_embed")

        def norm(delta, gamma, what):
            # h[cur] + delta -> h[1 - cur]; the Q8_1 of its norm -> q8_hidden.
            nonlocal cur
            out = None if delta is None else h[1 - cur]
            check(L.mllb_rmsnorm_q8_1(h[cur], delta, out, P(gamma), cfg.eps, P(b.q8_hidden), cfg.hidden, 0, fl, s),
                  what)
            if out is not None:
                cur = 1 - cur

        def matvec_norm(weights, q8_in, k, gamma, ws, what):
            # h[cur] + W a -> h[1 - cur]; the Q8_1 of its norm -> q8_hidden.
            nonlocal cur
            check(L.mllb_q4k_matvec_norm(P(weights), q8_in, None, cfg.hidden, k, h[cur], h[1 - cur], P(gamma),
                                         cfg.eps, P(b.q8_hidden), P(ws), ws.numel(), fl, s), what)
            cur = 1 - cur

        ffn_local = w.ffn_shard.local_rows
        self._prefetch_layer(0)
        norm_pending = True  # this layer's attention norm still needs its own launch
        for layer, lw in enumerate(w.layers):
            self._prefetch_layer(layer + 1)
            if norm_pending:
                norm(None if layer == 0 else P(b.down_out), lw.attn_norm, "attn_norm")
            check(L.mllb_q4k_matvec_ex(P(lw.qkv), P(b.q8_hidden), P(b.qkv), cfg.qkv_rows, cfg.hidden, fl, s),
                  "qkv")
            self._attention(layer, lw, state, fl, s)
            if self.norm_tail_o:
                matvec_norm(lw.o, P(b.q8_attn), cfg.attn_width, lw.ffn_norm, b.extra["norm_ws_o"], "o + ffn_norm")
            else:
                check(L.mllb_q4k_matvec_ex(P(lw.o), P(b.q8_attn), P(b.o_out), cfg.hidden, cfg.attn_width, fl, s),
                      "o")
                norm(P(b.o_out), lw.ffn_norm, "ffn_norm")
            if self.quant_tail:
                check(L.mllb_q4k_gate_up_q8(P(lw.up), P(lw.gate), P(b.q8_hidden), None, None, P(b.prod),
                                            P(b.q8_prod), P(b.extra["prod_counters"]), ffn_local, cfg.hidden, fl, s),
                      "gate_up + Q8_1")
                q8_prod = P(b.q8_prod)
            elif self.gather_tail:
                half = layer % 2
                check(L.mllb_q4k_gate_up_q8_gather(P(lw.up), P(lw.gate), P(b.q8_hidden), None, None, P(b.prod),
                                                   P(b.extra["prod_counters"]), ffn_local, cfg.hidden,
                                                   self.peer["tables"][half], fl, s), "gate_up + Q8_1 gather")
                q8_prod = self.peer["buf"].data_ptr() + half * self.peer["half"]
            else:
                check(L.mllb_q4k_gate_up_ex(P(lw.up), P(lw.gate), P(b.q8_hidden), None, None, P(b.prod), ffn_local,
                                            cfg.hidden, fl, s), "gate_up")
                if self.world == 1:
                    check(L.mllb_q8_1_quantize_ex(P(b.prod), P(b.q8_prod), cfg.ffn, 0, fl, s), "quantize prod")
                    q8_prod = P(b.q8_prod)
                else:
                    q8_prod = self._gather_prod(s, fl, layer)
            if self.norm_tail_down and layer + 1 < cfg.layers:
                matvec_norm(lw.down, q8_prod, cfg.ffn, w.layers[layer + 1].attn_norm, b.extra["norm_ws_down"],
                            "down + attn_norm")
                norm_pending = False
            else:
                check(L.mllb_q4k_matvec_ex(P(lw.down), q8_prod, P(b.down_out), cfg.hidden, cfg.ffn, fl, s), "down")
                norm_pending = True
        check(L.mllb_decode_final_norm(h[cur], P(b.down_out), h[1 - cur], P(w.out_norm), cfg.eps,
                                       P(b.q8_hidden), cfg.hidden, state, fl, s), "final_norm")
        check(L.mllb_q6k_matvec_ex(P(w.output), P(b.q8_hidden), P(b.logits), w.vocab_shard.local_rows, cfg.hidden,
                                   fl, s), "logits")
        if self.world == 1:
            check(L.mllb_argmax_f32(P(b.logits), cfg.vocab, 0, state, fl, s), "argmax")
        else:
            self._reduce_argmax(s, fl)
        self._join_side()

    def launches_per_step(self) -> int:
        """Kernels of this library one step launches (collectives not counted)."""
        # embedding; per layer (fused) QKV, attention split + combine, O,
        # gate/up, down or (unfused) those plus two norms and the quantiser;
        # final norm (unfused) and logits; argmax.
        L = self.cfg.layers
        if self.fused:
            return 1 + L * 6 + 1 + 1
        per_layer = 6 if (self.quant_tail or self.gather_tail) else 7  # QKV, attention x 2, O, gate/up (+ quantiser / gather), down
        norms = (0 if self.norm_tail_o else L) + (1 if self.norm_tail_down else L)
        return 1 + L * per_layer + norms + 1 + 1 + 1       # embed, ..., final norm, logits, argmax

    # -- sharded pieces -----------------------------------------------------
    def _setup_peer_gather(self):
        """Symmetric buffer [half 0 | half 1 | counters[world] | gather count]
        mapped on every rank; layer l gathers into half l % 2, so a rank can
        run at most one gather ahead of a peer's down projection without
        overwriting what it reads.  None if symmetric memory is unavailable."""
        import os

        import torch.distributed as dist
        try:
            import torch.distributed._symmetric_memory as symm_mem
        except ImportError:
            return None
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        world, rank = self.world, self.w.ffn_shard.rank
        half = -(-(self.cfg.ffn // 32 * 36) // 256) * 256
        flags_off, count_off = 2 * half, 2 * half + 256
        try:
            buf = symm_mem.empty(count_off + 256, dtype=torch.uint8, device=self.device)
            buf.zero_()
            handle = symm_mem.rendezvous(buf, self.group)
            ptrs = [int(p) for p in handle.buffer_ptrs]
        except Exception:  # noqa: BLE001 -- no peer mappings here: NCCL all-gather instead
            return None
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every counter is zero before anyone signals
        tables = []
        for h in range(2):
            t = PeerGather()
            t.rank, t.world = rank, world
            for r in range(world):
                t.buffers[r] = ptrs[r] + h * half
                t.flags[r] = ptrs[r] + flags_off
            t.count = ptrs[rank] + count_off
            tables.append(t)
        return {"buf": buf, "handle": handle, "tables": tables, "half": half}

    def _gather_prod(self, s: int, fl: int, layer: int = 0) -> int:
        """Q8_1 of the full SwiGLU product on every rank; returns its address."""
        if self.peer is not None:
            h = layer % 2
            check(lib().mllb_q8_1_quantize_allgather(self.b.prod.data_ptr(), self.w.ffn_shard.per_rank,
                                                     self.peer["tables"][h], fl, s), "peer all-gather")
            return self.peer["buf"].data_ptr() + h * self.peer["half"]
        self._gather_prod_nccl(s, fl)
        return self.b.q8_prod.data_ptr()

    def _gather_prod_nccl(self, s: int, fl: int) -> None:
        import torch.distributed as dist

        b, L, shard = self.b, lib(), self.w.ffn_shard
        local = b.extra.get("q8_prod_local")
        if local is None:
            local = b.extra["q8_prod_local"] = torch.zeros(shard.per_rank // 32 * 36, dtype=torch.uint8,
                                                           device=self.device)
        check(L.mllb_q8_1_quantize_ex(b.prod.data_ptr(), local.data_ptr(), shard.per_rank, 0, fl, s),
              "quantize prod shard")
        dist.all_gather_into_tensor(b.q8_prod, local, group=self.group)

    def _reduce_argmax(self, s: int, fl: int) -> None:
        import torch.distributed as dist

        b, L, shard = self.b, lib(), self.w.vocab_shard
        # The final norm reset the key in the state; each rank folds in its
        # rows, then MAX over ranks leaves the global (value, lowest index).
        key = b.state[:8].view(torch.int64)
        check(L.mllb_argmax_f32(b.logits.data_ptr(), shard.local_rows, shard.start, key.data_ptr(), fl, s),
              "argmax shard")
        dist.all_reduce(key, op=dist.ReduceOp.MAX, group=self.group)

    # -- graphs -------------------------------------------------------------
    def capture(self) -> torch.cuda.CUDAGraph:
        """Record one step into a CUDA graph on the current (non-default)
        stream.  One eager step runs first, so that every kernel's launch
        attributes are set outside the capture; it leaves the KV row at the
        state's position written, which the first replay rewrites, and the
        state is restored afterwards."""
        stream = torch.cuda.current_stream(self.device)
        if stream == torch.cuda.default_stream(self.device):
            raise RuntimeError("capture on a non-default stream (torch.cuda.stream(...))")
        saved = self.b.state.clone()
        self.step()
        self.b.state.copy_(saved)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            self.step()
        self.graph = g
        return g

    def replay(self) -> None:
        if self.graph is None:
            raise RuntimeError("capture() first")
        self.graph.replay()

    def generate(self, token: int, n: int, pos: int | None = None) -> list[int]:
        """Decode n tokens greedily after `token` (public API; H2D of the seed
        state, D2H of the tokens).  Uses the captured graph when there is one."""
        if n > self.cfg.new_tokens:
            raise ValueError("n exceeds the KV capacity reserved for new tokens")
        self.reset(token, pos)
        for _ in range(n):
            self.replay() if self.graph is not None else self.step()
        st = self.read_state()
        seen = self.b.tokens[:n].cpu().tolist()
        return seen[1:] + [st["next_token"]]


def main(argv=None) -> None:
    """python -m mojo_llm_lab_b200.decode: run greedy decode steps of the
    synthetic stack on the current GPU and print the tokens and µs/token."""
    import argparse
    import time

    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--graph", action="store_true", help="replay one captured CUDA graph per token")
    ap.add_argument("--fused", action="store_true", help="activations built inside the matvecs")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--kv", choices=["f16", "q4_0"], default="f16", help="KV cache type")
    args = ap.parse_args(argv)
    cfg = DecodeConfig(layers=args.layers)
    w = generate_weights(cfg, "cuda")
    k, v = generate_kv_cache(cfg, "cuda") if args.kv == "f16" else (generate_kv_cache_q4_0(cfg, "cuda"), None)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dec = Decoder(w, k, v, pdl=not args.no_pdl, fused=args.fused)
        dec.reset(17)
        if args.graph:
            dec.capture()
            dec.reset(17)
        stream.synchronize()
        t0 = time.perf_counter()
        tokens = dec.generate(17, args.steps)
        el = time.perf_counter() - t0
    print(f"tokens {tokens}  {el / args.steps * 1e6:.1f} us/token (host clock, {'graph' if args.graph else 'eager'})")


if __name__ == "__main__":
    main()
