"""GGUF tensor files: read (memory-mapped), write, and load a Qwen3-style
decode stack for this library's kernels.

The format is GGML's public GGUF v3 layout: "GGUF", version, tensor count,
metadata key/value count, the metadata (typed values, length-prefixed
strings, arrays), the tensor infos (name, dimensions with ne[0] the
contiguous one, ggml type, offset into the data section), padding to
``general.alignment`` (32 by default), then the tensor data.  The quantised
blocks are GGML's (Q4_K 144 B, Q5_K 176 B, Q6_K 210 B per 256 values), which
are exactly the bytes the kernels here take, so a tensor is handed to the GPU
as its raw bytes.

The reference runs real models through llama.cpp's own loader; this module
is the "on-disk GGUF tensor import for real weights" that lets the decode
stack here run them (``load_decode_weights``: llama.cpp's tensor names for a
Qwen3 model, the separate Q/K/V projections fused into one QKV matrix).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = b"GGUF"
VERSION = 3
DEFAULT_ALIGNMENT = 32

# ggml_type ids of the public GGML enum and their (values, bytes) per block.
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_BF16 = 0, 1, 8, 12, 13, 14, 30
BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 9: (32, 36),
         10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292),
         30: (1, 2)}
TYPE_NAMES = {0: "F32", 1: "F16", 2: "Q4_0", 3: "Q4_1", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0", 9: "Q8_1", 10: "Q2_K",
              11: "Q3_K", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 15: "Q8_K", 30: "BF16"}

# metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
           _U64: "<Q", _I64: "<q", _F64: "<d"}


@dataclass
class TensorInfo:
    name: str
    dims: tuple          # ne[0] first (the contiguous dimension)
    ggml_type: int
    offset: int          # into the data section

    @property
    def nbytes(self) -> int:
        if self.ggml_type not in BLOCK:
            raise ValueError(f"{self.name}: unsupported ggml type {self.ggml_type}")
        per, size = BLOCK[self.ggml_type]
        n = int(np.prod(self.dims, dtype=np.int64))
        if self.dims[0] % per:
            raise ValueError(f"{self.name}: row of {self.dims[0]} values is not whole blocks of {per}")
        return n // per * size

    @property
    def rows(self) -> int:
        return int(np.prod(self.dims[1:], dtype=np.int64)) if len(self.dims) > 1 else 1


class _Reader:
    def __init__(self, buf: memoryview):
        self.buf, self.pos = buf, 0

    def take(self, fmt: str):
        v = struct.unpack_from(fmt, self.buf, self.pos)[0]
        self.pos += struct.calcsize(fmt)
        return v

    def string(self) -> str:
        n = self.take("<Q")
        if n > len(self.buf) - self.pos:
            raise ValueError("truncated GGUF string")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8")
        self.pos += n
        return s

    def value(self, vtype: int):
        if vtype in _SCALAR:
            return self.take(_SCALAR[vtype])
        if vtype == _STR:
            return self.string()
        if vtype == _ARR:
            etype, n = self.take("<I"), self.take("<Q")
            if etype in _SCALAR and etype != _BOOL:
                fmt = _SCALAR[etype]
                size = struct.calcsize(fmt)
                arr = np.frombuffer(self.buf, dtype=np.dtype(fmt), count=n, offset=self.pos).copy()
                self.pos += n * size
                return arr
            return [self.value(etype) for _ in range(n)]
        raise ValueError(f"unknown GGUF metadata type {vtype}")


class GgufFile:
    """A GGUF file mapped read-only: ``metadata`` (dict), ``tensors`` (name ->
    TensorInfo), ``raw(name)`` (the tensor's bytes as a uint8 array view)."""

    def __init__(self, path):
        self.path = Path(path)
        self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        r = _Reader(memoryview(self._map))
        if bytes(self._map[:4]) != MAGIC:
            raise ValueError(f"{self.path}: not a GGUF file")
        r.pos = 4
        self.version = r.take("<I")
        if self.version not in (2, 3):
            raise ValueError(f"{self.path}: GGUF version {self.version} not supported")
        n_tensors, n_kv = r.take("<Q"), r.take("<Q")
        self.metadata = {}
        for _ in range(n_kv):
            key = r.string()
            self.metadata[key] = r.value(r.take("<I"))
        self.tensors = {}
        for _ in range(n_tensors):
            name = r.string()
            nd = r.take("<I")
            dims = tuple(r.take("<Q") for _ in range(nd))
            self.tensors[name] = TensorInfo(name, dims, r.take("<I"), r.take("<Q"))
        self.alignment = int(self.metadata.get("general.alignment", DEFAULT_ALIGNMENT))
        self.data_offset = (r.pos + self.alignment - 1) // self.alignment * self.alignment
        for t in self.tensors.values():
            if self.data_offset + t.offset + t.nbytes > len(self._map):
                raise ValueError(f"{self.path}: tensor {t.name} runs past the end of the file")

    def raw(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        start = self.data_offset + t.offset
        return self._map[start:start + t.nbytes]


def write_gguf(path, metadata: dict, tensors: list, alignment: int = DEFAULT_ALIGNMENT) -> None:
    """Write a GGUF v3 file.  metadata values: int (stored as int64 unless the
    key's value is a numpy scalar of another type), float (float32), str,
    bool, or a numpy array (array of its element type).  tensors: (name,
    ggml_type, dims with ne[0] first, bytes)."""
    def enc_str(s: str) -> bytes:
        b = s.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    def enc_value(v) -> bytes:
        if isinstance(v, bool):
            return struct.pack("<I?", _BOOL, v)
        if isinstance(v, np.integer):
            kinds = {np.dtype(np.uint8): _U8, np.dtype(np.int8): _I8, np.dtype(np.uint16): _U16,
                     np.dtype(np.int16): _I16, np.dtype(np.uint32): _U32, np.dtype(np.int32): _I32,
                     np.dtype(np.uint64): _U64, np.dtype(np.int64): _I64}
            vt = kinds[np.asarray(v).dtype]
            return struct.pack("<I", vt) + struct.pack(_SCALAR[vt], int(v))
        if isinstance(v, int):
            return struct.pack("<Iq", _I64, v)
        if isinstance(v, (float, np.floating)):
            return struct.pack("<If", _F32, float(v))
        if isinstance(v, str):
            return struct.pack("<I", _STR) + enc_str(v)
        if isinstance(v, np.ndarray):
            codes = {np.dtype(np.uint8): _U8, np.dtype(np.int8): _I8, np.dtype(np.int32): _I32,
                     np.dtype(np.uint32): _U32, np.dtype(np.float32): _F32, np.dtype(np.int64): _I64,
                     np.dtype(np.float64): _F64}
            et = codes[v.dtype]
            return struct.pack("<IIQ", _ARR, et, v.size) + v.astype(v.dtype.newbyteorder("<")).tobytes()
        raise TypeError(f"unsupported metadata value {v!r}")

    meta = dict(metadata)
    if alignment != DEFAULT_ALIGNMENT:
        meta["general.alignment"] = np.uint32(alignment)
    head = bytearray(MAGIC + struct.pack("<IQQ", VERSION, len(tensors), len(meta)))
    for k, v in meta.items():
        head += enc_str(k) + enc_value(v)
    offset = 0
    blobs = []
    for name, gtype, dims, data in tensors:
        info = TensorInfo(name, tuple(int(d) for d in dims), int(gtype), offset)
        data = bytes(data)
        if len(data) != info.nbytes:
            raise ValueError(f"{name}: {len(data)} bytes, the dimensions need {info.nbytes}")
        head += enc_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", int(d)) for d in dims)
        head += struct.pack("<IQ", int(gtype), offset)
        blobs.append((offset, data))
        offset = (offset + len(data) + alignment - 1) // alignment * alignment
    pad = (-len(head)) % alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * pad)
        pos = 0
        for off, data in blobs:
            f.write(b"\0" * (off - pos))
            f.write(data)
            pos = off + len(data)


# ------------------------------------------------------------ decode stack

def _arch_key(meta: dict, name: str):
    arch = meta.get("general.architecture", "qwen3")
    return meta[f"{arch}.{name}"]


def decode_config(g: GgufFile, context: int = 0, new_tokens: int = 128):
    """A DecodeConfig from a Qwen3-style GGUF's metadata and tensor shapes."""
    from .decode import HEAD_DIM, DecodeConfig
    meta = g.metadata
    heads = int(_arch_key(meta, "attention.head_count"))
    head_dim = int(meta.get(f"{meta.get('general.architecture', 'qwen3')}.attention.key_length", HEAD_DIM))
    if head_dim != HEAD_DIM:
        raise ValueError(f"head dimension {head_dim}: the kernels here take {HEAD_DIM}")
    base = float(meta.get(f"{meta.get('general.architecture', 'qwen3')}.rope.freq_base", 10000.0))
    theta = np.float32(base ** (-2.0 / HEAD_DIM))
    return DecodeConfig(
        layers=int(_arch_key(meta, "block_count")), hidden=int(_arch_key(meta, "embedding_length")),
        q_heads=heads, kv_heads=int(_arch_key(meta, "attention.head_count_kv")),
        ffn=int(_arch_key(meta, "feed_forward_length")), vocab=int(g.tensors["token_embd.weight"].dims[1]),
        context=context, new_tokens=new_tokens,
        # GGUF stores eps as float32; its shortest decimal (e.g. 1e-06) is the value the model was given
        eps=float(str(np.float32(meta.get(f"{meta.get('general.architecture', 'qwen3')}.attention.layer_norm_rms_epsilon",
                                          1e-6)))),
        theta_bits=int(np.array([theta], dtype=np.float32).view(np.uint32)[0]))


def load_decode_weights(path, device, context: int = 0, new_tokens: int = 128):
    """Load a Qwen3-style GGUF (llama.cpp tensor names) into DecodeWeights:
    Q4_K attention and FFN matrices (Q, K, V fused into one QKV matrix in
    that row order), Q6_K token embedding / output (tied when the file has no
    ``output.weight``), fp32 norms.  Other quantisations raise ValueError."""
    import torch

    from .decode import HEAD_DIM, DecodeWeights, LayerWeights
    from .shard import RowShard
    g = GgufFile(path)
    cfg = decode_config(g, context, new_tokens)
    cfg.validate()

    def raw(name, gtype, dims):
        t = g.tensors.get(name)
        if t is None:
            raise ValueError(f"{path}: tensor {name} missing")
        if t.ggml_type != gtype:
            raise ValueError(f"{name}: {TYPE_NAMES.get(t.ggml_type, t.ggml_type)}, the kernels here take "
                             f"{TYPE_NAMES[gtype]}")
        if tuple(t.dims) != tuple(dims):
            raise ValueError(f"{name}: dimensions {t.dims}, expected {tuple(dims)}")
        return torch.from_numpy(np.array(g.raw(name))).to(device)

    def f32(name, n):
        return raw(name, GGML_F32, (n,)).view(torch.float32)

    layers = []
    for i in range(cfg.layers):
        p = f"blk.{i}."
        q = raw(p + "attn_q.weight", GGML_Q4_K, (cfg.hidden, cfg.q_heads * HEAD_DIM))
        k = raw(p + "attn_k.weight", GGML_Q4_K, (cfg.hidden, cfg.kv_heads * HEAD_DIM))
        v = raw(p + "attn_v.weight", GGML_Q4_K, (cfg.hidden, cfg.kv_heads * HEAD_DIM))
        layers.append(LayerWeights(
            qkv=torch.cat([q, k, v]),
            o=raw(p + "attn_output.weight", GGML_Q4_K, (cfg.attn_width, cfg.hidden)),
            up=raw(p + "ffn_up.weight", GGML_Q4_K, (cfg.hidden, cfg.ffn)),
            gate=raw(p + "ffn_gate.weight", GGML_Q4_K, (cfg.hidden, cfg.ffn)),
            down=raw(p + "ffn_down.weight", GGML_Q4_K, (cfg.ffn, cfg.hidden)),
            attn_norm=f32(p + "attn_norm.weight", cfg.hidden),
            q_norm=f32(p + "attn_q_norm.weight", HEAD_DIM),
            k_norm=f32(p + "attn_k_norm.weight", HEAD_DIM),
            ffn_norm=f32(p + "ffn_norm.weight", cfg.hidden)))
    embedding = raw("token_embd.weight", GGML_Q6_K, (cfg.hidden, cfg.vocab))
    output = raw("output.weight", GGML_Q6_K, (cfg.hidden, cfg.vocab)) if "output.weight" in g.tensors else embedding
    return DecodeWeights(cfg=cfg, layers=layers, out_norm=f32("output_norm.weight", cfg.hidden), output=output,
                         embedding=embedding, ffn_shard=RowShard(cfg.ffn, 1, 0), vocab_shard=RowShard(cfg.vocab, 1, 0))


def save_decode_weights(path, weights, arch: str = "qwen3") -> None:
    """Write DecodeWeights (one GPU's full stack) as a Qwen3-style GGUF with
    llama.cpp's tensor names -- the inverse of load_decode_weights."""
    from .decode import HEAD_DIM
    import math
    cfg = weights.cfg
    if weights.ffn_shard.world != 1:
        raise ValueError("save the unsharded weights")
    # rope.freq_base such that base^(-2/128) rounds to the config's fp32 theta scale
    freq_base = math.exp(-(HEAD_DIM / 2) * math.log(cfg.theta_scale))
    host = lambda t: t.detach().cpu().contiguous().view(-1).numpy().view(np.uint8).tobytes()  # noqa: E731
    meta = {"general.architecture": arch, f"{arch}.block_count": np.uint32(cfg.layers),
            f"{arch}.embedding_length": np.uint32(cfg.hidden), f"{arch}.feed_forward_length": np.uint32(cfg.ffn),
            f"{arch}.attention.head_count": np.uint32(cfg.q_heads),
            f"{arch}.attention.head_count_kv": np.uint32(cfg.kv_heads),
            f"{arch}.attention.key_length": np.uint32(HEAD_DIM), f"{arch}.rope.freq_base": float(freq_base),
            f"{arch}.attention.layer_norm_rms_epsilon": float(cfg.eps)}
    q_rows, kv_rows = cfg.q_heads * HEAD_DIM, cfg.kv_heads * HEAD_DIM
    rb = cfg.hidden // 256 * 144
    tensors = [("token_embd.weight", GGML_Q6_K, (cfg.hidden, cfg.vocab), host(weights.embedding)),
               ("output_norm.weight", GGML_F32, (cfg.hidden,), host(weights.out_norm))]
    if weights.output.data_ptr() != weights.embedding.data_ptr():
        tensors.append(("output.weight", GGML_Q6_K, (cfg.hidden, cfg.vocab), host(weights.output)))
    for i, lw in enumerate(weights.layers):
        p = f"blk.{i}."
        qkv = host(lw.qkv)
        tensors += [
            (p + "attn_q.weight", GGML_Q4_K, (cfg.hidden, q_rows), qkv[:q_rows * rb]),
            (p + "attn_k.weight", GGML_Q4_K, (cfg.hidden, kv_rows), qkv[q_rows * rb:(q_rows + kv_rows) * rb]),
            (p + "attn_v.weight", GGML_Q4_K, (cfg.hidden, kv_rows), qkv[(q_rows + kv_rows) * rb:]),
            (p + "attn_output.weight", GGML_Q4_K, (cfg.attn_width, cfg.hidden), host(lw.o)),
            (p + "ffn_up.weight", GGML_Q4_K, (cfg.hidden, cfg.ffn), host(lw.up)),
            (p + "ffn_gate.weight", GGML_Q4_K, (cfg.hidden, cfg.ffn), host(lw.gate)),
            (p + "ffn_down.weight", GGML_Q4_K, (cfg.ffn, cfg.hidden), host(lw.down)),
            (p + "attn_norm.weight", GGML_F32, (cfg.hidden,), host(lw.attn_norm)),
            (p + "attn_q_norm.weight", GGML_F32, (HEAD_DIM,), host(lw.q_norm)),
            (p + "attn_k_norm.weight", GGML_F32, (HEAD_DIM,), host(lw.k_norm)),
            (p + "ffn_norm.weight", GGML_F32, (cfg.hidden,), host(lw.ffn_norm))]
    write_gguf(path, meta, tensors)
