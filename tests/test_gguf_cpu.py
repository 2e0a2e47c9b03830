"""GGUF v3 files: the writer and the memory-mapped reader agree byte for byte
(metadata of every kind, tensors of every quantised type the kernels take,
padding to the alignment), malformed files are refused, and a Qwen3-style
decode stack survives a save / load round trip with llama.cpp's tensor names."""
import struct

import numpy as np
import pytest
import torch

from mojo_llm_lab_b200 import decode as D
from mojo_llm_lab_b200 import gguf


def test_round_trip_metadata_and_tensors(tmp_path):
    rng = np.random.default_rng(0)
    q4 = rng.integers(0, 256, 3 * 2560 // 256 * 144, dtype=np.uint8)
    q6 = rng.integers(0, 256, 5 * 512 // 256 * 210, dtype=np.uint8)
    f32 = rng.standard_normal(96).astype(np.float32)
    meta = {"general.architecture": "qwen3", "qwen3.block_count": np.uint32(36), "x.i64": -5, "x.f": 0.5,
            "x.flag": True, "x.arr": np.arange(7, dtype=np.int32), "x.name": "tokenizer ü"}
    path = tmp_path / "t.gguf"
    gguf.write_gguf(path, meta, [("a.weight", gguf.GGML_Q4_K, (2560, 3), q4.tobytes()),
                                 ("b.weight", gguf.GGML_Q6_K, (512, 5), q6.tobytes()),
                                 ("c", gguf.GGML_F32, (96,), f32.tobytes())], alignment=64)
    g = gguf.GgufFile(path)
    assert g.version == 3 and g.alignment == 64 and g.data_offset % 64 == 0
    assert g.metadata["qwen3.block_count"] == 36 and g.metadata["x.i64"] == -5 and g.metadata["x.flag"] is True
    assert g.metadata["x.f"] == 0.5 and g.metadata["x.name"] == "tokenizer ü"
    assert np.array_equal(g.metadata["x.arr"], np.arange(7))
    assert g.tensors["a.weight"].dims == (2560, 3) and g.tensors["a.weight"].rows == 3
    assert np.array_equal(g.raw("a.weight"), q4) and np.array_equal(g.raw("b.weight"), q6)
    assert np.array_equal(g.raw("c").view(np.float32), f32)
    assert all(t.offset % 64 == 0 for t in g.tensors.values())


def test_refuses_malformed_files(tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + bytes(20))
    with pytest.raises(ValueError):
        gguf.GgufFile(bad)
    path = tmp_path / "short.gguf"
    gguf.write_gguf(path, {}, [("a", gguf.GGML_Q4_K, (256, 2), bytes(288))])
    data = path.read_bytes()
    path.write_bytes(data[:-10])                       # tensor data cut short
    with pytest.raises(ValueError):
        gguf.GgufFile(path)
    with pytest.raises(ValueError):                    # bytes do not match the dimensions
        gguf.write_gguf(tmp_path / "x.gguf", {}, [("a", gguf.GGML_Q4_K, (256, 2), bytes(100))])
    ver = bytearray(data)
    ver[4:8] = struct.pack("<I", 9)
    (tmp_path / "v.gguf").write_bytes(bytes(ver))
    with pytest.raises(ValueError):
        gguf.GgufFile(tmp_path / "v.gguf")


def test_decode_stack_round_trip(tmp_path):
    cfg = D.DecodeConfig(layers=2, hidden=512, q_heads=4, kv_heads=2, ffn=768, vocab=300, context=8, new_tokens=4)
    w = D.generate_weights(cfg, "cpu")
    path = tmp_path / "stack.gguf"
    gguf.save_decode_weights(path, w)
    g = gguf.GgufFile(path)
    assert "blk.1.attn_q.weight" in g.tensors and g.tensors["blk.0.ffn_down.weight"].dims == (768, 512)
    back = gguf.load_decode_weights(path, "cpu", context=8, new_tokens=4)
    for f in ("layers", "hidden", "q_heads", "kv_heads", "ffn", "vocab", "eps", "theta_bits"):
        assert getattr(back.cfg, f) == getattr(cfg, f), f
    assert torch.equal(back.embedding, w.embedding) and torch.equal(back.out_norm, w.out_norm)
    for a, b in zip(back.layers, w.layers):
        for f in ("qkv", "o", "up", "gate", "down", "attn_norm", "q_norm", "k_norm", "ffn_norm"):
            assert torch.equal(getattr(a, f), getattr(b, f)), f


def test_decode_load_refuses_other_quantisations(tmp_path):
    cfg = D.DecodeConfig(layers=1, hidden=512, q_heads=4, kv_heads=2, ffn=768, vocab=300, context=8, new_tokens=4)
    w = D.generate_weights(cfg, "cpu")
    path = tmp_path / "stack.gguf"
    gguf.save_decode_weights(path, w)
    g = gguf.GgufFile(path)
    tensors = []
    for name, t in g.tensors.items():
        gtype = t.ggml_type
        data = bytes(g.raw(name))
        if name == "blk.0.ffn_up.weight":          # relabel as Q5_K with the matching byte count
            gtype, data = gguf.GGML_Q5_K, bytes(t.dims[1] * t.dims[0] // 256 * 176)
        tensors.append((name, gtype, t.dims, data))
    gguf.write_gguf(tmp_path / "q5.gguf", dict(g.metadata), tensors)
    with pytest.raises(ValueError, match="Q5_K"):
        gguf.load_decode_weights(tmp_path / "q5.gguf", "cpu", context=8, new_tokens=4)
