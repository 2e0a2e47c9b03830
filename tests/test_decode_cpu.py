"""Host logic of the synthetic decode and the oracle's decode ops (CPU only)."""
import numpy as np
import pytest
import torch

from mojo_llm_lab_b200 import decode as D
from oracle import decode as OD


def test_default_config_is_the_36_layer_stack():
    cfg = D.DecodeConfig()
    cfg.validate()
    assert (cfg.layers, cfg.hidden, cfg.q_heads, cfg.kv_heads, cfg.ffn, cfg.vocab) == (36, 2560, 32, 8, 9728, 151936)
    assert cfg.qkv_rows == 6144 and cfg.attn_width == 4096 and cfg.ctx_capacity == 4224
    assert cfg.q4k_bytes() == 2_043_740_160
    assert cfg.q6k_bytes() == 319_065_600
    assert cfg.kv_bytes_read(4096) == 603_979_776
    assert cfg.bytes_per_token(4096) == 2_966_785_536
    assert abs(cfg.theta_scale - np.array([0x3F492C27], np.uint32).view(np.float32)[0]) == 0


@pytest.mark.parametrize("bad", [dict(hidden=2500), dict(q_heads=12, kv_heads=8), dict(q_heads=48, kv_heads=3),
                                 dict(q_heads=1, kv_heads=1), dict(layers=0), dict(new_tokens=0)])
def test_config_validation(bad):
    with pytest.raises(ValueError):
        D.DecodeConfig(**bad).validate()


def test_state_image_round_trip():
    raw = D.state_bytes(151935, 4096, 3)
    assert len(raw) == D.STATE_BYTES
    st = D.parse_state(raw)
    assert st == {"next_token": 151935, "pos": 4096, "token": 151935, "steps": 3}
    assert D.parse_state(b"\x00" * 7 + b"\x80" + b"\x00" * 24)["next_token"] == -1


def test_random_blocks_follow_the_fixture_distributions():
    q4 = D.random_q4k(64, 2560, seed=1, device="cpu").view(-1, 144).numpy()
    d = np.abs(q4[:, 0:2].copy().view(np.float16).astype(np.float64))
    dmin = np.abs(q4[:, 2:4].copy().view(np.float16).astype(np.float64))
    assert d.min() >= 0.000999 and d.max() <= 0.01001 and dmin.min() >= 0 and dmin.max() <= 0.005001
    signs = q4[:, [1, 3]] >> 7
    assert 0.4 < signs.mean() < 0.6  # random signs of d and dmin (zero-mean rows)
    plain = D.random_q4k(64, 2560, seed=1, device="cpu", signed_scales=False).view(-1, 144).numpy()
    assert not (plain[:, [1, 3]] >> 7).any()
    q6 = D.random_q6k(64, 2560, seed=2, device="cpu").view(-1, 210).numpy()
    sc = q6[:, 192:208].view(np.int8)
    assert sc.min() >= -32 and sc.max() <= 31
    assert np.array_equal(D.random_q4k(4, 256, 9, "cpu").numpy(), D.random_q4k(4, 256, 9, "cpu").numpy())


def test_sharded_weights_are_row_slices_of_the_full_matrices():
    cfg = D.DecodeConfig(layers=1, hidden=256, q_heads=2, kv_heads=1, ffn=512, vocab=96, context=4, new_tokens=2)
    full = D.generate_weights(cfg, "cpu")
    row4, row6 = 144, 210
    for rank in range(4):
        part = D.generate_weights(cfg, "cpu", world=4, rank=rank)
        f, v = part.ffn_shard, part.vocab_shard
        assert torch.equal(part.layers[0].up, full.layers[0].up[f.start * row4:f.stop * row4])
        assert torch.equal(part.layers[0].gate, full.layers[0].gate[f.start * row4:f.stop * row4])
        assert torch.equal(part.output, full.output[v.start * row6:v.stop * row6])
        assert torch.equal(part.embedding, full.embedding)


def tiny_model():
    cfg = D.DecodeConfig(layers=2, hidden=256, q_heads=2, kv_heads=1, ffn=512, vocab=96, context=5, new_tokens=3,
                         seed=11)
    w = D.generate_weights(cfg, "cpu")
    k, v = D.generate_kv_cache(cfg, "cpu")
    return cfg, OD.host_model(w), k.numpy().view(np.uint16).copy(), v.numpy().view(np.uint16).copy()


def test_oracle_decode_step_is_deterministic_and_appends_kv(orc):
    cfg, host, kh, vh = tiny_model()
    k2, v2 = kh.copy(), vh.copy()
    logits, nxt = OD.reference_step(host, kh, vh, 7, cfg.context)
    again, nxt2 = OD.reference_step(host, k2, v2, 7, cfg.context)
    assert np.array_equal(logits, again) and nxt == nxt2 == int(np.argmax(logits))
    assert np.isfinite(logits).all() and logits.shape == (cfg.vocab,)
    assert kh[:, :, cfg.context].any() and vh[:, :, cfg.context].any()
    assert not kh[:, :, cfg.context + 1:].any()


def test_oracle_attention_against_numpy(orc):
    rng = np.random.default_rng(4)
    hq, hkv, ctx, n = 4, 2, 40, 33
    k = rng.standard_normal((hkv, ctx, 128)).astype(np.float16)
    v = rng.standard_normal((hkv, ctx, 128)).astype(np.float16)
    q = rng.standard_normal(hq * 128).astype(np.float32)
    got = orc.attention(q, k.view(np.uint16), v.view(np.uint16), n, hq, hkv)
    for h in range(hq):
        j = h // (hq // hkv)
        s = (k[j, :n].astype(np.float64) @ q[h * 128:(h + 1) * 128].astype(np.float64)) / np.sqrt(128.0)
        p = np.exp(s - s.max())
        ref = (p @ v[j, :n].astype(np.float64)) / p.sum()
        np.testing.assert_allclose(got[h * 128:(h + 1) * 128], ref, rtol=1e-6, atol=1e-7)


def test_oracle_rmsnorm_q8_1_against_numpy(orc):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(256).astype(np.float32)
    d = rng.standard_normal(256).astype(np.float32)
    g = rng.uniform(0.5, 1.5, 256).astype(np.float32)
    h, q8 = orc.rmsnorm_q8_1(x, d, g)
    assert np.array_equal(h, x + d)
    hd = h.astype(np.float64)
    y = (hd / np.sqrt((hd * hd).mean() + 1e-6) * g).astype(np.float32)
    assert q8.tobytes() == orc.quantize_q8_1(y)


def test_logit_agreement_criterion():
    ref = np.array([1.0, 100.0, -3.0], dtype=np.float32)
    ok = OD.logit_agreement(ref, ref + np.float32(1e-4))
    assert ok["violations"] == 0 and ok["top_match"]
    bad = OD.logit_agreement(ref, np.array([1.0, 100.0, -2.99], dtype=np.float32))
    assert bad["violations"] == 1
    assert not OD.logit_agreement(ref, np.array([200.0, 100.0, -3.0], dtype=np.float32))["top_match"]


def test_kv_bytes_of_both_cache_types():
    cfg = D.DecodeConfig()
    assert cfg.kv_bytes_read(4096, "f16") == 603_979_776
    assert cfg.kv_bytes_read(4096, "q4_0") == 36 * 8 * 4096 * 144
    assert cfg.bytes_per_token(4096, "q4_0") == cfg.q4k_bytes() + cfg.q6k_bytes() + 36 * 8 * 4096 * 144


def test_oracle_step_over_a_q4_0_cache(orc):
    """The whole-step oracle with a Q4_0 cache (tiny stack, CPU): it appends
    the token's K / V rows to the planes by the GGML rule, leaves the other
    rows alone, and its logits stay close to the fp16-cache step over the
    same rows (the cache's 4-bit error is the only difference)."""
    cfg = D.DecodeConfig(layers=2, hidden=256, q_heads=2, kv_heads=1, ffn=256, vocab=64, context=40,
                         new_tokens=2, seed=5)
    w = D.generate_weights(cfg, "cpu")
    host = OD.host_model(w)
    k16, v16 = D.generate_kv_cache(cfg, "cpu")
    kh, vh = k16.numpy().view(np.uint16).copy(), v16.numpy().view(np.uint16).copy()
    qs = (cfg.layers, cfg.kv_heads, cfg.ctx_capacity, 64)
    planes = (np.zeros(qs, np.uint8), np.zeros(qs, np.uint8), np.zeros(qs[:3] + (8,), np.uint16))
    for layer in range(cfg.layers):
        for slot, p, lo in ((9, planes[0], 0), (10, planes[1], 4)):
            rows = D._kv_values(cfg, layer, slot, "cpu").numpy()
            p[layer, :, :cfg.context], planes[2][layer, :, :cfg.context, lo:lo + 4] = orc.kv_q4_0_rows(rows)
    before = [p.copy() for p in planes]
    ref16, tok16 = OD.reference_step(host, kh, vh, 7, cfg.context)
    ref4, tok4 = OD.reference_step(host, None, None, 7, cfg.context, q4_0=planes)
    assert np.all(np.isfinite(ref4))
    for b, p in zip(before, planes):
        assert np.array_equal(b[:, :, :cfg.context], p[:, :, :cfg.context])   # prefilled rows untouched
        assert np.array_equal(b[:, :, cfg.context + 1:], p[:, :, cfg.context + 1:])
        assert p[:, :, cfg.context].any()                                     # the token's row appended
    # 4-bit K / V (about 1/16 of each block's range per value) over random
    # weights move these logits by ~12 % (relative L2); a wrong row or plane
    # would decorrelate them entirely.
    rel = np.linalg.norm(ref4.astype(np.float64) - ref16) / np.linalg.norm(ref16.astype(np.float64))
    assert rel < 0.25, rel
    assert np.corrcoef(ref4, ref16)[0, 1] > 0.95
