"""Whole decode steps of the synthetic Qwen3-style stack against the oracle.

The acceptance criterion is the reference's decode check: every logit within
atol 1e-4 + rtol 1e-5 of the reference and the same top-1 token at every
position (integration/logit_validation.h:14,76-80).  Because every kernel
rounds once from fp64, the logits are expected to agree bit for bit, so the
tests also require a bit-exact majority.
"""
import numpy as np
import pytest
import torch

from mojo_llm_lab_b200 import decode as D
from mojo_llm_lab_b200 import ops
from oracle import decode as OD

pytestmark = pytest.mark.gpu

SMALL = D.DecodeConfig(layers=2, vocab=4096, context=300, new_tokens=6)
ODD = D.DecodeConfig(layers=3, hidden=2048, q_heads=8, kv_heads=4, ffn=4096, vocab=1000, context=37, new_tokens=5,
                     seed=7)


def build(cfg):
    w = D.generate_weights(cfg, "cuda")
    k, v = D.generate_kv_cache(cfg, "cuda")
    return w, k, v


def host_cache(t):
    return t.cpu().numpy().view(np.uint16).copy()


def run_against_oracle(cfg, steps, token=17, graph=False, mode="quant_tail"):
    """mode: "quant_tail" (the default Decoder), "separate" (a separate Q8_1
    launch after gate/up), "norm_tail" (the default plus the residual norms
    built into the O and down projections) or "fused"."""
    w, k, v = build(cfg)
    host = OD.host_model(w)
    kh, vh = host_cache(k), host_cache(v)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dec = D.Decoder(w, k, v, fused=mode == "fused", quant_tail=mode in ("quant_tail", "norm_tail"),
                        norm_tail=mode == "norm_tail")
        assert dec.fused == (mode == "fused")
        assert dec.quant_tail == (mode in ("quant_tail", "norm_tail"))
        if mode == "norm_tail":
            assert dec.norm_tail_down and dec.norm_tail_o == (cfg.attn_width // 256 in (8, 10, 16, 38))
        dec.reset(token)
        if graph:
            dec.capture()
        pos = cfg.context
        for _ in range(steps):
            dec.replay() if graph else dec.step()
            stream.synchronize()
            got = dec.b.logits.cpu().numpy()
            ref, ref_next = OD.reference_step(host, kh, vh, token, pos)
            agree = OD.logit_agreement(ref, got)
            assert agree["violations"] == 0, agree
            assert agree["top_match"], agree
            assert agree["bit_exact"] > 0.99 * agree["values"], agree
            st = dec.read_state()
            assert st["next_token"] == ref_next and st["pos"] == pos + 1 and st["token"] == token
            token, pos = ref_next, pos + 1
    kd, vd = host_cache(k), host_cache(v)
    assert (kd[:, :, cfg.context:pos] == kh[:, :, cfg.context:pos]).mean() > 0.999
    assert np.array_equal(kd[:, :, :cfg.context], kh[:, :, :cfg.context])
    assert (vd[:, :, cfg.context:pos] == vh[:, :, cfg.context:pos]).mean() > 0.999
    assert ops.device_error() == 0


@pytest.mark.parametrize("cfg", [SMALL, ODD], ids=["qwen-2layer", "odd-shapes"])
@pytest.mark.parametrize("mode", ["quant_tail", "separate", "norm_tail", "fused"])
def test_decode_steps_match_oracle(orc, cfg, mode):
    run_against_oracle(cfg, steps=3, mode=mode)


def test_graph_replay_matches_oracle(orc):
    run_against_oracle(SMALL, steps=4, graph=True)


def test_graph_and_eager_generate_identical_tokens():
    w, k, v = build(SMALL)
    k2, v2 = k.clone(), v.clone()
    eager = D.Decoder(w, k, v)
    tokens_eager = eager.generate(123, 5)
    logits_eager = eager.b.logits.clone()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        graphed = D.Decoder(w, k2, v2)
        graphed.reset(123)
        graphed.capture()
        tokens_graph = graphed.generate(123, 5)
    assert tokens_graph == tokens_eager
    assert torch.equal(graphed.b.logits, logits_eager)
    assert torch.equal(k, k2) and torch.equal(v, v2)


def test_full_size_decode_matches_oracle(orc):
    """The 36-layer, 151936-vocab stack at context 4096: two greedy steps."""
    run_against_oracle(D.DecodeConfig(), steps=2)


def test_gguf_loaded_stack_decodes_identically(tmp_path):
    """The stack written as a GGUF file (llama.cpp's tensor names) and read
    back decodes the same tokens with the same logits."""
    from mojo_llm_lab_b200 import gguf
    w, k, v = build(SMALL)
    path = tmp_path / "small.gguf"
    gguf.save_decode_weights(path, w)
    w2 = gguf.load_decode_weights(path, "cuda", context=SMALL.context, new_tokens=SMALL.new_tokens)
    k2, v2 = k.clone(), v.clone()
    a = D.Decoder(w, k, v)
    b = D.Decoder(w2, k2, v2)
    assert a.generate(123, 4) == b.generate(123, 4)
    assert torch.equal(a.b.logits, b.b.logits)


def run_q4_0_against_oracle(cfg, steps, token=17, graph=False, mode="quant_tail"):
    """The same steps over the Q4_0 KV cache (the reference's KV type)."""
    w = D.generate_weights(cfg, "cuda")
    cache = D.generate_kv_cache_q4_0(cfg, "cuda")
    host = OD.host_model(w)
    planes = (cache.k_qs.cpu().numpy().copy(), cache.v_qs.cpu().numpy().copy(),
              cache.d.cpu().numpy().view(np.uint16).copy())
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dec = D.Decoder(w, cache, fused=mode == "fused", quant_tail=mode == "quant_tail")
        assert dec.kv == "q4_0"
        dec.reset(token)
        if graph:
            dec.capture()
        pos = cfg.context
        for _ in range(steps):
            dec.replay() if graph else dec.step()
            stream.synchronize()
            got = dec.b.logits.cpu().numpy()
            ref, ref_next = OD.reference_step(host, None, None, token, pos, q4_0=planes)
            agree = OD.logit_agreement(ref, got)
            assert agree["violations"] == 0, agree
            assert agree["top_match"], agree
            assert agree["bit_exact"] > 0.99 * agree["values"], agree
            st = dec.read_state()
            assert st["next_token"] == ref_next and st["pos"] == pos + 1
            token, pos = ref_next, pos + 1
    got_planes = (cache.k_qs.cpu().numpy(), cache.v_qs.cpu().numpy(), cache.d.cpu().numpy().view(np.uint16))
    for got_p, ref_p in zip(got_planes, planes):
        assert np.array_equal(got_p[:, :, :cfg.context], ref_p[:, :, :cfg.context])
        assert (got_p[:, :, cfg.context:pos] == ref_p[:, :, cfg.context:pos]).mean() > 0.99
    assert ops.device_error() == 0


def test_q4_0_cache_holds_the_quantised_fp16_rows(orc):
    """generate_kv_cache_q4_0 quantises the same seeded rows generate_kv_cache holds."""
    cfg = D.DecodeConfig(layers=1, vocab=1000, context=40, new_tokens=2)
    cache = D.generate_kv_cache_q4_0(cfg, "cuda")
    k16, _ = D.generate_kv_cache(cfg, "cuda")
    deq = orc.dequantize_q4_0(np.concatenate(
        [cache.d[0, :, :cfg.context, :4].cpu().numpy().view(np.uint8).reshape(-1, 4, 2),
         cache.k_qs[0, :, :cfg.context].cpu().numpy().reshape(-1, 4, 16)], axis=-1).reshape(-1))
    k = k16[0, :, :cfg.context].float().cpu().numpy().reshape(-1)
    assert np.abs(deq - k).max() < 0.5  # N(0, 1) rows: |d| <= ~0.6, error <= |d|


@pytest.mark.parametrize("cfg", [SMALL, ODD], ids=["qwen-2layer", "odd-shapes"])
@pytest.mark.parametrize("mode", ["quant_tail", "fused"])
def test_decode_steps_q4_0_cache_match_oracle(orc, cfg, mode):
    run_q4_0_against_oracle(cfg, steps=3, mode=mode)


def test_graph_replay_q4_0_cache_matches_oracle(orc):
    run_q4_0_against_oracle(SMALL, steps=3, graph=True)


def test_full_size_decode_q4_0_cache_matches_oracle(orc):
    """36 layers, 151936 vocabulary, context 4096, Q4_0 cache: two steps."""
    run_q4_0_against_oracle(D.DecodeConfig(), steps=2)
