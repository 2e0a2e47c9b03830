"""Decode-step kernels on the GPU against the oracle.

Every value these kernels hand on is fp64 inside and rounded once, so the
fp32 outputs are compared bit for bit where the oracle rounds at the same
place (embedding, residual, Q8_1 bytes, fp16 cache rows, argmax) and within
the 1e-5 + 1e-5 |ref| tolerance (with a bit-exact majority) elsewhere.
"""
import struct

import numpy as np
import pytest
import torch

from gpu_util import assert_within_tolerance, dev
from mojo_llm_lab_b200 import decode as D
from mojo_llm_lab_b200 import fixtures as fx
from mojo_llm_lab_b200 import formats as F
from mojo_llm_lab_b200 import ops

pytestmark = pytest.mark.gpu

INT64_MIN = -(1 << 63)


def state_tensor(token=0, pos=0, steps=0, key=None):
    raw = bytearray(D.state_bytes(token, pos, steps))
    if key is not None:
        raw[0:8] = struct.pack("<q", key)
    return torch.frombuffer(raw, dtype=torch.uint8).cuda()


def read_state(t):
    return D.parse_state(bytes(t.cpu().numpy().tobytes()))


# ------------------------------------------------------------------ embed

@pytest.mark.parametrize("vocab,k,token", [(1000, 2560, 0), (1000, 2560, 999), (151936, 2560, 151935),
                                           (77, 512, 31)])
def test_embed_bit_exact(orc, vocab, k, token):
    w = fx.seeded_q6k_matrix(vocab, k, seed=vocab + token)
    state = state_tensor(token=token, steps=3)
    hidden = torch.full((k,), 7.0, device="cuda")
    tokens = torch.full((8,), -1, dtype=torch.int32, device="cuda")
    ops.decode_embed(dev(w), vocab, state, hidden, tokens)
    ref = orc.embed_q6k(w, k, token)
    assert np.array_equal(hidden.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    st = read_state(state)
    assert st["token"] == token and st["steps"] == 3
    assert tokens.cpu().tolist() == [-1, -1, -1, token, -1, -1, -1, -1]
    assert ops.device_error() == 0


def test_embed_bad_key_reports_and_uses_row_zero(orc):
    vocab, k = 50, 256
    w = fx.seeded_q6k_matrix(vocab, k, seed=5)
    for key in (ops.token_key(vocab), INT64_MIN):
        state = state_tensor(key=key)
        hidden = torch.zeros(k, device="cuda")
        ops.decode_embed(dev(w), vocab, state, hidden)
        assert ops.device_error(clear=True) & 8
        assert np.array_equal(hidden.cpu().numpy(), orc.embed_q6k(w, k, 0))
        assert read_state(state)["token"] == 0


# --------------------------------------------------------- rmsnorm -> Q8_1

@pytest.mark.parametrize("k,with_delta,scale", [(2560, True, 1.0), (2560, False, 1.0), (4096, True, 1e4),
                                                (32, True, 1e-3), (9728, False, 30.0), (32768, True, 1.0)])
@pytest.mark.parametrize("in_place", [True, False])
def test_rmsnorm_q8_1_bit_exact(orc, k, with_delta, scale, in_place):
    rng = np.random.default_rng(k)
    x = (rng.standard_normal(k) * scale).astype(np.float32)
    delta = (rng.standard_normal(k) * scale).astype(np.float32) if with_delta else None
    gamma = rng.uniform(0.5, 1.5, k).astype(np.float32)
    xd = dev(x)
    out = xd if in_place else torch.full((k,), 9.0, device="cuda")
    q8 = ops.rmsnorm_q8_1(xd, dev(gamma), None if delta is None else dev(delta), x_out=out)
    h_ref, q8_ref = orc.rmsnorm_q8_1(x, delta, gamma)
    assert np.array_equal(out.cpu().numpy(), h_ref)
    assert np.array_equal(q8.cpu().numpy(), q8_ref)
    if not in_place:
        assert np.array_equal(xd.cpu().numpy(), x)


def test_rmsnorm_rejects_partial_overlap():
    buf = torch.zeros(4096 + 32, device="cuda")
    g = torch.ones(4096, device="cuda")
    with pytest.raises(Exception):
        ops.rmsnorm_q8_1(buf[:4096], g, x_out=buf[32:])


def test_rmsnorm_zero_input_and_rejects_bad_k():
    k = 64
    q8 = ops.rmsnorm_q8_1(torch.zeros(k, device="cuda"), torch.ones(k, device="cuda"))
    assert not q8.cpu().numpy().any()  # amax 0 -> d 0, q 0, s 0
    with pytest.raises(Exception):
        ops.rmsnorm_q8_1(torch.zeros(48, device="cuda"), torch.ones(48, device="cuda"))


def test_final_norm_advances_state(orc):
    k = 2560
    rng = np.random.default_rng(3)
    x = rng.standard_normal(k).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, k).astype(np.float32)
    state = state_tensor(token=5, pos=4096, steps=7)
    q8 = ops.decode_final_norm(dev(x), dev(gamma), state)
    assert np.array_equal(q8.cpu().numpy(), orc.rmsnorm_q8_1(x, None, gamma)[1])
    st = read_state(state)
    assert st["pos"] == 4097 and st["steps"] == 8 and st["next_token"] == -1


# ------------------------------------------------- q/k rope + KV append

@pytest.mark.parametrize("hq,hkv,pos,ctx", [(32, 8, 4096, 4224), (32, 8, 0, 16), (8, 8, 32767, 32768),
                                            (16, 2, 7, 9)])
def test_qk_rope_append(orc, hq, hkv, pos, ctx):
    rng = np.random.default_rng(pos + hq)
    qkv = (rng.standard_normal((hq + 2 * hkv) * 128) * 40).astype(np.float32)
    qg = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    kg = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    kc = torch.zeros((hkv, ctx, 128), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    state = state_tensor(pos=pos)
    theta = F.theta_scale_f32()
    q_out = ops.decode_qk_rope_append(dev(qkv), dev(qg), dev(kg), state, kc, vc, hq, hkv, theta)
    q_ref, k_ref, v_ref = orc.qk_rope_append(qkv, hq, hkv, qg, kg, pos, theta)
    got_q = q_out.cpu().numpy()
    assert_within_tolerance(got_q, q_ref, "q heads")
    assert (got_q.view(np.uint32) == q_ref.view(np.uint32)).mean() > 0.99
    kh = kc.cpu().numpy().view(np.uint16)
    vh = vc.cpu().numpy().view(np.uint16)
    k_match = (kh[:, pos, :].reshape(-1) == k_ref).mean()
    assert k_match > 0.999, k_match
    assert np.array_equal(vh[:, pos, :].reshape(-1), v_ref)
    others = np.ones(ctx, dtype=bool)
    others[pos] = False
    assert not kh[:, others].any() and not vh[:, others].any()
    assert ops.device_error() == 0


def test_qk_rope_append_rejects_overflow():
    hq, hkv, ctx = 4, 2, 8
    kc = torch.zeros((hkv, ctx, 128), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    qkv = torch.ones((hq + 2 * hkv) * 128, device="cuda")
    g = torch.ones(128, device="cuda")
    ops.decode_qk_rope_append(qkv, g, g, state_tensor(pos=ctx), kc, vc, hq, hkv)
    assert ops.device_error(clear=True) & 16
    assert not kc.any() and not vc.any()


# ---------------------------------------------------------------- attention

def random_cache(hkv, ctx, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    k = (rng.standard_normal((hkv, ctx, 128)) * scale).astype(np.float16)
    v = (rng.standard_normal((hkv, ctx, 128)) * scale).astype(np.float16)
    return k, v


@pytest.mark.parametrize("hq,hkv,ctx,pos", [
    (32, 8, 4224, 4096), (32, 8, 4224, 4223), (32, 8, 4224, 0), (32, 8, 4224, 15), (32, 8, 4224, 16),
    (32, 8, 4224, 287), (8, 8, 300, 299), (8, 4, 1000, 517), (64, 8, 2048, 2047), (4, 4, 5000, 4999),
    (16, 2, 64, 63),
    # past one wave of the default shape: the long-context shape
    (32, 8, 8192, 8000), (32, 8, 33000, 32999), (8, 8, 20000, 19999), (16, 4, 12000, 11999)])
def test_attention_against_oracle(orc, hq, hkv, ctx, pos):
    k, v = random_cache(hkv, ctx, seed=ctx + pos)
    rng = np.random.default_rng(pos)
    q = rng.standard_normal(hq * 128).astype(np.float32)
    state = state_tensor(pos=pos)
    out, q8 = ops.decode_attention(dev(q), dev(k), dev(v), state)
    ref = orc.attention(q, k.view(np.uint16), v.view(np.uint16), pos + 1, hq, hkv)
    got = out.cpu().numpy()
    assert_within_tolerance(got, ref, f"attention pos={pos}")
    exact = (got.view(np.uint32) == ref.view(np.uint32)).mean()
    assert exact > 0.999, exact
    assert np.array_equal(q8.cpu().numpy(), np.frombuffer(orc.quantize_q8_1(got), dtype=np.uint8))
    assert ops.device_error() == 0


@pytest.mark.parametrize("hq,hkv,ctx,pos", [
    (32, 8, 4224, 4096), (32, 8, 4224, 0), (32, 8, 4224, 63), (32, 8, 4224, 64), (32, 8, 4224, 4223),
    (8, 8, 300, 299), (8, 4, 1000, 517), (64, 8, 2048, 1000), (4, 4, 5000, 4999), (16, 2, 64, 63),
    (32, 8, 8192, 8191), (32, 8, 33000, 20000), (32, 8, 33000, 64)])
def test_fused_rope_append_attention(orc, hq, hkv, ctx, pos):
    """decode_attention_qkv == qk_rope_append + attention, cache rows included."""
    k, v = random_cache(hkv, ctx, seed=ctx * 3 + pos)
    rng = np.random.default_rng(pos + 11)
    qkv = (rng.standard_normal((hq + 2 * hkv) * 128) * 30).astype(np.float32)
    qg = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    kg = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    kd, vd = dev(k), dev(v)
    theta = F.theta_scale_f32()
    out, q8 = ops.decode_attention_qkv(dev(qkv), dev(qg), dev(kg), state_tensor(pos=pos), kd, vd, hq, theta)
    q_ref, k_row, v_row = orc.qk_rope_append(qkv, hq, hkv, qg, kg, pos, theta)
    kh, vh = k.view(np.uint16).copy(), v.view(np.uint16).copy()
    kh[:, pos, :] = k_row.reshape(hkv, 128)
    vh[:, pos, :] = v_row.reshape(hkv, 128)
    ref = orc.attention(q_ref, kh, vh, pos + 1, hq, hkv)
    got = out.cpu().numpy()
    assert_within_tolerance(got, ref, f"fused attention pos={pos}")
    assert (got.view(np.uint32) == ref.view(np.uint32)).mean() > 0.999
    assert np.array_equal(q8.cpu().numpy(), np.frombuffer(orc.quantize_q8_1(got), dtype=np.uint8))
    got_k = kd.cpu().numpy().view(np.uint16)
    assert (got_k[:, pos] == kh[:, pos]).mean() > 0.999
    assert np.array_equal(vd.cpu().numpy().view(np.uint16), vh)
    others = np.ones(ctx, dtype=bool)
    others[pos] = False
    assert np.array_equal(got_k[:, others], kh[:, others])
    assert ops.device_error() == 0


def test_fused_attention_overflow_appends_nothing():
    hq, hkv, ctx = 8, 4, 40
    k, v = random_cache(hkv, ctx, seed=2)
    kd, vd = dev(k), dev(v)
    qkv = torch.ones((hq + 2 * hkv) * 128, device="cuda")
    g = torch.ones(128, device="cuda")
    out, _ = ops.decode_attention_qkv(qkv, g, g, state_tensor(pos=ctx), kd, vd, hq)
    assert ops.device_error(clear=True) & 16
    assert np.array_equal(kd.cpu().numpy(), k) and np.array_equal(vd.cpu().numpy(), v)
    assert torch.isfinite(out).all()


def test_attention_peaked_and_subnormal_values(orc):
    """One key dominates the softmax; fp16 subnormals and zeros in the cache."""
    hq, hkv, ctx, pos = 8, 2, 600, 599
    k, v = random_cache(hkv, ctx, seed=9)
    k[:, 123, :] = np.float16(3.0)
    v[:, ::7, ::3] = np.float16(0.0)
    v[:, 1::5, 1::3] = np.float16(3e-6)  # subnormal half
    q = np.full(hq * 128, 2.0, dtype=np.float32)
    out, _ = ops.decode_attention(dev(q), dev(k), dev(v), state_tensor(pos=pos))
    ref = orc.attention(q, k.view(np.uint16), v.view(np.uint16), pos + 1, hq, hkv)
    assert_within_tolerance(out.cpu().numpy(), ref, "peaked attention")


def test_attention_pdl_chain_equals_plain(orc):
    hq, hkv, ctx, pos = 32, 8, 4224, 4100
    k, v = random_cache(hkv, ctx, seed=1)
    q = np.random.default_rng(2).standard_normal(hq * 128).astype(np.float32)
    a = ops.decode_attention(dev(q), dev(k), dev(v), state_tensor(pos=pos))[0].cpu()
    kd, vd, qd, st = dev(k), dev(v), dev(q), state_tensor(pos=pos)
    for _ in range(3):
        b = ops.decode_attention(qd, kd, vd, st, pdl=True)[0]
    assert torch.equal(a, b.cpu())


# ------------------------------------------------------------------ argmax

def test_argmax_first_maximum_and_offsets():
    x = torch.randn(151936, device="cuda")
    x[1000] = 50.0
    x[90000] = 50.0
    key = torch.full((1,), INT64_MIN, dtype=torch.int64, device="cuda")
    ops.argmax_key(x, key)
    assert ops.key_token(int(key.item())) == 1000
    # Shards fold into one key in any order; the lower global index wins ties.
    key.fill_(INT64_MIN)
    ops.argmax_key(x[75968:], key, index_offset=75968)
    ops.argmax_key(x[:75968], key, index_offset=0)
    assert ops.key_token(int(key.item())) == 1000


@pytest.mark.parametrize("n", [1, 7, 256, 257, 18992, 151936])
def test_argmax_matches_oracle(orc, n):
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32) - 5.0
    key = torch.full((1,), INT64_MIN, dtype=torch.int64, device="cuda")
    ops.argmax_key(dev(x), key)
    assert ops.key_token(int(key.item())) == orc.argmax(x)


def test_argmax_negative_values_and_signed_zero():
    x = torch.tensor([-3.0, -0.0, 0.0, -1.0], device="cuda")
    key = torch.full((1,), INT64_MIN, dtype=torch.int64, device="cuda")
    ops.argmax_key(x, key)
    assert ops.key_token(int(key.item())) == 2  # +0 sorts above -0
    x = torch.tensor([-3.0, -2.0, -2.5], device="cuda")
    key.fill_(INT64_MIN)
    ops.argmax_key(x, key)
    assert ops.key_token(int(key.item())) == 1
