"""Q4_0 KV cache on the GPU against the oracle.

The cache store is bit-exact with GGML's quantize_row_q4_0 rule (the oracle);
attention over the Q4_0 planes is fp64 inside and rounded once, so its fp32
outputs meet 1e-5 + 1e-5 |ref| with a bit-exact majority, and its Q8_1 bytes
equal the oracle's quantisation of the GPU's own fp32 output.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_within_tolerance, dev
from mojo_llm_lab_b200 import decode as D
from mojo_llm_lab_b200 import formats as F
from mojo_llm_lab_b200 import ops
from test_kv_q4_0_cpu import edge_blocks

pytestmark = pytest.mark.gpu


def state_tensor(pos):
    return torch.frombuffer(bytearray(D.state_bytes(0, pos)), dtype=torch.uint8).cuda()


def empty_planes(hkv, ctx):
    return (torch.zeros((hkv, ctx, 64), dtype=torch.uint8, device="cuda"),
            torch.zeros((hkv, ctx, 64), dtype=torch.uint8, device="cuda"),
            torch.zeros((hkv, ctx, 8), dtype=torch.float16, device="cuda"))


def host_planes(orc, k, v):
    """Oracle planes of fp32 K / V rows [hkv, ctx, 128]."""
    kq, kd = orc.kv_q4_0_rows(k)
    vq, vd = orc.kv_q4_0_rows(v)
    return kq, vq, np.ascontiguousarray(np.concatenate([kd, vd], axis=-1))


def random_rows(hkv, ctx, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    return tuple((rng.standard_normal((hkv, ctx, 128)) * scale).astype(np.float32) for _ in range(2))


def planes_np(kq, vq, d):
    return kq.cpu().numpy(), vq.cpu().numpy(), d.cpu().numpy().view(np.uint16)


# ------------------------------------------------------------------ store

@pytest.mark.parametrize("hkv,ctx,row0,rows", [(8, 4224, 0, 4096), (2, 50, 13, 37), (1, 8, 7, 1), (3, 300, 0, 300)])
def test_store_bit_exact(orc, hkv, ctx, row0, rows):
    k, v = random_rows(hkv, rows, seed=ctx + row0)
    kq, vq, d = empty_planes(hkv, ctx)
    ops.kv_q4_0_store(dev(k), dev(v), kq, vq, d, row0=row0)
    ref_kq, ref_vq, ref_d = host_planes(orc, k, v)
    got_kq, got_vq, got_d = planes_np(kq, vq, d)
    sl = slice(row0, row0 + rows)
    assert np.array_equal(got_kq[:, sl], ref_kq)
    assert np.array_equal(got_vq[:, sl], ref_vq)
    assert np.array_equal(got_d[:, sl], ref_d)
    outside = np.ones(ctx, dtype=bool)
    outside[sl] = False
    assert not got_kq[:, outside].any() and not got_vq[:, outside].any() and not got_d[:, outside].any()


def test_store_edge_blocks_bit_exact(orc):
    """Ties in magnitude, zeros, -0.0, the clamp at 15, tiny and huge blocks."""
    blocks = edge_blocks()
    rows = np.concatenate(blocks + blocks[:4]).reshape(1, -1, 128).astype(np.float32)  # 16 blocks -> 4 rows
    v = -rows[:, ::-1].copy()
    kq, vq, d = empty_planes(1, rows.shape[1])
    ops.kv_q4_0_store(dev(rows), dev(v), kq, vq, d)
    ref = host_planes(orc, rows, v)
    for got, want in zip(planes_np(kq, vq, d), ref):
        assert np.array_equal(got, want)


def test_store_rejects_bad_rows():
    kq, vq, d = empty_planes(2, 10)
    k = torch.zeros((2, 4, 128), device="cuda")
    with pytest.raises(Exception):
        ops.kv_q4_0_store(k, k, kq, vq, d, row0=7)   # rows 7..10 past ctx
    with pytest.raises(ValueError):
        ops.kv_q4_0_store(k[:1], k[:1], kq, vq, d)


# -------------------------------------------------------------- attention

@pytest.mark.parametrize("hq,hkv,ctx,pos", [
    (32, 8, 4224, 4096), (32, 8, 4224, 4223), (32, 8, 4224, 0), (32, 8, 4224, 15), (32, 8, 4224, 16),
    (32, 8, 4224, 287), (8, 8, 300, 299), (8, 4, 1000, 517), (64, 8, 2048, 2047), (4, 4, 5000, 4999),
    (16, 2, 64, 63),
    # past one wave of the default shape: the long-context shape
    (32, 8, 8192, 8000), (32, 8, 33000, 32999), (8, 8, 20000, 19999), (16, 4, 12000, 11999)])
def test_attention_q4_0_against_oracle(orc, hq, hkv, ctx, pos):
    k, v = random_rows(hkv, ctx, seed=ctx + pos)
    kq, vq, d = host_planes(orc, k, v)
    rng = np.random.default_rng(pos)
    q = rng.standard_normal(hq * 128).astype(np.float32)
    out, q8 = ops.decode_attention_q4_0(dev(q), dev(kq), dev(vq), dev(d).view(torch.float16), state_tensor(pos))
    ref = orc.attention_q4_0(q, kq, vq, d, pos + 1, hq, hkv)
    got = out.cpu().numpy()
    assert_within_tolerance(got, ref, f"Q4_0 attention pos={pos}")
    assert (got.view(np.uint32) == ref.view(np.uint32)).mean() > 0.999
    assert np.array_equal(q8.cpu().numpy(), np.frombuffer(orc.quantize_q8_1(got), dtype=np.uint8))
    assert ops.device_error() == 0


@pytest.mark.parametrize("hq,hkv,ctx,pos", [
    (32, 8, 4224, 4096), (32, 8, 4224, 0), (32, 8, 4224, 63), (32, 8, 4224, 64), (32, 8, 4224, 4223),
    (8, 8, 300, 299), (8, 4, 1000, 517), (64, 8, 2048, 1000), (4, 4, 5000, 4999), (16, 2, 64, 63),
    (32, 8, 8192, 8191), (32, 8, 33000, 20000), (32, 8, 33000, 64)])
def test_fused_append_attention_q4_0(orc, hq, hkv, ctx, pos):
    """decode_attention_qkv_q4_0 == rope + Q4_0 append + attention_q4_0, cache planes included."""
    k, v = random_rows(hkv, ctx, seed=ctx * 3 + pos)
    kq, vq, d = host_planes(orc, k, v)
    rng = np.random.default_rng(pos + 11)
    qkv = (rng.standard_normal((hq + 2 * hkv) * 128) * 30).astype(np.float32)
    qg = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    kg = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    gk, gv, gd = dev(kq), dev(vq), dev(d).view(torch.float16)
    theta = F.theta_scale_f32()
    out, q8 = ops.decode_attention_qkv_q4_0(dev(qkv), dev(qg), dev(kg), state_tensor(pos), gk, gv, gd, hq, theta)
    q_ref, k_row, v_row = orc.qk_rope_f32(qkv, hq, hkv, qg, kg, pos, theta)
    kq[:, pos], d[:, pos, :4] = orc.kv_q4_0_rows(k_row.reshape(hkv, 128))
    vq[:, pos], d[:, pos, 4:] = orc.kv_q4_0_rows(v_row.reshape(hkv, 128))
    got_kq, got_vq, got_d = planes_np(gk, gv, gd)
    # Row pos: V bit-exact; K from the fp64 rotation rounded once, equal to
    # the oracle's block for block barring a rounding tie.
    assert np.array_equal(got_vq, vq) and np.array_equal(got_d[:, :, 4:], d[:, :, 4:])
    others = np.ones(ctx, dtype=bool)
    others[pos] = False
    assert np.array_equal(got_kq[:, others], kq[:, others]) and np.array_equal(got_d[:, others], d[:, others])
    same_blocks = (got_kq[:, pos].reshape(hkv, 4, 16) == kq[:, pos].reshape(hkv, 4, 16)).all(-1) & \
        (got_d[:, pos, :4] == d[:, pos, :4])
    assert same_blocks.mean() >= 0.96, same_blocks
    # The attention against the oracle over the cache the GPU wrote.
    ref = orc.attention_q4_0(q_ref, got_kq, got_vq, np.ascontiguousarray(got_d), pos + 1, hq, hkv)
    got = out.cpu().numpy()
    assert_within_tolerance(got, ref, f"fused Q4_0 attention pos={pos}")
    assert (got.view(np.uint32) == ref.view(np.uint32)).mean() > 0.999
    assert np.array_equal(q8.cpu().numpy(), np.frombuffer(orc.quantize_q8_1(got), dtype=np.uint8))
    assert ops.device_error() == 0


def test_fused_q4_0_overflow_appends_nothing():
    hq, hkv, ctx = 8, 4, 40
    kq, vq, d = empty_planes(hkv, ctx)
    qkv = torch.ones((hq + 2 * hkv) * 128, device="cuda")
    g = torch.ones(128, device="cuda")
    out, _ = ops.decode_attention_qkv_q4_0(qkv, g, g, state_tensor(ctx), kq, vq, d, hq)
    assert ops.device_error(clear=True) & 16
    assert not kq.any() and not vq.any() and not d.any()
    assert torch.isfinite(out).all()


def test_attention_q4_0_peaked_and_zero_blocks(orc):
    """One key dominates; whole blocks of zeros (d = -0) in the cache."""
    hq, hkv, ctx, pos = 8, 2, 600, 599
    k, v = random_rows(hkv, ctx, seed=9)
    k[:, 123, :] = 3.0
    v[:, ::7, :32] = 0.0
    kq, vq, d = host_planes(orc, k, v)
    q = np.full(hq * 128, 2.0, dtype=np.float32)
    out, _ = ops.decode_attention_q4_0(dev(q), dev(kq), dev(vq), dev(d).view(torch.float16), state_tensor(pos))
    ref = orc.attention_q4_0(q, kq, vq, d, pos + 1, hq, hkv)
    assert_within_tolerance(out.cpu().numpy(), ref, "peaked Q4_0 attention")


def test_attention_q4_0_pdl_chain_equals_plain(orc):
    hq, hkv, ctx, pos = 32, 8, 4224, 4100
    k, v = random_rows(hkv, ctx, seed=1)
    kq, vq, d = (dev(a) for a in host_planes(orc, k, v))
    d = d.view(torch.float16)
    q = dev(np.random.default_rng(2).standard_normal(hq * 128).astype(np.float32))
    a = ops.decode_attention_q4_0(q, kq, vq, d, state_tensor(pos))[0].cpu()
    st = state_tensor(pos)
    for _ in range(3):
        b = ops.decode_attention_q4_0(q, kq, vq, d, st, pdl=True)[0]
    assert torch.equal(a, b.cpu())


def test_q4_0_and_fp16_caches_attend_alike(orc):
    """The same rows through both cache types: outputs differ only by the
    4-bit quantisation error (a sanity bound, not a parity criterion)."""
    hq, hkv, ctx, pos = 32, 8, 1024, 1000
    k, v = random_rows(hkv, ctx, seed=4)
    q = dev(np.random.default_rng(3).standard_normal(hq * 128).astype(np.float32))
    kq, vq, d = (dev(a) for a in host_planes(orc, k, v))
    a = ops.decode_attention_q4_0(q, kq, vq, d.view(torch.float16), state_tensor(pos))[0]
    b = ops.decode_attention(q, dev(k).half(), dev(v).half(), state_tensor(pos))[0]
    rel = ((a - b).norm() / b.norm()).item()
    assert rel < 0.2, rel
