"""mllb_decode_attention_qkv_noalloc: the decode attention with its chunk
partials in the library's own device array, against mllb_decode_attention_qkv
with a caller buffer.  Collected last on purpose: it must also pass after
every other test has used the library in the same process."""
import numpy as np
import pytest
import torch

from mojo_llm_lab_b200 import decode as D
from mojo_llm_lab_b200 import formats as F
from mojo_llm_lab_b200 import ops
from mojo_llm_lab_b200._lib import MllbError, check, lib

pytestmark = pytest.mark.gpu


def noalloc(qkv, qg, kg, state, kc, vc, out, q8, q_heads):
    check(lib().mllb_decode_attention_qkv_noalloc(
        qkv.data_ptr(), qg.data_ptr(), kg.data_ptr(), F.theta_scale_f32(), state.data_ptr(), kc.data_ptr(),
        vc.data_ptr(), out.data_ptr(), q8.data_ptr(), q_heads, kc.shape[0], kc.shape[1], 0,
        torch.cuda.current_stream().cuda_stream), "decode_attention_qkv_noalloc")


def state_at(pos):
    return torch.frombuffer(bytearray(D.state_bytes(0, pos)), dtype=torch.uint8).cuda()


def test_noalloc_equals_caller_scratch_two_calls_in_a_row():
    hq, hkv, ctx = 32, 8, 4224
    rng = np.random.default_rng(0)
    k = torch.from_numpy(rng.standard_normal((hkv, ctx, 128)).astype(np.float16)).cuda()
    v = torch.from_numpy(rng.standard_normal((hkv, ctx, 128)).astype(np.float16)).cuda()
    qg = torch.from_numpy(rng.uniform(0.5, 1.5, 128).astype(np.float32)).cuda()
    kg = torch.from_numpy(rng.uniform(0.5, 1.5, 128).astype(np.float32)).cuda()
    ka, va, kb, vb = k.clone(), v.clone(), k.clone(), v.clone()
    for pos in (4096, 4097):  # two calls in a row; each appends its row
        qkv = torch.from_numpy((rng.standard_normal((hq + 2 * hkv) * 128) * 20).astype(np.float32)).cuda()
        ref_out, ref_q8 = ops.decode_attention_qkv(qkv, qg, kg, state_at(pos), ka, va, hq)
        out = torch.full_like(ref_out, 7.0)
        q8 = torch.zeros_like(ref_q8)
        noalloc(qkv, qg, kg, state_at(pos), kb, vb, out, q8, hq)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out)
        assert torch.equal(q8, ref_q8)
        assert torch.equal(kb, ka) and torch.equal(vb, va)
    assert ops.device_error() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    hq, hkv, ctx = 64, 8, 4224  # 64 x 18 chunks x 130 doubles > 131072
    kc = torch.zeros((hkv, ctx, 128), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    qkv = torch.zeros((hq + 2 * hkv) * 128, device="cuda")
    g = torch.ones(128, device="cuda")
    out = torch.empty(hq * 128, device="cuda")
    q8 = torch.empty(hq * 128 // 32 * 36, dtype=torch.uint8, device="cuda")
    with pytest.raises(MllbError, match="built-in scratch"):
        noalloc(qkv, g, g, state_at(100), kc, vc, out, q8, hq)
