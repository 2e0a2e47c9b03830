"""Q8_1 quantiser on the GPU: bit-exact against the oracle."""
import numpy as np
import pytest
import torch

from gpu_util import dev
from mojo_llm_lab_b200 import ops

pytestmark = pytest.mark.gpu


def _inputs():
    rng = np.random.default_rng(3)
    cases = {
        "normal_2560": rng.standard_normal(2560).astype(np.float32),
        "normal_9728": rng.standard_normal(9728).astype(np.float32),
        "wide_range": (rng.standard_normal(4096) * 10.0 ** rng.integers(-6, 4, 4096)).astype(np.float32),
        "zeros_and_spikes": np.zeros(1024, dtype=np.float32),
        "ties": np.tile(np.float32(127.0) * np.arange(-16, 16, dtype=np.float32) / np.float32(32.0), 8),
        "tiny": (rng.standard_normal(512) * 1e-30).astype(np.float32),
    }
    cases["zeros_and_spikes"][::97] = 3.5
    return cases


@pytest.mark.parametrize("s_mode", [ops.S_D_SUMQ, ops.S_SUM_X])
@pytest.mark.parametrize("name", list(_inputs()))
def test_quantize_bit_exact(orc, name, s_mode):
    x = _inputs()[name]
    got = ops.quantize_q8_1(dev(x), s_mode=s_mode).cpu().numpy().tobytes()
    assert got == orc.quantize_q8_1(x, s_mode)
    assert ops.device_error() == 0


def test_quantize_reproduces_reference_activation_bytes(orc, golden):
    g = golden["q8_1_known_answer"]
    x = np.array(g["x"], dtype=np.float32)
    import hashlib
    for mode in (ops.S_D_SUMQ, ops.S_SUM_X):
        got = ops.quantize_q8_1(dev(x), s_mode=mode).cpu().numpy().tobytes()
        assert hashlib.sha256(got).hexdigest() == g["bytes_sha256"]


def test_quantize_rejects_bad_sizes():
    with pytest.raises(ValueError):
        ops.quantize_q8_1(torch.zeros(33, device="cuda"))
    with pytest.raises(ValueError):
        ops.quantize_q8_1(torch.zeros(32, device="cuda", dtype=torch.float64))


@pytest.mark.parametrize("s_mode", [ops.S_D_SUMQ, ops.S_SUM_X])
@pytest.mark.parametrize("offset", [0, 1, 2, 3])
@pytest.mark.parametrize("k", [32, 160, 2560, 9728, 32 * 4097])
def test_both_kernels_bit_exact(orc, k, offset, s_mode):
    """A 16-byte-aligned x takes the four-values-per-lane kernel, others the
    lane-per-value one; block counts not a multiple of four leave a partial
    group of blocks in the last warp.  Both give the oracle's bytes."""
    rng = np.random.default_rng(k + offset)
    x = (rng.standard_normal(k) * 10.0 ** rng.integers(-3, 3, k)).astype(np.float32)
    x[5::37] = 0.0
    x[64:96] = 0.0                                  # a zero block
    if k >= 160:
        x[96:128] = np.float32(0.5) * np.arange(-16, 16, dtype=np.float32)  # ties at x / d = k + 0.5
    buf = torch.zeros(k + 4, dtype=torch.float32, device="cuda")
    buf[offset:offset + k] = torch.from_numpy(x).cuda()
    got = ops.quantize_q8_1(buf[offset:offset + k], s_mode=s_mode).cpu().numpy().tobytes()
    assert got == orc.quantize_q8_1(x, s_mode)
    assert ops.device_error() == 0
