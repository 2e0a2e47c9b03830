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
