"""CPU checks of the C-ABI boundary: the library loads, exports every symbol
the public header declares, and rejects bad arguments before touching CUDA."""
import ctypes as C

import pytest

from mojo_llm_lab_b200 import _lib, build


def test_library_exports_every_declared_symbol():
    names = _lib.declared_symbols()
    assert len(names) >= 11
    handle = _lib.lib()
    for name in names:
        assert hasattr(handle, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_abi_version_and_error_string():
    assert _lib.lib().mllb_abi_version() == 1
    assert isinstance(_lib.lib().mllb_last_error(), bytes)


@pytest.mark.parametrize("call", [
    lambda L: L.mllb_q4k_matvec(None, None, None, 4096, 2560, None),
    lambda L: L.mllb_q4k_gate_up(None, None, None, None, None, None, 1, 2560, None),
    lambda L: L.mllb_q6k_matvec(None, None, None, 1, 2560, None),
    lambda L: L.mllb_q8_1_quantize(None, None, 32, 0, None),
    lambda L: L.mllb_rmsnorm_imrope_q(None, None, None, None, None, 32, None),
    lambda L: L.mllb_q4k_subdots(None, None, None, None, 1, 256, None),
    lambda L: L.mllb_stream_read(None, 16, None, 0, None),
    lambda L: L.mllb_kv_q4_0_store(None, None, None, None, None, 8, 64, 0, 1, 0, None),
    lambda L: L.mllb_decode_attention_q4_0(None, 16, 16, 16, 16, 16, 1 << 20, 16, 16, 32, 8, 64, 0, None),
    lambda L: L.mllb_decode_attention_qkv_q4_0(None, None, None, 0.5, 16, 16, 16, 16, 16, 1 << 20, 16, 16, 32, 8,
                                               64, 0, None),
    lambda L: L.mllb_q4k_matvec_norm(None, None, None, 2560, 4096, None, None, None, 1e-6, None, None, 4096, 0,
                                     None),
    lambda L: L.mllb_q4k_gate_up_q8(None, None, None, None, None, None, None, None, 32, 2560, 0, None),
])
def test_null_pointers_rejected_without_cuda(call):
    assert call(_lib.lib()) == _lib.MLLB_EINVAL
    assert b"null" in _lib.lib().mllb_last_error()


def test_shape_and_alignment_rejections():
    L = _lib.lib()
    # K not a multiple of 256, zero rows, bad s_mode, misaligned weights
    assert L.mllb_q4k_matvec(16, 16, 16, 4, 2500, None) == _lib.MLLB_EINVAL
    assert L.mllb_q4k_matvec(16, 16, 16, 0, 2560, None) == _lib.MLLB_EINVAL
    assert L.mllb_q8_1_quantize(16, 16, 31, 0, None) == _lib.MLLB_EINVAL
    assert L.mllb_q8_1_quantize(16, 16, 32, 7, None) == _lib.MLLB_EINVAL
    assert L.mllb_q4k_matvec(8, 16, 16, 4, 2560, None) == _lib.MLLB_EALIGN
    assert L.mllb_q6k_matvec(8, 16, 16, 4, 2560, None) == _lib.MLLB_EALIGN
    assert L.mllb_q4k_gate_up(16, 16, 16, None, None, None, 4, 2560, None) == _lib.MLLB_EINVAL


def test_new_entry_rejections_without_cuda():
    L = _lib.lib()
    # residual-norm matvec: rows not whole Q8_1 groups, workspace too small,
    # negative eps; its workspace size is pure arithmetic.
    assert L.mllb_q4k_matvec_norm(16, 16, None, 48, 2560, 16, 16, 16, 1e-6, 16, 16, 4096, 0, None) == _lib.MLLB_EINVAL
    assert L.mllb_q4k_matvec_norm(16, 16, None, 64, 2560, 16, 16, 16, 1e-6, 16, 16, 8, 0, None) == _lib.MLLB_EINVAL
    assert L.mllb_q4k_matvec_norm(16, 16, None, 64, 2560, 16, 16, 16, -1.0, 16, 16, 4096, 0, None) == _lib.MLLB_EINVAL
    assert L.mllb_q4k_matvec_norm_workspace(2560, 4096) == 16 + 8 * 640
    # q8_out inside x_out, workspace inside q8_out
    assert L.mllb_q4k_matvec_norm(16, 16, None, 64, 2560, 4096, 8192, 16384, 1e-6, 8192 + 64, 1 << 20, 4096, 0,
                                  None) == _lib.MLLB_EINVAL
    assert L.mllb_q4k_matvec_norm(16, 16, None, 64, 2560, 4096, 8192, 16384, 1e-6, 32768, 32768 + 16, 4096, 0,
                                  None) == _lib.MLLB_EINVAL
    # workspace over x, over gamma, over the Q8_1 input; q8_out over the Q8_1 input
    assert L.mllb_q4k_matvec_norm(16, 1 << 16, None, 64, 2560, 4096, 8192, 16384, 1e-6, 32768, 4096, 4096, 0,
                                  None) == _lib.MLLB_EINVAL
    assert L.mllb_q4k_matvec_norm(16, 1 << 16, None, 64, 2560, 4096, 8192, 16384, 1e-6, 32768, 16384, 4096, 0,
                                  None) == _lib.MLLB_EINVAL
    assert L.mllb_q4k_matvec_norm(16, 1 << 16, None, 64, 2560, 4096, 8192, 16384, 1e-6, 32768, 1 << 16, 4096, 0,
                                  None) == _lib.MLLB_EINVAL
    assert L.mllb_q4k_matvec_norm(16, 1 << 16, None, 64, 2560, 4096, 8192, 16384, 1e-6, 1 << 16, 1 << 20, 4096, 0,
                                  None) == _lib.MLLB_EINVAL
    # Q4_0 cache store: rows past the cache, misaligned scale plane for the attention
    assert L.mllb_kv_q4_0_store(16, 16, 16, 16, 16, 2, 10, 7, 4, 0, None) == _lib.MLLB_EINVAL
    assert L.mllb_decode_attention_q4_0(16, 16, 16, 18, 16, 16, 1 << 20, 16, 16, 32, 8, 64, 0,
                                        None) == _lib.MLLB_EALIGN
    assert L.mllb_decode_attention_q4_0(16, 16, 16, None, 16, 16, 1 << 20, 16, 16, 32, 8, 64, 0,
                                        None) == _lib.MLLB_EINVAL


def test_compat_cubin_built_for_sm100a():
    data = build.CUBIN.read_bytes()
    assert data[:4] == b"\x7fELF"
    for entry in (b"fused_q_imrope_runtime_fastpow", b"q4_k_q8_1_matvec_dp4a_128", b"q4_k_q8_1_gate_order",
                  b"q4_k_q8_1_matvec_dp4a", b"stream_read_roofline", b"q6_k_q8_1_matvec"):
        assert entry in data


def test_interposer_exports_the_runtime_launch_hooks():
    """lib/libmllb200_interpose.so (LD_PRELOAD) defines the CUDA runtime's two
    launch entries and links to libmllb200.so, not to a CUDA runtime of its own."""
    import shutil
    import subprocess
    build.build()
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm not available")
    out = subprocess.run([nm, "-D", "--defined-only", str(build.INTERPOSE)], capture_output=True, text=True,
                         check=True).stdout
    defined = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert {"cudaLaunchKernel", "cudaLaunchKernelExC", "mllb_interpose_counts"} <= defined
    needed = subprocess.run(["readelf", "-d", str(build.INTERPOSE)], capture_output=True, text=True).stdout
    assert "libmllb200.so" in needed and "libcudart" not in needed
