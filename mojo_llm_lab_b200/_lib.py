"""ctypes binding of lib/libmllb200.so (the C ABI of include/mllb200.h).

Loading fails loudly: there is no CPU or eager-PyTorch fallback anywhere in
this package.  If the library is missing it is built in place with nvcc; if
that fails the import error propagates.
"""
from __future__ import annotations

import ctypes as C
import re
import threading
from pathlib import Path

from . import build as _build

HEADER = _build.INCLUDE / "mllb200.h"

MLLB_OK = 0
MLLB_EINVAL = -1
MLLB_EALIGN = -2
MLLB_ECUDA = -3
MLLB_EUNSUPPORTED = -4

LAUNCH_PDL = 1
LAUNCH_CONST_AUX = 2  # IMROPE: gamma / positions / theta not written by the preceding kernel

S_D_SUMQ = 0
S_SUM_X = 1

_P = C.c_void_p
_I64 = C.c_int64


class ActF32(C.Structure):
    """mllb_act_f32 of include/mllb200.h (an activation built in the kernel)."""
    _fields_ = [("x", C.c_void_p), ("delta", C.c_void_p), ("gamma", C.c_void_p), ("x_out", C.c_void_p),
                ("eps", C.c_double), ("advance", C.c_void_p)]


_ACT = C.POINTER(ActF32)



class PeerGather(C.Structure):
    """mllb_peer_gather of include/mllb200.h."""
    _fields_ = [("rank", C.c_int32), ("world", C.c_int32), ("buffers", C.c_void_p * 8),
                ("flags", C.c_void_p * 8), ("count", C.c_void_p)]

SIGNATURES = {
    "mllb_abi_version": (C.c_int, []),
    "mllb_last_error": (C.c_char_p, []),
    "mllb_device_error": (C.c_int, [C.POINTER(C.c_uint32), C.c_int]),
    "mllb_q8_1_quantize": (C.c_int, [_P, _P, _I64, C.c_int, _P]),
    "mllb_q4k_matvec": (C.c_int, [_P, _P, _P, _I64, _I64, _P]),
    "mllb_q4k_matvec_ex": (C.c_int, [_P, _P, _P, _I64, _I64, C.c_uint, _P]),
    "mllb_q4k_gate_up_ex": (C.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, C.c_uint, _P]),
    "mllb_q6k_matvec_ex": (C.c_int, [_P, _P, _P, _I64, _I64, C.c_uint, _P]),
    "mllb_q4k_gate_up": (C.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, _P]),
    "mllb_q6k_matvec": (C.c_int, [_P, _P, _P, _I64, _I64, _P]),
    "mllb_rmsnorm_imrope_q": (C.c_int, [_P, _P, _P, _P, _P, _I64, _P]),
    "mllb_rmsnorm_imrope_q_batched": (C.c_int, [_P, _P, _P, _P, C.c_double, _P, _I64, _I64, _P]),
    "mllb_rmsnorm_imrope_q_batched_ex": (C.c_int, [_P, _P, _P, _P, C.c_double, _P, _I64, _I64, C.c_uint, _P]),
    "mllb_q4k_subdots": (C.c_int, [_P, _P, _P, _P, _I64, _I64, _P]),
    "mllb_stream_read": (C.c_int, [_P, _I64, _P, _I64, _P]),
    "mllb_q8_1_quantize_ex": (C.c_int, [_P, _P, _I64, C.c_int, C.c_uint, _P]),
    "mllb_token_key": (_I64, [C.c_int32]),
    "mllb_key_token": (_I64, [_I64]),
    "mllb_decode_embed": (C.c_int, [_P, _I64, _I64, _P, _P, _I64, _P, C.c_uint, _P]),
    "mllb_rmsnorm_q8_1": (C.c_int, [_P, _P, _P, _P, C.c_double, _P, _I64, C.c_int, C.c_uint, _P]),
    "mllb_decode_final_norm": (C.c_int, [_P, _P, _P, _P, C.c_double, _P, _I64, _P, C.c_uint, _P]),
    "mllb_decode_qk_rope_append": (C.c_int, [_P, _P, _P, _P, C.c_double, _P, _P, _P, _I64, _I64, _I64, C.c_uint,
                                             _P]),
    "mllb_decode_attention_scratch": (_I64, [_I64, _I64, _I64]),
    "mllb_decode_attention": (C.c_int, [_P, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _I64, C.c_uint, _P]),
    "mllb_decode_attention_qkv": (C.c_int, [_P, _P, _P, C.c_double, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _I64,
                                            C.c_uint, _P]),
    "mllb_decode_attention_qkv_noalloc": (C.c_int, [_P, _P, _P, C.c_double, _P, _P, _P, _P, _P, _I64, _I64, _I64,
                                                    C.c_uint, _P]),
    "mllb_kv_q4_0_store": (C.c_int, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, C.c_uint, _P]),
    "mllb_decode_attention_q4_0": (C.c_int, [_P, _P, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _I64, C.c_uint, _P]),
    "mllb_decode_attention_qkv_q4_0": (C.c_int, [_P, _P, _P, C.c_double, _P, _P, _P, _P, _P, _I64, _P, _P, _I64,
                                                 _I64, _I64, C.c_uint, _P]),
    "mllb_argmax_f32": (C.c_int, [_P, _I64, _I64, _P, C.c_uint, _P]),
    "mllb_q8_1_quantize_allgather": (C.c_int, [_P, _I64, C.POINTER(PeerGather), C.c_uint, _P]),
    "mllb_q4k_gate_up_q8_gather": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, C.POINTER(PeerGather),
                                             C.c_uint, _P]),
    "mllb_prefetch_l2": (C.c_int, [_P, _I64, _P]),
    "mllb_q5k_matvec": (C.c_int, [_P, _P, _P, _I64, _I64, _P]),
    "mllb_q5k_matvec_ex": (C.c_int, [_P, _P, _P, _I64, _I64, C.c_uint, _P]),
    "mllb_q4k_matvec_act": (C.c_int, [_P, _ACT, _P, _I64, _I64, C.c_uint, _P]),
    "mllb_q4k_gate_up_act": (C.c_int, [_P, _P, _ACT, _P, _P, _P, _I64, _I64, C.c_uint, _P]),
    "mllb_q6k_matvec_act": (C.c_int, [_P, _ACT, _P, _I64, _I64, C.c_uint, _P]),
    "mllb_q4k_gate_up_q8": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, C.c_uint, _P]),
    "mllb_q4k_matvec_norm_workspace": (_I64, [_I64, _I64]),
    "mllb_q4k_matvec_norm": (C.c_int, [_P, _P, _P, _I64, _I64, _P, _P, _P, C.c_double, _P, _P, _I64, C.c_uint, _P]),
    "mllb_q4k_matmul_tokens_workspace": (C.c_int64, [_I64, _I64, _I64]),
    "mllb_q4k_matmul_tokens": (C.c_int, [_P, _P, _P, _I64, _I64, _I64, _P, _I64, C.c_uint, _P]),
}

_lock = threading.Lock()
_handle = None


class MllbError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{message} (code {code})")
        self.code = code


def declared_symbols() -> list[str]:
    """Every function the public header declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(mllb_\w+)\s*\(", text, re.M)))


def lib() -> C.CDLL:
    global _handle
    with _lock:
        if _handle is None:
            if not _build.LIB.exists():
                _build.build()
            handle = C.CDLL(str(_build.LIB))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            if handle.mllb_abi_version() != 1:
                raise RuntimeError("libmllb200.so ABI version mismatch")
            _handle = handle
    return _handle


def check(rc: int, what: str) -> None:
    if rc != MLLB_OK:
        msg = lib().mllb_last_error().decode(errors="replace")
        if rc in (MLLB_EINVAL, MLLB_EALIGN):
            raise ValueError(f"{what}: {msg} (code {rc})")
        raise MllbError(rc, f"{what}: {msg}")


def device_error(clear: bool = True) -> int:
    bits = C.c_uint32(0)
    check(lib().mllb_device_error(C.byref(bits), 1 if clear else 0), "mllb_device_error")
    return bits.value
