"""ctypes binding of ``libfaquant_b200.so`` (the C ABI of ``include/faquant_b200.h``).

The library sits next to this file (built in-tree by ``build.py``). Loading it
is the only way these operators run: a missing library or a missing CUDA device
raises, there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libfaquant_b200.so")

FAQ_OK = 0
FAQ_BF16 = 0
FAQ_F32 = 1
FAQ_STATUS_TIMEOUT = 1

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int

# name -> argument types (all return int status)
SIGNATURES: dict[str, list] = {
    "faq_version": [],
    "faq_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "faq_device_status": [ctypes.POINTER(ctypes.c_uint), _int],
    "faq_hif4_quantize": [_c_void_p, _int, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _int, _int,
                          _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p],
    "faq_hif4_quantize_rms_norm": [_c_void_p, _i64, _i64, _i64, _c_void_p, ctypes.c_float, _c_void_p, _c_void_p,
                                   _c_void_p, _int, _int, _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p],
    "faq_hif4_quantize_layer_norm": [_c_void_p, _i64, _i64, _i64, ctypes.c_float, _c_void_p, _c_void_p, _c_void_p,
                                     _int, _int, _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p],
    "faq_hif4_quantize_act": [_c_void_p, _int, _i64, _i64, _i64, _c_void_p, _c_void_p, _int, _int, _c_void_p,
                              _c_void_p, _c_void_p, _i64, _c_void_p],
    "faq_set_gemm_sm_target": [_int],
    "faq_hif4_dequantize": [_c_void_p, _c_void_p, _i64, _i64, _c_void_p, _int, _i64, _c_void_p],
    "faq_hif4_pack_weight": [_c_void_p, _int, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _int,
                             _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    "faq_gemm_bf16_tn": [_c_void_p, _i64, _c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p, _i64,
                         _c_void_p],
    "faq_gemm_bf16_tn_residual": [_c_void_p, _i64, _c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p,
                                  _i64, _c_void_p, _i64, _c_void_p],
    "faq_w4a4_gemm": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _i64,
                      _c_void_p, _i64, _c_void_p],
    "faq_w4a4_gemm_qdq_a": [_c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _i64,
                            _c_void_p, _i64, _c_void_p],
    "faq_qk_prep": [_c_void_p, _int, _i64, _i64, _i64, _int, _i64, _i64, _i64, _c_void_p, _c_void_p, _i64, _int,
                    _int, _int, _c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p],
    "faq_qk_norm_rope_prep": [_c_void_p, _int, _i64, _i64, _i64, _int, _i64, _i64, _i64, _c_void_p,
                              ctypes.c_float, _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _i64, _int, _int,
                              _int, _c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p],
    "faq_rms_norm": [_c_void_p, _i64, _i64, _i64, _c_void_p, ctypes.c_float, _c_void_p, _i64, _c_void_p],
    "faq_silu_mul": [_c_void_p, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p],
    "faq_layer_norm": [_c_void_p, _i64, _i64, _i64, ctypes.c_float, _c_void_p, _i64, _c_void_p],
    "faq_gelu_tanh": [_c_void_p, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p],
    "faq_row_sumsq": [_c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p],
    "faq_wan_qk_prep": [_c_void_p, _i64, _i64, _i64, _int, _i64, _i64, _i64, _c_void_p, _i64, _i64, _i64, _i64,
                        _c_void_p, ctypes.c_float, _c_void_p, _c_void_p, _c_void_p, _i64, _int, _int, _int, _c_void_p, _i64,
                        _i64, _i64, _c_void_p],
    "faq_hif4_attention": [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64, _int,
                           _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _int, _int,
                           _int, _c_void_p, _i64, _i64, _i64, _c_void_p],
    "faq_hif4_decode_attention": [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64, _int,
                                  _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _int,
                                  _int, _c_void_p, _i64, _i64, _i64, _c_void_p, ctypes.c_size_t, _c_void_p],
    "faq_hif4_decode_attention_static": [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64, _int,
                                         _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float,
                                         _int, _int, _c_void_p, _i64, _i64, _i64, _c_void_p],
    "faq_gptq_hif4_block": [_c_void_p, _i64, _i64, _int, _i64, _c_void_p, _i64, _i64, _int, _c_void_p, _i64,
                            _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p],
    "faq_selftest_wait_timeout": [_i64, _c_void_p],
    "faq_selftest_ex2_monotone": [ctypes.POINTER(ctypes.c_uint64), _c_void_p],
    "faq_device_trace": [ctypes.POINTER(ctypes.c_uint), _int, _int],
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class FaqError(RuntimeError):
    """A C-ABI call returned an error status."""


def load() -> ctypes.CDLL:
    """Load the library (once) and declare every exported signature."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise FaqError(
                    f"{LIB_PATH} is missing; build it with `python faquant-public_b200/build.py` "
                    "(the HiF4 operators have no CPU fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, argtypes in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = ctypes.c_int
            # size queries return size_t, not a status
            lib.faq_hif4_decode_workspace_bytes.argtypes = [_i64, _i64, _i64, _i64, _i64, _int]
            lib.faq_hif4_decode_workspace_bytes.restype = ctypes.c_size_t
            _lib = lib
        return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().faq_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


_CODE_NAMES = {1: "FAQ_ERR_ARG", 2: "FAQ_ERR_CUDA", 3: "FAQ_ERR_UNSUPPORTED", 4: "FAQ_ERR_TIMEOUT"}


def check(rc: int, what: str) -> None:
    if rc != FAQ_OK:
        exc = ValueError if rc == 1 else NotImplementedError if rc == 3 else FaqError
        raise exc(f"{what}: {_CODE_NAMES.get(rc, rc)}: {last_error()}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def device_trace(reset: bool = False) -> list[tuple[int, int, int, int, int]]:
    """Records of the device waits that gave up: (site, tile, block x, block y, block z)."""
    buf = (ctypes.c_uint * 96)()
    n = load().faq_device_trace(buf, 32, int(reset))
    if n < 0:
        raise FaqError(f"faq_device_trace failed: {last_error()}")
    out = []
    for i in range(min(n, 32)):
        w0, w1, w2 = buf[3 * i], buf[3 * i + 1], buf[3 * i + 2]
        out.append((w0 & 0xFF, w0 >> 8, w1 & 0xFFFF, w1 >> 16, w2))
    return out


def device_status(reset: bool = False) -> int:
    status = ctypes.c_uint(0)
    check(load().faq_device_status(ctypes.byref(status), int(reset)), "faq_device_status")
    return status.value
