"""The C-ABI library: it loads, exports every symbol include/faquant_b200.h declares,
and rejects bad arguments on the host (no GPU needed for any of this)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared() -> list[str]:
    text = (ROOT / "include" / "faquant_b200.h").read_text()
    return re.findall(r"^int (faq_\w+)\(", text, re.M)


def test_header_declares_the_abi() -> None:
    names = _declared()
    assert {"faq_hif4_quantize", "faq_gemm_bf16_tn", "faq_hif4_attention", "faq_qk_prep"} <= set(names)


def test_library_exports_every_declared_symbol() -> None:
    from faquant_b200 import _lib

    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, name
    assert lib.faq_version() == 100


def test_host_side_argument_validation() -> None:
    from faquant_b200 import _lib

    lib = _lib.load()
    # null input, bad levels, no outputs: rejected before any CUDA call
    assert lib.faq_hif4_quantize(None, 0, 4, 64, 64, None, None, None, 0, 123, None, None, None, 64, None) == 1
    assert "null" in _lib.last_error()
    fake = ctypes.c_void_p(16)
    assert lib.faq_hif4_quantize(fake, 0, 4, 64, 64, None, None, None, 0, 7, None, None, fake, 64, None) == 1
    assert "levels" in _lib.last_error()
    assert lib.faq_hif4_quantize(fake, 0, 4, 64, 64, None, None, None, 0, 123, None, None, None, 64, None) == 1
    assert lib.faq_gemm_bf16_tn(fake, 12, fake, 16, 4, 4, 12, None, fake, 4, None) == 1
    assert "multiples of 8" in _lib.last_error()
    # the GEMM SM target is host state: a negative count is refused, 0 (every SM) accepted
    assert lib.faq_set_gemm_sm_target(-1) == 1 and "sms" in _lib.last_error()
    assert lib.faq_set_gemm_sm_target(0) == 0
    # the fused-norm quantizer needs at least one of codes and qdq
    assert lib.faq_hif4_quantize_rms_norm(fake, 4, 1024, 1024, fake, ctypes.c_float(1e-6), None, fake, None, 1024,
                                          123, None, None, None, 1024, None) == 1
    assert "both null" in _lib.last_error()
    with pytest.raises(ValueError):
        _lib.check(1, "demo")


def test_operators_refuse_cpu_tensors() -> None:
    import torch

    from faquant_b200 import ops

    with pytest.raises(RuntimeError, match="CUDA"):
        ops.hif4_quantize(torch.zeros(2, 64))
