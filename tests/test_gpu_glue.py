"""GPU tests of the fused decoder glue: faq_rms_norm, faq_silu_mul and the Qwen3 K4
variant faq_qk_norm_rope_prep, against torch's own ops on the CPU (the reference's
glue) and the oracle. Where the ops are pure bf16-rounded elementwise math (RoPE, the
HiF4 steps) the results are bit-exact; the row reductions (RMSNorm) and exp (SiLU) sum or
round differently from torch's CPU kernels, so those are held to one bf16 ulp."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import hif4 as oh

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _within_ulp(got: torch.Tensor, ref: torch.Tensor) -> None:
    g, r = got.float().cpu(), ref.float().cpu()
    assert torch.all((g - r).abs() <= 2.0**-7 * r.abs() + 1e-30)


def test_rms_norm_matches_qwen3_rmsnorm() -> None:
    from faquant_b200 import ops
    from faquant_b200.tensor_parallel import rms_norm

    g = torch.Generator().manual_seed(1)
    for k in (128, 5120, 12288, 25600):
        x = (torch.randn(37, k, generator=g) * 3).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
        _within_ulp(ops.rms_norm(x.to(DEV), w.to(DEV), 1e-6), rms_norm(x, w, 1e-6))
    empty = ops.rms_norm(torch.zeros(0, 64, dtype=torch.bfloat16, device=DEV), torch.ones(64, device=DEV), 1e-6)
    assert empty.shape == (0, 64)


def test_silu_mul_matches_torch() -> None:
    from faquant_b200 import ops

    gu = (torch.randn(50, 2 * 1728, generator=torch.Generator().manual_seed(2)) * 4).to(torch.bfloat16)
    ref = torch.nn.functional.silu(gu[:, :1728]) * gu[:, 1728:]
    _within_ulp(ops.silu_mul(gu.to(DEV)), ref)


def test_qk_norm_rope_prep_stages() -> None:
    """No norm, no RoPE: exactly faq_qk_prep. RoPE alone: bit-exact with torch's bf16
    RoPE followed by the oracle's Hadamard + HiF4. Norm + RoPE: codes of >= 99.5% of the
    values equal (a one-ulp norm difference can move a HiF4 block)."""
    from faquant_b200 import ops
    from faquant_b200.tensor_parallel import apply_rope, rms_norm, rope_tables

    g = torch.Generator().manual_seed(3)
    b, h, s, d = 2, 6, 96, 128
    x = torch.randn(b, s, h, d, generator=g).to(torch.bfloat16)  # projection layout [B, S, H, D]
    xv = x.to(DEV).transpose(1, 2)  # strided [B, H, S, D] view, as the prefill passes it
    cos, sin = rope_tables(s, d, 1e6, torch.device("cpu"))
    w = (1 + 0.2 * torch.randn(d, generator=g)).to(torch.bfloat16)
    plain = ops.qk_norm_rope_prep(xv, norm_weight=None, levels="123")
    assert torch.equal(plain, ops.qk_prep(xv, levels="123", rotate=True)[0])
    roped = ops.qk_norm_rope_prep(xv, norm_weight=None, cos=cos.to(DEV), sin=sin.to(DEV), levels="123")
    r = apply_rope(x, cos, sin).transpose(1, 2).float().numpy()
    expect = oh.fake_quantize(oatt.qk_pretransform(r, r)[0], "123")
    assert np.array_equal(roped.float().cpu().numpy(), expect)
    full = ops.qk_norm_rope_prep(xv, norm_weight=w.to(DEV), eps=1e-6, cos=cos.to(DEV), sin=sin.to(DEV), levels="123")
    r = apply_rope(rms_norm(x, w, 1e-6), cos, sin).transpose(1, 2).float().numpy()
    expect = oh.fake_quantize(oatt.qk_pretransform(r, r)[0], "123")
    got = full.float().cpu().numpy()
    assert np.mean(got == expect) >= 0.995
    assert np.linalg.norm(got - expect) <= 2e-2 * np.linalg.norm(expect)
