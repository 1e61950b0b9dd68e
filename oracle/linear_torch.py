"""The reference's ``FakeQuantLinear`` forward restated in CPU torch (test infrastructure).

This is the CPU baseline of ``bench.py`` when the reference itself cannot be imported on
the machine (the reference is a Python package that does not travel with this
repository). It restates, with the same torch operations in the same order -- so with the
same arithmetic and the same cost profile on the host's cores, which is what a baseline
has to measure -- the forward pass of ``FakeQuantLinear``
(``src/faquant/quantization.py:199-277``) for the deployed recipe:

- the input rotation in 256-row chunks (``:203-221``): ``x.float() * signs``, a gather by
  the permutation, the block Hadamard of ``chunked_block_hadamard_transform``
  (``rotation.py:117-135``), whose butterflies go stride 1, 2, 4, ... with one
  ``torch.cat`` per stage (``rotation.py:14-29``), the division by ``sqrt(block)`` and
  the cast back to the input dtype;
- the HiF4 fake quantization of ``fake_quantize_hif4`` (``hif4.py:376-390``): zero-pad to
  64, the three amax levels over ``[.., 8, 2, 4]`` views, the E6M2 scale of
  ``_e6m2_scale`` (``hif4.py:91-115``: bf16 multiply by bf16(1/divisor), clamp, the bf16
  and E6M2 roundings through ``log2``/``exp2``, the bf16 reciprocal), the lv2/lv3
  exponents (``:188-213``), and ``floor(|x| q 4 + 0.5) / 4`` clamped to 1.75 times the
  sign and the dequantization scale (``:254-271``);
- ``F.linear`` on the bf16 operands (``:277``).

Only ``tests/`` and ``bench.py``'s CPU legs use it; ``test_oracle_golden.py`` checks it
against the reference's own outputs.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _bf16_rounded(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(t.dtype)


def _fwht(x: torch.Tensor) -> torch.Tensor:
    """Normalized Walsh-Hadamard over the last axis, stage by stage (rotation.py:14-29)."""
    n = x.shape[-1]
    shape = x.shape
    y = x.reshape(-1, n)
    h = 1
    while h < n:
        pairs = y.reshape(-1, n // (2 * h), 2, h)
        lo, hi = pairs[:, :, 0, :], pairs[:, :, 1, :]
        y = torch.cat((lo + hi, lo - hi), dim=2).reshape(-1, n)
        h *= 2
    return (y / math.sqrt(n)).reshape(shape)


def _block_fwht(x: torch.Tensor, block: int, chunk_rows: int = 256) -> torch.Tensor:
    """``chunked_block_hadamard_transform`` (rotation.py:117-135)."""
    rows, k = x.shape
    out = torch.empty_like(x)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(r0 + chunk_rows, rows)
        part = x[r0:r1].float().reshape(-1, block)
        out[r0:r1].copy_(_fwht(part).reshape(r1 - r0, k).to(x.dtype))
    return out


def _e6m2(maximum: torch.Tensor, divisor: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Scale and bf16 reciprocal of a block maximum (hif4.py:91-115)."""
    inv = _bf16_rounded(torch.ones_like(maximum) / divisor)
    s = _bf16_rounded(maximum * inv).clamp(min=2.0**-48, max=49152.0)
    e = torch.floor(torch.log2(s))
    s = torch.round(s * torch.exp2(7.0 - e)) * torch.exp2(e - 7.0)
    e = torch.floor(torch.log2(s))
    s = torch.round(s * torch.exp2(2.0 - e)) * torch.exp2(e - 2.0)
    return s, _bf16_rounded(1.0 / s)


def hif4_fake_quantize(x: torch.Tensor, levels: str = "123") -> torch.Tensor:
    """HiF4 QDQ along the last axis (hif4.py:376-390), in torch on x's device."""
    k = x.shape[-1]
    pad = (-k) % 64
    xp = F.pad(x, (0, pad)) if pad else x
    blocks = xp.reshape(*xp.shape[:-1], -1, 64)
    w = blocks.float().reshape(*blocks.shape[:-1], 8, 2, 4)
    mag = w.abs()
    m3 = mag.amax(dim=-1, keepdim=True)
    m2 = m3.amax(dim=-2, keepdim=True)
    m1 = m2.amax(dim=-3, keepdim=True)
    s, rec = _e6m2(m1, 7.0 if levels == "123" else 3.5)
    if levels == "123":
        e2 = torch.floor((m2 * rec).clamp(0.0, 4.0) / 4.0)
        e3 = torch.floor((m3 * rec / torch.exp2(e2)).clamp(0.0, 2.0) / 2.0)
    elif levels == "12":
        e2 = torch.floor((m2 * rec).clamp(0.0, 2.0) / 2.0)
        e3 = torch.zeros_like(m3)
    elif levels == "13":
        e2 = torch.zeros_like(m2)
        e3 = torch.floor((m3 * rec).clamp(0.0, 2.0) / 2.0)
    else:
        raise ValueError(f"unknown HiF4 levels {levels!r}")
    # the expanded per-value multiplier and scale (hif4.py:222-243), then the rounding
    shape = w.shape
    mult = (rec / torch.exp2(e2.to(torch.int8).float()) / torch.exp2(e3.to(torch.int8).float())).expand(shape)
    dq = (s * torch.exp2(e2.to(torch.int8).float()) * torch.exp2(e3.to(torch.int8).float())).expand(shape)
    mant = torch.floor(w.abs() * mult * 4.0 + 0.5) / 4.0
    mant.clamp_(max=1.75)
    out = (torch.sign(w) * mant * dq).to(x.dtype)
    return out.reshape(*blocks.shape[:-2], -1)[..., :k]


def fake_quant_linear(x: torch.Tensor, weight_q: torch.Tensor, bias: torch.Tensor | None, *, levels: str,
                      signs: torch.Tensor | None, permutation: torch.Tensor | None,
                      block: int | None) -> torch.Tensor:
    """One ``FakeQuantLinear.forward`` on CPU: x [T, K] bf16, weight_q [N, K] bf16 (already
    on the HiF4 grid, as the module stores it) -> [T, N] bf16."""
    if signs is not None:
        rows, k = x.shape
        rotated = torch.empty_like(x)
        sf = signs.to(torch.float32)
        for r0 in range(0, rows, 256):
            r1 = min(r0 + 256, rows)
            work = (x[r0:r1].float() * sf).index_select(-1, permutation)
            if block is not None:
                work = _block_fwht(work, block)
            rotated[r0:r1].copy_(work.to(x.dtype))
        x = rotated
    xq = hif4_fake_quantize(x, levels)
    return F.linear(xq, weight_q, bias)
