"""Seeded input builders shared by ``make_golden.py`` and the tests.

Inputs are drawn from the torch CPU generator, which is deterministic for a
given torch build, so fixtures store only a SHA-256 of each input and the
tests rebuild it here and check the hash before comparing outputs.
"""

from __future__ import annotations

import hashlib

import torch


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def outlier_rows(rows: int, cols: int, seed: int, outliers: int, factor: float = 20.0) -> torch.Tensor:
    """N(0,1) rows whose ``outliers`` randomly chosen channels are scaled by ``factor``."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g)
    idx = torch.randperm(cols, generator=g)[:outliers]
    x[:, idx] *= factor
    return x


def special_rows() -> torch.Tensor:
    """Rows exercising zero blocks, tiny/huge magnitudes, -0.0 and exact ties."""
    g = torch.Generator().manual_seed(7)
    x = torch.randn(12, 200, generator=g)
    x[0, :64] = 0.0  # zero block -> scale clamp 2^-48
    x[1, :64] = -0.0
    x[2] *= 1e-30  # tiny
    x[3] *= 3.0e4  # near the 49152 clamp after /7
    x[4] *= 1e6  # clamp at 49152
    x[5, :] = torch.linspace(-17.25, 18.75, 200)
    x[6] = torch.round(x[6] * 8) / 8  # dyadic values -> exact ties
    x[7, ::3] = 0.0
    x[8] = x[8].abs()  # unsigned (P-like)
    x[9] = torch.exp(-x[9].abs() * 4)  # softmax-probability-like values in (0, 1]
    x[10, 5] = 1e-3
    x[10, :5] = -1e-12  # small negatives that round to -0.0
    x[11] *= 2.0**-126  # subnormal-range magnitudes
    return x


LINEAR_CASES = [
    # (tag, rows, in, out, block, seed, rotation name, rotation seed)
    ("r64", 96, 256, 80, 64, 21, "global_residual", 0),
    ("hisq1024", 40, 2048, 24, 1024, 22, "model.layers.0.mlp.down_proj", 17),
    ("plain", 33, 200, 48, None, 23, None, None),
]


def linear_inputs(rows: int, fin: int, fout: int, seed: int):
    x = outlier_rows(rows, fin, seed=seed, outliers=max(1, fin // 200)).to(torch.bfloat16)
    g = torch.Generator().manual_seed(seed + 1000)
    w = (torch.randn(fout, fin, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(fout, generator=g) * 0.1).to(torch.bfloat16)
    return x, w, b


ATTENTION_CASES = [
    # (tag, B, H, KV, Sq, Sk, causal, normalizer, qk_quant, pv_quant, seed)
    ("gqa_causal", 1, 4, 2, 160, 160, True, "quantized_same", True, True, 31),
    ("mha_noncausal", 1, 2, 2, 150, 333, False, "unquantized", True, True, 32),
    ("bottom_right", 2, 2, 1, 70, 260, True, "quantized_same", True, True, 33),
    ("pv_only", 1, 2, 1, 130, 130, True, "unquantized", False, True, 34),
]


def attention_inputs(b: int, h: int, kv: int, sq: int, sk: int, seed: int, d: int = 128):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, sq, d, generator=g).to(torch.bfloat16)
    k = torch.randn(b, kv, sk, d, generator=g).to(torch.bfloat16)
    v = torch.randn(b, kv, sk, d, generator=g).to(torch.bfloat16)
    return q, k, v


def config1_linear_inputs():
    """BASELINE config 1's QuantLinear: X [2048, 4096] ~N(0,1) with 8 random channels x20
    (bf16), W [4096, 4096] ~N(0, 0.02) (bf16), seeds 0 and 1."""
    x = outlier_rows(2048, 4096, seed=0, outliers=8).to(torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    w = (torch.randn(4096, 4096, generator=g) * 0.02).to(torch.bfloat16)
    return x, w


def c2_projection_inputs(tokens: int = 512):
    """A config-2 projection (q_proj 4096 -> 4096): activations ~N(0,1) with 0.5 % outlier
    channels x20 (20 of 4096), W ~N(0, 0.02), seeds 2 and 3."""
    x = outlier_rows(tokens, 4096, seed=2, outliers=20).to(torch.bfloat16)
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(4096, 4096, generator=g) * 0.02).to(torch.bfloat16)
    return x, w
