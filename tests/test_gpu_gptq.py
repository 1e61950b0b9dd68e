"""GPTQ with HiF4 grids on the GPU (``faquant_b200.gptq.GPTQ``) against the reference's CPU
solver (``src/faquant/gptq.py``), on the fixtures ``tests/golden/make_golden.py`` wrote by
running it: the small case of ``gptq.npz`` (48 x 256) and, at the deployed GPTQ settings,
a full-Hessian layer (256 x 1024, block 128) and a block-diagonal one (128 x 512, 64-column
Hessian blocks). The inputs are rebuilt from the same seeds.

The GPU solver performs the reference's arithmetic; its fp32 GEMMs (the Hessian, the
lazy update) and the Cholesky factorization sum in another order than the CPU libraries,
so a value can differ in its last bits before it is quantized, but HiF4's decisions are
discrete and did not sit on such a boundary in these cases (an fp64-accumulated Hessian
in the reference's own solver gives the same result too): the quantized weights and every
metadata field are required to be equal bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from inputs import outlier_rows

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _solve(n: int, k: int, seed: int, x: torch.Tensor, hblock: int | None):
    from faquant_b200.gptq import GPTQ

    torch.manual_seed(seed)
    lin = torch.nn.Linear(k, n, bias=False)  # the reference draws the init, then N(0, 0.02)
    with torch.no_grad():
        lin.weight.normal_(0.0, 0.02)
    lin = lin.to(DEV)
    gp = GPTQ(lin, hessian_block_size=hblock)
    gp.add_batch(x.to(DEV))
    stats = gp.quantize(quant_format="hif4", bits=4, group_size=64, damp=0.01, block_size=128,
                        capture_hif4_metadata=True)
    assert stats.samples == x.shape[0] and stats.damp_multiplier == 1.0
    return lin, lin.faquant_hif4_qat_parameters


def _agree(got: np.ndarray, ref: np.ndarray, what: str) -> None:
    bad = int((got != ref).sum())
    assert bad == 0, f"{what}: {bad} of {ref.size} differ"


def test_small_case_matches_the_reference_solver() -> None:
    g = load_golden("gptq")
    x = torch.randn(512, 256, generator=torch.Generator().manual_seed(52))
    lin, meta = _solve(48, 256, 51, x, None)
    _agree(_bits(lin.weight), g["w"], "weights")
    _agree(meta.scale.reshape(48, 4).cpu().numpy(), g["scale"], "scale")
    _agree(meta.reciprocal.reshape(48, 4).cpu().numpy(), g["rec"], "reciprocal")
    _agree(meta.scale_lv2_exponent.reshape(48, 4, 8).cpu().numpy(), g["lv2"], "lv2")
    _agree(meta.scale_lv3_exponent.reshape(48, 4, 16).cpu().numpy(), g["lv3"], "lv3")


@pytest.mark.parametrize("tag,n,k,hblock,seed", [("full", 256, 1024, None, 61), ("blockdiag", 128, 512, 64, 62)])
def test_deployed_settings_match_the_reference_solver(tag: str, n: int, k: int, hblock: int | None,
                                                      seed: int) -> None:
    g = load_golden("gptq_cases")
    x = outlier_rows(4096, k, seed=seed + 1, outliers=max(1, k // 100))
    lin, meta = _solve(n, k, seed, x, hblock)
    groups = k // 64
    _agree(_bits(lin.weight), g[f"{tag}_w"], "weights")
    _agree(meta.scale.reshape(n, groups).cpu().numpy(), g[f"{tag}_scale"], "scale")
    _agree(meta.scale_lv2_exponent.reshape(n, groups, 8).cpu().numpy(), g[f"{tag}_lv2"], "lv2")
    _agree(meta.scale_lv3_exponent.reshape(n, groups, 16).cpu().numpy(), g[f"{tag}_lv3"], "lv3")


def test_gptq_weight_packs_exactly_and_runs_in_the_packed_gemm() -> None:
    """The solved weight with its captured metadata packs exactly (K2 reports no value it
    does not reproduce) and serves a packed FakeQuantLinear."""
    from faquant_b200 import ops
    from faquant_b200.quantization import FakeQuantLinear

    x = outlier_rows(4096, 1024, seed=62, outliers=10)
    lin, meta = _solve(256, 1024, 61, x, None)
    codes, packed_meta, bad = ops.hif4_pack_weight(lin.weight.detach(), scale=meta.scale.reshape(256, 16),
                                                   lv2=meta.scale_lv2_exponent.reshape(256, 16, 8),
                                                   lv3=meta.scale_lv3_exponent.reshape(256, 16, 16))
    assert bad == 0
    assert torch.equal(ops.hif4_dequantize(codes, packed_meta, 1024), lin.weight.detach().to(torch.bfloat16))
    mod = FakeQuantLinear(lin.to(torch.bfloat16), quant_format="hif4", bits=4, weight_group_size=64,
                          activation_group_size=64, symmetric=True, clip_ratio=1.0, quantize_weight=False)
    mod.use_packed(codes, packed_meta)
    xs = torch.randn(300, 1024, device=DEV).to(torch.bfloat16)
    ref = ops.gemm_bf16(ops.hif4_quantize(xs, levels="123")[0], lin.weight.detach().to(torch.bfloat16))
    with torch.no_grad():
        assert torch.equal(mod(xs), ref)
