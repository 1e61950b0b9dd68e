"""GPU tests against the reference implementation itself, on the same GPU.

The reference checkout is pip-installed (offline) under ``baseline/_ref``; that folder is
git-ignored but travels with the repository to the GPU box. These tests import the
reference's own modules from it and compare, on identical inputs:

* K5 with the reference's Triton kernel ``wan22_attention.hif4_attention`` (Wan2.2's
  non-causal HiF4 attention, both normalizer modes);
* the HF attention backend with the reference's PyTorch simulator
  ``simulated_flash_attention_forward`` (causal GQA, HiF4 Q/K/P/V, P-Reordering) at a
  sequence length the CPU fixtures do not reach;
* ``FakeQuantLinear`` with the reference's ``FakeQuantLinear`` (HiSQ1024 rotation,
  three-level HiF4): the RTN weight grid bit for bit, the outputs up to the GEMM's fp32
  summation order.

Without that install (or if it does not import) the tests skip.
"""

from __future__ import annotations

import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
REF_DIR = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module")
def ref():
    if not (REF_DIR / "faquant").is_dir():
        pytest.skip("no reference install under baseline/_ref")
    sys.path.insert(0, str(REF_DIR))
    try:
        import faquant.hisq_rotation as hr
        import faquant.quantization as q
        import faquant.simulated_flash_attention as sfa
        import faquant.wan22_attention as wan
    except Exception as e:  # noqa: BLE001 - an unusable install skips, it does not fail
        pytest.skip(f"reference install does not import: {type(e).__name__}: {e}")
    return SimpleNamespace(hr=hr, q=q, sfa=sfa, wan=wan)


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("quantized_normalizer", [True, False])
def test_k5_matches_the_reference_triton_kernel(ref, quantized_normalizer) -> None:
    from faquant_b200 import ops

    seq, heads, d = 3000, 4, 128
    g = torch.Generator(device=DEV).manual_seed(5)
    q, k, v = (ops.qk_prep(torch.randn(1, heads, seq, d, device=DEV, generator=g).to(torch.bfloat16),
                           levels="123", rotate=rot)[0] for rot in (True, True, False))
    theirs = ref.wan.hif4_attention(q[0].transpose(0, 1), k[0].transpose(0, 1), v[0].transpose(0, 1),
                                    softmax_scale=d**-0.5, quantize_p=True, quantized_normalizer=quantized_normalizer)
    ours = ops.hif4_attention(q, k, v, scale=d**-0.5, causal=False, p_levels="123",
                              quantized_normalizer=quantized_normalizer)[0]
    assert ours.shape == theirs.shape
    assert _rel(ours, theirs) <= 5e-3


def _namespace(stats_factory) -> SimpleNamespace:
    return SimpleNamespace(
        is_causal=True, training=False,
        faquant_attention_query_chunk_size=256, faquant_attention_key_chunk_size=128,
        faquant_qk_matmul_quant=True, faquant_pv_matmul_quant=True, faquant_pv_normalizer_mode="quantized_same",
        faquant_matmul_quant_kwargs={"quant_format": "hif4", "bits": 4, "group_size": 64, "symmetric": True,
                                     "clip_ratio": 1.0},
        faquant_simulated_attention_stats=stats_factory(),
    )


def test_attention_backend_matches_the_reference_simulator(ref) -> None:
    from faquant_b200.attention import new_simulated_attention_stats, simulated_flash_attention_forward

    b, h, kv, s, d = 1, 8, 2, 2048, 128
    g = torch.Generator(device=DEV).manual_seed(6)
    q = torch.randn(b, h, s, d, device=DEV, generator=g).to(torch.bfloat16)
    k = torch.randn(b, kv, s, d, device=DEV, generator=g).to(torch.bfloat16)
    v = torch.randn(b, kv, s, d, device=DEV, generator=g).to(torch.bfloat16)
    theirs, _ = ref.sfa.simulated_flash_attention_forward(_namespace(ref.sfa.new_simulated_attention_stats), q, k, v,
                                                          None, scaling=d**-0.5)
    ours, _ = simulated_flash_attention_forward(_namespace(new_simulated_attention_stats), q, k, v, None,
                                                scaling=d**-0.5)
    assert ours.shape == theirs.shape == (b, s, h, d)
    assert _rel(ours, theirs) <= 5e-3


def test_fake_quant_linear_matches_the_reference_module(ref) -> None:
    from faquant_b200.quantization import FakeQuantLinear

    n, k = 1024, 4096
    rot = ref.hr.derive_hisq_rotation("model.layers.0.self_attn.q_proj", k, seed=17, block_size=1024)
    g = torch.Generator(device=DEV).manual_seed(7)
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(512, k, device=DEV, generator=g).to(torch.bfloat16)
    kw = dict(quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64, symmetric=True,
              clip_ratio=1.0, quantize_weight=True, input_rotation_signs=rot.signs.to(DEV),
              input_rotation_permutation=rot.permutation.to(DEV), input_rotation_block_size=1024)

    def linear():
        lin = torch.nn.Linear(k, n, bias=False, device=DEV, dtype=torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(w)
        return lin

    theirs_mod, ours_mod = ref.q.FakeQuantLinear(linear(), **kw), FakeQuantLinear(linear(), **kw)
    assert torch.equal(ours_mod.weight, theirs_mod.weight)  # the RTN HiF4 grid, bit for bit
    with torch.no_grad():
        theirs, ours = theirs_mod(x), ours_mod(x)
    assert ours.shape == theirs.shape and ours.dtype == theirs.dtype
    assert _rel(ours, theirs) <= 2e-3
