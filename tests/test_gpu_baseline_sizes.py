"""GPU parity at the BASELINE configurations' own sizes.

* Config 1 in full, against fixtures the reference itself wrote
  (``tests/golden/make_golden.py``): the attention (B=1, 32/8 heads, S=2048, causal,
  post-RoPE Hadamard, HiF4 Q/K/P/V, P-Reordering) through this package's HF attention
  backend, and the QuantLinear (X [2048, 4096] with outliers, ``rbh_r64`` reader rotation,
  two-level HiF4, RTN) through ``FakeQuantLinear``; plus one config-2 projection
  (HiSQ1024, three-level). Sampled rows are compared value by value and every row through
  its sum.
* Configs 3 and 4 at full size (S=32768 causal GQA with Smooth-QK; S=75600 non-causal,
  40 heads): the whole attention runs on the GPU, then the oracle recomputes on the CPU
  the first, a middle and the last query tile of one head per KV group (config 3) or of
  four heads (config 4) over the full key range. Each output row depends only on its own
  query and all keys, so those rows must match the full computation; the method itself is
  pinned against the reference at config 1 (``test_oracle_golden.py``). These rows reach
  what small cases cannot: the running max over 256 / 591 key tiles, fp32 sums of 32K /
  75K P.V terms, the causal tile skip at depth and the ragged last tile of 80 queries.
Full-width layers of configs 4 and 5 are checked stage by stage in
``test_gpu_tensor_parallel.py``.
"""

from __future__ import annotations

import json
import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import load_golden
from inputs import attention_inputs, c2_projection_inputs, config1_linear_inputs, sha
from oracle import attention as oatt
from oracle import hif4 as oh

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
ATT_REL_FRO = 5e-3  # HiF4 attention: hardware ex2 vs CPU exp can move P codes
ATT_MAX_ABS = 6e-2


def _check_attention(got: np.ndarray, ref: np.ndarray) -> None:
    err = got - ref
    rel = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
    assert rel <= ATT_REL_FRO and float(np.abs(err).max()) <= ATT_MAX_ABS, (rel, float(np.abs(err).max()))


def _module():
    from faquant_b200.attention import new_simulated_attention_stats

    return SimpleNamespace(
        is_causal=True, training=False,
        faquant_attention_query_chunk_size=256, faquant_attention_key_chunk_size=128,
        faquant_qk_matmul_quant=True, faquant_pv_matmul_quant=True, faquant_pv_normalizer_mode="quantized_same",
        faquant_matmul_quant_kwargs={"quant_format": "hif4", "bits": 4, "group_size": 64, "symmetric": True,
                                     "clip_ratio": 1.0},
        faquant_simulated_attention_stats=new_simulated_attention_stats(),
    )


def test_config1_attention_in_full_matches_the_reference_simulator() -> None:
    from faquant_b200 import ops
    from faquant_b200.attention import simulated_flash_attention_forward

    g = load_golden("config1_attention")
    q, k, v = attention_inputs(1, 32, 8, 2048, 2048, seed=0)
    assert str(g["in_sha"]) == sha(q) + sha(k) + sha(v)
    # the post-RoPE transform of qwen3._attention_forward (Hadamard, one bf16 cast); the
    # backend then quantizes Q/K/V itself, as the reference simulator does
    qh = ops.qk_prep(q.to(DEV), levels=None, rotate=True)[0]
    kh = ops.qk_prep(k.to(DEV), levels=None, rotate=True)[0]
    module = _module()
    out, _ = simulated_flash_attention_forward(module, qh, kh, v.to(DEV), None, scaling=128**-0.5)
    assert out.shape == (1, 2048, 32, 128)
    rows = g["rows"]
    _check_attention(out[0, torch.from_numpy(rows).to(DEV)].float().cpu().numpy(), oh.bf16_to_f32(g["out_rows"]))
    # every (query, head) through its sum over head_dim
    sums = out[0].float().sum(dim=-1).cpu().numpy()
    ref = g["head_sums"]
    assert np.linalg.norm(sums - ref) <= 1e-2 * np.linalg.norm(ref)
    assert module.faquant_simulated_attention_stats == json.loads(bytes(g["stats"]).decode())


@pytest.mark.parametrize("name", ["config1_linear", "c2_projection"])
def test_baseline_size_linear_matches_the_reference_module(name: str, monkeypatch) -> None:
    from faquant_b200.hisq_rotation import derive_hisq_rotation
    from faquant_b200.quantization import FakeQuantLinear

    g = load_golden(name)
    levels = str(g["levels"])
    monkeypatch.setenv("FAQUANT_HIF4_SCALE_LEVELS", levels)
    monkeypatch.delenv("FAQUANT_HIF4_ACT_SCALE_LEVELS", raising=False)
    if name == "config1_linear":
        x, w = config1_linear_inputs()
        rot, block = derive_hisq_rotation("global_residual", 4096, seed=0, block_size=64), 64
    else:
        x, w = c2_projection_inputs()
        rot, block = derive_hisq_rotation("model.layers.0.self_attn.q_proj", 4096, seed=17, block_size=1024), 1024
    assert str(g["in_sha"]) == sha(x) + sha(w)
    lin = torch.nn.Linear(4096, 4096, bias=False, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w.to(DEV))
    mod = FakeQuantLinear(lin, quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64,
                          symmetric=True, clip_ratio=1.0, input_rotation_signs=rot.signs.to(DEV),
                          input_rotation_permutation=rot.permutation.to(DEV), input_rotation_block_size=block)
    assert sha(mod.dequantized_weight().cpu()) == str(g["wq_sha"])  # the RTN grid, bit for bit
    with torch.no_grad():
        y = mod(x.to(DEV))
    rows = torch.from_numpy(g["rows"]).to(DEV)
    got = y[rows].float().cpu().numpy()
    ref = oh.bf16_to_f32(g["y_rows"])
    # two fp32 sums of the same exact products in different orders, each rounded to bf16
    assert np.all(np.abs(got - ref) <= 2.0**-7 * np.abs(ref) + 1e-3 * np.abs(ref).max())
    sums = y.double().sum(dim=1).cpu().numpy()
    assert np.all(np.abs(sums - g["row_sums"]) <= 1e-2 * np.abs(g["row_sums"]).max())


def _sampled_rows_check(qd, kd, vd, out, heads, kv_of, tiles, causal) -> None:
    """Oracle rows of query tiles ``tiles`` (start, end) of ``heads`` over all keys."""
    s = qd.shape[2]
    kvh = sorted({kv_of(h) for h in heads})
    kk = kd[0, kvh].float().cpu().numpy()[None]
    vv = vd[0, kvh].float().cpu().numpy()[None]
    sel = [kvh.index(kv_of(h)) for h in heads]
    for start, end in tiles:
        rows = np.arange(start, end)
        qq = qd[0, heads, start:end].float().cpu().numpy()[None]
        ref = oatt.attention(qq, kk[:, sel], vv[:, sel], causal=causal, scale=128**-0.5,
                             normalizer="quantized_same", operands_quantized=True, query_positions=rows,
                             full_queries=s, return_f32=True)
        got = out[0, start:end][:, heads].float().cpu().numpy()[None]
        _check_attention(got, ref)


def test_config3_attention_sampled_rows_at_full_size() -> None:
    """B=1, 32/8 heads, S=32768, causal GQA, Smooth-QK scales
    LogUniform(0.5, 2), post-RoPE Hadamard, HiF4 group 64, P-Reordering."""
    from faquant_b200 import ops

    s, hq, hkv = 32768, 32, 8
    g = torch.Generator(device=DEV).manual_seed(3)
    q = torch.randn(1, hq, s, 128, device=DEV, generator=g).to(torch.bfloat16)
    k = torch.randn(1, hkv, s, 128, device=DEV, generator=g).to(torch.bfloat16)
    v = torch.randn(1, hkv, s, 128, device=DEV, generator=g).to(torch.bfloat16)
    smooth = torch.exp(torch.empty(128, device=DEV).uniform_(math.log(0.5), math.log(2.0), generator=g))
    qd = ops.qk_prep(q, levels="123", rotate=True, smooth_scale=smooth, smooth_mode="mul")[0]
    kd = ops.qk_prep(k, levels="123", rotate=True, smooth_scale=smooth, smooth_mode="div")[0]
    vd = ops.qk_prep(v, levels="123", rotate=False)[0]
    del q, k, v
    out = ops.hif4_attention(qd, kd, vd, scale=128**-0.5, causal=True, p_levels="123", quantized_normalizer=True)
    group = hq // hkv
    heads = [group * j + j % group for j in range(hkv)]  # one head of every KV group
    tiles = [(0, 128), (s // 2, s // 2 + 128), (s - 128, s)]
    _sampled_rows_check(qd, kd, vd, out, heads, lambda h: h // group, tiles, causal=True)


def test_config4_attention_sampled_rows_at_full_size() -> None:
    """BASELINE config 4's self-attention: S=75600 (21 x 45 x 80), 40 heads, non-causal,
    post-RoPE Hadamard, HiF4 group 64, P-Reordering; the last query tile holds 80 rows."""
    from faquant_b200 import ops

    s, h = 75600, 40
    g = torch.Generator(device=DEV).manual_seed(4)
    qd = ops.qk_prep(torch.randn(1, h, s, 128, device=DEV, generator=g).to(torch.bfloat16), levels="123",
                     rotate=True)[0]
    kd = ops.qk_prep(torch.randn(1, h, s, 128, device=DEV, generator=g).to(torch.bfloat16), levels="123",
                     rotate=True)[0]
    vd = ops.qk_prep(torch.randn(1, h, s, 128, device=DEV, generator=g).to(torch.bfloat16), levels="123",
                     rotate=False)[0]
    out = ops.hif4_attention(qd, kd, vd, scale=128**-0.5, causal=False, p_levels="123", quantized_normalizer=True)
    last = s - s % 128
    tiles = [(0, 128), (37760, 37888), (last, s)]
    _sampled_rows_check(qd, kd, vd, out, [0, 13, 27, 39], lambda hh: hh, tiles, causal=False)
