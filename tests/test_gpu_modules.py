"""GPU tests of the reference-facing module layer: FakeQuantLinear, the HF attention
backend, the Qwen3 Q/K transform and the Wan2.2 drop-ins, each against the
reference fixtures or the oracle on the same inputs."""

from __future__ import annotations

import json
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import load_golden
from inputs import ATTENTION_CASES, LINEAR_CASES, attention_inputs, linear_inputs, sha
from oracle import attention as oatt
from oracle import hif4 as oh
from oracle import linear as olin

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATT_REL_FRO = 5e-3
ATT_MAX_ABS = 6e-2


def _bf16(bits: np.ndarray) -> np.ndarray:
    return oh.bf16_to_f32(bits)


def _close_attention(out: torch.Tensor, ref: np.ndarray) -> None:
    o = out.float().cpu().numpy()
    err = o - ref
    rel = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
    assert rel <= ATT_REL_FRO and float(np.abs(err).max()) <= ATT_MAX_ABS, rel


@pytest.mark.parametrize("levels", ["123", "12"])
@pytest.mark.parametrize("case", LINEAR_CASES, ids=[c[0] for c in LINEAR_CASES])
def test_fake_quant_linear_matches_reference_module(levels: str, case, monkeypatch) -> None:
    """FakeQuantLinear built from the same Linear and rotation gives the reference's y
    (bf16 GEMM output: within one bf16 rounding of the exact product)."""
    from faquant_b200.hisq_rotation import derive_hisq_rotation
    from faquant_b200.quantization import FakeQuantLinear

    monkeypatch.setenv("FAQUANT_HIF4_SCALE_LEVELS", levels)
    monkeypatch.delenv("FAQUANT_HIF4_ACT_SCALE_LEVELS", raising=False)
    g = load_golden(f"linear_{levels}")
    tag, rows, fin, fout, block, seed, rname, rseed = case
    x, w, b = linear_inputs(rows, fin, fout, seed)
    lin = torch.nn.Linear(fin, fout, bias=True).to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(b)
    kwargs = {}
    if rname is not None:
        rot = derive_hisq_rotation(rname, fin, seed=rseed, block_size=block)
        kwargs = dict(input_rotation_signs=rot.signs, input_rotation_permutation=rot.permutation,
                      input_rotation_block_size=block)
    mod = FakeQuantLinear(lin, quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64,
                          symmetric=True, clip_ratio=1.0, **kwargs).to(DEV)
    assert np.array_equal(mod.weight.detach().cpu().view(torch.int16).numpy().view(np.uint16), g[f"{tag}_wq"])
    y = mod(x.to(DEV)).float().cpu().numpy()
    ref = _bf16(g[f"{tag}_y"])
    exact = _bf16(g[f"{tag}_xq"]) @ _bf16(g[f"{tag}_wq"]).T + b.float().numpy()
    assert np.all(np.abs(y - exact) <= 2.0**-8 * np.abs(exact) + 1e-4 * np.abs(exact).max())
    assert np.all(np.abs(y - ref) <= 2.0**-7 * np.abs(ref) + 1e-3)


def test_replace_linear_with_fake_quant_reads_faquant_attributes() -> None:
    from faquant_b200.hisq_rotation import derive_hisq_rotation
    from faquant_b200.quantization import FakeQuantLinear, replace_linear_with_fake_quant

    parent = torch.nn.Module()
    parent.proj = torch.nn.Linear(256, 64, bias=False).to(torch.bfloat16).to(DEV)
    rot = derive_hisq_rotation("replace", 256, seed=3, block_size=64)
    parent.proj.faquant_input_rotation_signs = rot.signs
    parent.proj.faquant_input_rotation_permutation = rot.permutation
    parent.proj.faquant_input_rotation_block_size = 64
    config = SimpleNamespace(quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64,
                             symmetric=True, clip_ratio=1.0)
    replace_linear_with_fake_quant(parent, "proj", config, weights_prequantized=False)
    assert isinstance(parent.proj, FakeQuantLinear)
    assert parent.proj.input_rotation_block_size == 64
    x = torch.randn(8, 256, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    y = parent.proj(x.to(DEV)).float().cpu().numpy()
    ref = olin.fake_quant_linear(x.float().numpy(), parent.proj.weight.float().cpu().numpy(), None, levels="123",
                                 signs=rot.signs.numpy(), permutation=rot.permutation.numpy(), block=64)
    assert np.all(np.abs(y - ref) <= 2.0**-8 * np.abs(ref) + 1e-3)


def _module(causal: bool, normalizer: str, qk: bool, pv: bool) -> SimpleNamespace:
    from faquant_b200.attention import new_simulated_attention_stats

    return SimpleNamespace(
        is_causal=causal, training=False,
        faquant_attention_query_chunk_size=256, faquant_attention_key_chunk_size=128,
        faquant_qk_matmul_quant=qk, faquant_pv_matmul_quant=pv, faquant_pv_normalizer_mode=normalizer,
        faquant_matmul_quant_kwargs={"quant_format": "hif4", "bits": 4, "group_size": 64, "symmetric": True,
                                     "clip_ratio": 1.0},
        faquant_simulated_attention_stats=new_simulated_attention_stats(),
    )


@pytest.mark.parametrize("case", ATTENTION_CASES, ids=[c[0] for c in ATTENTION_CASES])
def test_attention_backend_matches_reference_fixture(case) -> None:
    from faquant_b200.attention import simulated_flash_attention_forward

    g = load_golden("attention")
    tag, b, h, kv, sq, sk, causal, normalizer, qk, pv, seed = case
    q, k, v = attention_inputs(b, h, kv, sq, sk, seed)
    assert str(g[f"{tag}_in_sha"]) == sha(q) + sha(k) + sha(v)
    module = _module(causal, normalizer, qk, pv)
    out, weights = simulated_flash_attention_forward(module, q.to(DEV), k.to(DEV), v.to(DEV), None,
                                                     scaling=128**-0.5)
    assert weights is None and out.shape == (b, sq, h, 128) and out.dtype == torch.bfloat16
    _close_attention(out, _bf16(g[f"{tag}_out"]))
    assert module.faquant_simulated_attention_stats == json.loads(bytes(g[f"{tag}_stats"]).decode())


def test_attention_backend_decode_steps_with_qdq_cache() -> None:
    """Prefill, then three decode steps through the backend: the K/V QDQ caches grow by
    appending one quantized position (bit-identical to re-quantizing the whole cache, as
    the reference's _cached_decode_quantize guarantees) and each step -- run by the decode
    kernel -- matches the oracle over the whole cache."""
    from faquant_b200 import ops
    from faquant_b200.attention import simulated_flash_attention_forward

    module = _module(True, "quantized_same", True, True)
    g = torch.Generator().manual_seed(11)
    b, h, kv, s0 = 1, 8, 2, 300
    q = torch.randn(b, h, s0 + 3, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(b, kv, s0 + 3, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(b, kv, s0 + 3, 128, generator=g).to(torch.bfloat16)
    simulated_flash_attention_forward(module, q[:, :, :s0].to(DEV), k[:, :, :s0].to(DEV), v[:, :, :s0].to(DEV), None)
    for step in range(3):
        n = s0 + step + 1
        out, _ = simulated_flash_attention_forward(module, q[:, :, n - 1:n].to(DEV), k[:, :, :n].to(DEV),
                                                   v[:, :, :n].to(DEV), None)
        assert torch.equal(module.faquant_k_matmul_qdq_cache, ops.qk_prep(k[:, :, :n].to(DEV), levels="123",
                                                                           rotate=False)[0])
        assert torch.equal(module.faquant_v_matmul_qdq_cache, ops.qk_prep(v[:, :, :n].to(DEV), levels="123",
                                                                           rotate=False)[0])
        ref = oatt.attention(q[:, :, n - 1:n].float().numpy(), k[:, :, :n].float().numpy(),
                             v[:, :, :n].float().numpy(), causal=True, normalizer="quantized_same")
        _close_attention(out, ref)


def test_attention_backend_all_valid_mask_is_the_unmasked_path() -> None:
    from faquant_b200.attention import simulated_flash_attention_forward

    q, k, v = attention_inputs(1, 4, 2, 200, 200, 5)
    mask = torch.ones(1, 200, dtype=torch.long, device=DEV)
    a, _ = simulated_flash_attention_forward(_module(True, "quantized_same", True, True), q.to(DEV), k.to(DEV),
                                             v.to(DEV), mask)
    b_, _ = simulated_flash_attention_forward(_module(True, "quantized_same", True, True), q.to(DEV), k.to(DEV),
                                              v.to(DEV), None)
    assert torch.equal(a, b_)


def test_qwen3_qk_pretransform_matches_reference_fixture() -> None:
    from faquant_b200.qwen3 import qk_pretransform

    g = load_golden("qk_prep")
    q = torch.from_numpy(g["q"].view(np.int16)).view(torch.bfloat16).to(DEV)
    k = torch.from_numpy(g["k"].view(np.int16)).view(torch.bfloat16).to(DEV)
    module = SimpleNamespace(faquant_qk_smooth_scale=torch.from_numpy(g["scale"]).to(DEV),
                             faquant_qk_key_offset=torch.from_numpy(g["offset"])[:, None, :].to(DEV),
                             faquant_qk_rotation=True)
    qo, ko = qk_pretransform(module, q, k)
    assert np.array_equal(qo.cpu().view(torch.int16).numpy().view(np.uint16), g["q_out"])
    assert np.array_equal(ko.cpu().view(torch.int16).numpy().view(np.uint16), g["k_out"])


def test_wan_hif4_attention_and_flash_attention_match_oracle() -> None:
    from faquant_b200.wan22 import faquant_qdq, hif4_attention, make_flash_attention, rotate_heads

    g = torch.Generator().manual_seed(61)
    q = torch.randn(1, 300, 4, 128, generator=g)  # Wan layout [B, L, H, D], fp32 under autocast
    k = torch.randn(1, 300, 4, 128, generator=g)
    v = torch.randn(1, 300, 4, 128, generator=g)
    flash = make_flash_attention(faquant_qdq("123"), quantized_normalizer=True, qk_rotation=True)
    out = flash(q.to(DEV), k.to(DEV), v.to(DEV))
    qr, kr = oatt.qk_pretransform(q.transpose(1, 2).numpy(), k.transpose(1, 2).numpy())
    vb = oh.bf16_round(v.transpose(1, 2).numpy())
    ref = oatt.attention(qr, kr, vb, causal=False, normalizer="quantized_same")
    _close_attention(out, ref)
    # lower-level pieces: rotate_heads (bit-exact) and hif4_attention on [L, H, D]
    rh = rotate_heads(q[0].to(DEV))
    assert np.array_equal(rh.float().cpu().numpy(), qr[0].transpose(1, 0, 2))
    qd = torch.from_numpy(oh.fake_quantize(qr[0].transpose(1, 0, 2))).to(torch.bfloat16).to(DEV)
    kd = torch.from_numpy(oh.fake_quantize(kr[0].transpose(1, 0, 2))).to(torch.bfloat16).to(DEV)
    vd = torch.from_numpy(oh.fake_quantize(vb[0].transpose(1, 0, 2))).to(torch.bfloat16).to(DEV)
    o2 = hif4_attention(qd, kd, vd, quantized_normalizer=True)
    _close_attention(o2.unsqueeze(0), ref)


def test_wan_hif4_linear_with_fused_reader_rotation() -> None:
    from faquant_b200.hisq_rotation import derive_hisq_rotation
    from faquant_b200.wan22 import HiF4Linear, faquant_qdq

    rot = derive_hisq_rotation("model.layers.0.input_layernorm", 5120, seed=17, block_size=64)
    lin = torch.nn.Linear(5120, 256, bias=True).to(torch.bfloat16)
    qdq = faquant_qdq("123", signs=rot.signs.to(DEV), permutation=rot.permutation.to(DEV), block=64)
    mod = HiF4Linear(lin, weight_qdq=faquant_qdq("123"), input_qdq=qdq, device=DEV).to(DEV)
    x = torch.randn(300, 5120, generator=torch.Generator().manual_seed(62))
    y = mod(x.to(DEV)).float().cpu().numpy()
    ref = olin.fake_quant_linear(x.numpy(), mod.weight.float().cpu().numpy(), lin.bias.detach().float().numpy(),
                                 levels="123", dtype="f32", signs=rot.signs.numpy(),
                                 permutation=rot.permutation.numpy(), block=64)
    assert np.all(np.abs(y - ref) <= 2.0**-8 * np.abs(ref) + 1e-3 * np.abs(ref).max())


def test_chunked_prefill_equals_one_pass() -> None:
    """The long-context workflow prefills in chunks of whole query tiles against the growing
    cache (eval_longbench.py:505-540) and relies on every row being computed exactly as in
    one pass: the key tiles are anchored at key 0 whatever the query chunk, and the K/V HiF4
    operands are token-local, so the chunked rows are bit-identical to the single pass."""
    from faquant_b200.attention import simulated_flash_attention_forward

    g = torch.Generator().manual_seed(12)
    b, h, kv, s = 1, 8, 2, 768
    q = torch.randn(b, h, s, 128, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(b, kv, s, 128, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(b, kv, s, 128, generator=g).to(torch.bfloat16).to(DEV)
    whole, _ = simulated_flash_attention_forward(_module(True, "quantized_same", True, True), q, k, v, None)
    module = _module(True, "quantized_same", True, True)
    first, _ = simulated_flash_attention_forward(module, q[:, :, :512], k[:, :, :512], v[:, :, :512], None)
    second, _ = simulated_flash_attention_forward(module, q[:, :, 512:], k, v, None)
    assert torch.equal(first, whole[:, :512]) and torch.equal(second, whole[:, 512:])
    # the workflow then frees the QDQ copies (decode runs on the BF16 model)
    assert module.faquant_k_matmul_qdq_cache.shape == (b, kv, s, 128)
