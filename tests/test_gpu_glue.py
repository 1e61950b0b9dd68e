"""GPU tests of the fused decoder glue: faq_rms_norm, faq_silu_mul, the Qwen3 K4 variant
faq_qk_norm_rope_prep, and Wan's faq_layer_norm, faq_gelu_tanh, faq_row_sumsq and K4
variant faq_wan_qk_prep, against torch's own ops on the CPU (the reference's glue) and
the oracle. Where the ops are pure bf16-rounded elementwise math (RoPE, the HiF4 steps)
the results are bit-exact; the row reductions (RMSNorm, LayerNorm) and exp/tanh (SiLU,
GELU) sum or round differently from torch's CPU kernels, so those are held to one bf16
ulp."""

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


def test_layer_norm_matches_wan_layernorm() -> None:
    from faquant_b200 import ops

    g = torch.Generator().manual_seed(4)
    for k in (64, 512, 2048, 5120, 13824):
        x = (torch.randn(29, k, generator=g) * 3 + 0.7).to(torch.bfloat16)
        ref = torch.nn.functional.layer_norm(x.float(), (k,), eps=1e-6).to(torch.bfloat16)
        _within_ulp(ops.layer_norm(x.to(DEV), 1e-6), ref)
    assert ops.layer_norm(torch.zeros(0, 64, dtype=torch.bfloat16, device=DEV), 1e-6).shape == (0, 64)


def test_gelu_tanh_matches_torch() -> None:
    from faquant_b200 import ops

    x = (torch.randn(41, 1376, generator=torch.Generator().manual_seed(5)) * 4).to(torch.bfloat16)
    ref = torch.nn.functional.gelu(x.float(), approximate="tanh").to(torch.bfloat16).float()
    got = ops.gelu_tanh(x.to(DEV)).float().cpu()
    # one bf16 ulp; the far negative tail, where 1 + tanh cancels, to an absolute 1e-5
    assert torch.all((got - ref).abs() <= 2.0**-7 * ref.abs() + 1e-5)


def test_row_sumsq_segments() -> None:
    from faquant_b200 import ops

    g = torch.Generator().manual_seed(6)
    x = torch.randn(300, 3 * 640, generator=g).to(torch.bfloat16)
    for cols, segments in ((2 * 640, 10), (2 * 640, 2), (640, 1)):  # 128-wide heads, 640-wide halves, whole
        got = ops.row_sumsq(x.to(DEV)[:, :cols], segments=segments).cpu().double()
        ref = x[:, :cols].double().pow(2).reshape(300, segments, -1).sum(-1)
        assert got.shape == (300, segments)
        assert torch.allclose(got, ref, rtol=1e-5, atol=0)


@pytest.mark.parametrize("act,block,levels", [("swiglu", 64, "123"), ("swiglu", 256, "12"),
                                              ("gelu_tanh", 64, "123"), ("gelu_tanh", 8, "13")])
def test_quantize_act_equals_activation_then_quantize(act: str, block: int, levels: str) -> None:
    """faq_hif4_quantize_act (the activation fused into the row-parallel input
    quantization) gives the bits of faq_silu_mul / faq_gelu_tanh followed by
    faq_hif4_quantize: dequantized values, codes and meta, with and without input_scale."""
    from faquant_b200 import ops

    g = torch.Generator().manual_seed(block + len(act))
    rows, k = 333, 1536
    width = 2 * k if act == "swiglu" else k
    x = (torch.randn(rows, width, generator=g) * 3).to(torch.bfloat16).to(DEV)
    x[5, :64] = 0.0
    signs = torch.from_numpy(np.random.default_rng(block).choice([-1, 1], k).astype(np.int8)).to(DEV)
    scale = (0.5 + torch.rand(k, generator=g)).to(torch.bfloat16).to(DEV)
    a = ops.silu_mul(x) if act == "swiglu" else ops.gelu_tanh(x)
    for sc in (None, scale):
        fused = ops.hif4_quantize_act(x, act, levels=levels, input_scale=sc, signs=signs, rot_block=block,
                                      want_codes=True)
        separate = ops.hif4_quantize(a, levels=levels, input_scale=sc, signs=signs, rot_block=block, want_codes=True)
        for f, s in zip(fused, separate):
            assert torch.equal(f, s)


@pytest.mark.parametrize("k,block", [(1024, 1024), (4096, 1024), (5120, 1024), (5120, 64), (12288, 32), (16384, 1024)])
def test_quantize_rms_norm_equals_norm_then_quantize(k: int, block: int) -> None:
    """faq_hif4_quantize_rms_norm (the decoder layer's RMSNorm inside K1) gives the bits of
    faq_rms_norm followed by faq_hif4_quantize with the same HiSQ rotation, and
    faq_hif4_quantize_layer_norm those of faq_layer_norm then faq_hif4_quantize: dequantized
    values and meta, ragged row counts, with and without input_scale, two level sets."""
    from faquant_b200 import ops
    from faquant_b200.hisq_rotation import derive_hisq_rotation

    g = torch.Generator().manual_seed(k + block)
    rot = derive_hisq_rotation("model.layers.0.self_attn.q_proj", k, seed=17, block_size=block)
    signs, perm = rot.signs.to(DEV), rot.permutation.to(DEV)
    w = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16).to(DEV)
    scale = (0.5 + torch.rand(k, generator=g)).to(torch.bfloat16).to(DEV)
    assert ops.rms_norm_quantize_supported(k, block)
    for rows, levels, sc in ((37, "123", None), (1, "12", scale), (300, "123", scale)):
        x = (torch.randn(rows, k, generator=g) * 3).to(torch.bfloat16).to(DEV)
        x[0, :1024] = 0.0  # a zero chunk
        x[-1, :] *= 1e-3
        fused, fmeta = ops.hif4_quantize_rms_norm(x, w, 1e-6, levels=levels, input_scale=sc, signs=signs,
                                                  permutation=perm, rot_block=block, want_meta=True)
        h = ops.rms_norm(x, w, 1e-6)
        qdq, codes, meta = ops.hif4_quantize(h, levels=levels, input_scale=sc, signs=signs, permutation=perm,
                                             rot_block=block, want_codes=True)
        assert torch.equal(fused, qdq), (rows, levels)
        assert torch.equal(fmeta, meta), (rows, levels)
        # packed codes as well (with the QDQ, and alone: what a sequence-parallel rank
        # all-gathers); they expand back to exactly the QDQ values
        for want_qdq in (True, False):
            fc = torch.full_like(codes, 0xA5)
            fq, fm = ops.hif4_quantize_rms_norm(x, w, 1e-6, levels=levels, input_scale=sc, signs=signs,
                                                permutation=perm, rot_block=block, want_meta=True,
                                                want_qdq=want_qdq, codes_out=fc)
            assert torch.equal(fc, codes) and torch.equal(fm, meta), (rows, levels, want_qdq)
            assert (fq is None) != want_qdq and (fq is None or torch.equal(fq, qdq))
        assert torch.equal(ops.hif4_dequantize(codes, meta, k), qdq), (rows, levels)
        # the affine-free LayerNorm (norm_weight None), on values with an offset
        xo = x + 0.75
        fused, fmeta = ops.hif4_quantize_rms_norm(xo, None, 1e-6, levels=levels, input_scale=sc, signs=signs,
                                                  permutation=perm, rot_block=block, want_meta=True)
        qdq, codes, meta = ops.hif4_quantize(ops.layer_norm(xo, 1e-6), levels=levels, input_scale=sc, signs=signs,
                                             permutation=perm, rot_block=block, want_codes=True)
        assert torch.equal(fused, qdq), ("layer", rows, levels)
        assert torch.equal(fmeta, meta), ("layer", rows, levels)
        fc = torch.empty_like(codes)
        _, fm = ops.hif4_quantize_rms_norm(xo, None, 1e-6, levels=levels, input_scale=sc, signs=signs,
                                           permutation=perm, rot_block=block, want_meta=True, want_qdq=False,
                                           codes_out=fc)
        assert torch.equal(fc, codes) and torch.equal(fm, meta), ("layer codes", rows, levels)
        half = torch.empty(rows, 2 * k, dtype=torch.bfloat16, device=DEV)  # into a strided buffer
        ops.hif4_dequantize(codes, meta, k, out=half[:, k:])
        assert torch.equal(half[:, k:], qdq), ("layer", rows, levels)
    empty, _ = ops.hif4_quantize_rms_norm(torch.zeros(0, k, dtype=torch.bfloat16, device=DEV), w, 1e-6,
                                          signs=signs, permutation=perm, rot_block=block)
    assert empty.shape == (0, k)


def test_quantize_rms_norm_rejects_unsupported_shapes() -> None:
    from faquant_b200 import ops

    x = torch.zeros(4, 1536, dtype=torch.bfloat16, device=DEV)
    signs = torch.ones(1536, dtype=torch.int8, device=DEV)
    assert not ops.rms_norm_quantize_supported(1536, 64)
    with pytest.raises(NotImplementedError):
        ops.hif4_quantize_rms_norm(x, torch.ones(1536, device=DEV), 1e-6, signs=signs, rot_block=64)


def _wan_operands(seq, heads, d=128, seed=7):
    g = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(seq, 3 * heads * d, generator=g) * 2).to(torch.bfloat16)
    w = 1 + 0.2 * torch.randn(heads * d, generator=g)
    return qkv, w


def test_wan_qk_prep_matches_the_reference_glue() -> None:
    """WanRMSNorm over all heads + rope_apply (fp64) + Hadamard + HiF4 against torch's
    statement of Wan's glue and the oracle; with Smooth-QK (per head, multiply)."""
    from faquant_b200 import ops
    from faquant_b200.tensor_parallel import apply_rope3d, rope3d_tables, wan_qk_norm

    grid, heads, d = (2, 4, 6), 5, 128
    seq = grid[0] * grid[1] * grid[2]
    qkv, w = _wan_operands(seq, heads)
    n = heads * d
    cos, sin = rope3d_tables(grid, d, 10000.0, torch.device("cpu"))
    smooth = 0.5 + torch.rand(heads, d, generator=torch.Generator().manual_seed(8))
    dq = qkv.to(DEV)
    head_ss = ops.row_sumsq(dq[:, :2 * n], segments=2 * heads)[None]
    for lo, off, sm in ((0, 0, None), (n, heads, None), (0, 0, smooth)):
        x = dq[:, lo:lo + n].view(1, seq, heads, d).transpose(1, 2)
        got = ops.wan_qk_prep(x, head_ss, w.to(DEV), head_offset=off, eps=1e-6, cos=cos.to(DEV), sin=sin.to(DEV),
                              smooth_scale=None if sm is None else sm.to(DEV), smooth_mode=None if sm is None else "mul",
                              levels="123").float().cpu().numpy()
        r = apply_rope3d(wan_qk_norm(qkv[:, lo:lo + n], w, n, 1e-6).view(seq, heads, d), cos, sin)
        r = r.transpose(0, 1)[None].numpy()
        expect = oh.fake_quantize(oatt.qk_pretransform(r, r, smooth_scale=None if sm is None else sm.numpy())[0], "123")
        assert np.mean(got == expect) >= 0.995
        assert np.linalg.norm(got - expect) <= 2e-2 * np.linalg.norm(expect)


def test_wan_qk_prep_is_the_same_for_every_head_sharding() -> None:
    """The per-head sums laid out as a TP-4 all-gather ([4, L, 2 heads/4]) give each
    rank's heads the same bits as the unsharded call."""
    from faquant_b200 import ops
    from faquant_b200.tensor_parallel import rope3d_tables

    grid, heads, d, world = (3, 4, 5), 8, 128, 4
    seq, hl = grid[0] * grid[1] * grid[2], heads // world
    qkv, w = _wan_operands(seq, heads, seed=9)
    n = heads * d
    cos, sin = rope3d_tables(grid, d, 10000.0, DEV)
    dq, dw = qkv.to(DEV), w.to(DEV)
    full_ss = ops.row_sumsq(dq[:, :2 * n], segments=2 * heads)  # [L, 2 heads]: q heads, then k heads
    for lo, q_or_k in ((0, 0), (n, 1)):
        x = dq[:, lo:lo + n].view(1, seq, heads, d).transpose(1, 2)
        whole = ops.wan_qk_prep(x, full_ss[None], dw, head_offset=q_or_k * heads, cos=cos, sin=sin)
        gathered = torch.stack([torch.cat([full_ss[:, r * hl:(r + 1) * hl], full_ss[:, heads + r * hl:heads + (r + 1) * hl]],
                                          dim=1) for r in range(world)]).contiguous()
        for r in range(world):
            part = ops.wan_qk_prep(x[:, r * hl:(r + 1) * hl], gathered, dw[r * hl * d:(r + 1) * hl * d],
                                   head_offset=q_or_k * hl, cos=cos, sin=sin)
            assert torch.equal(part, whole[:, r * hl:(r + 1) * hl])


def test_wan_glue_rejects_bad_calls() -> None:
    from faquant_b200 import ops

    qkv, w = _wan_operands(16, 2)
    dq = qkv.to(DEV)
    x = dq[:, :256].view(1, 16, 2, 128).transpose(1, 2)
    ss = ops.row_sumsq(dq[:, :512], segments=4)
    with pytest.raises(TypeError):  # the sums must be [ranks, tokens, columns]
        ops.wan_qk_prep(x, ss, w.to(DEV))
    with pytest.raises(ValueError):  # heads 3..4 of a 4-column block do not exist
        ops.wan_qk_prep(x, ss[None], w.to(DEV), head_offset=3)
    with pytest.raises(ValueError):  # 100 columns do not split into 3 segments
        ops.row_sumsq(dq[:, :100], segments=3)
