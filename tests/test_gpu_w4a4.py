"""The W4A4 GEMM on packed HiF4 operands (``faq_w4a4_gemm``, ``faq_w4a4_gemm_qdq_a``).

Both operands stay in the 4.5-bit packed format; the kernel expands them into the bf16
tiles the tensor cores read. The tests check that the output is bit-identical (signed
zeros included) to the bf16 GEMM on the dequantized operands -- which the GEMM tests pin
to the fp64 product and which is F.linear on the reference's fake-quantized tensors --
for the BASELINE config-2 projection shapes, ragged and small shapes, bias and residual,
and blocks at the ends of the scale range; and that the packed path is the one
``FakeQuantLinear`` runs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _ops():
    from faquant_b200 import ops

    return ops


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy()


def _operands(m: int, n: int, k: int, seed: int):
    """Packed activation (K1, HiSQ-style signs + 64-block Hadamard) and packed RTN weight (K2)."""
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(m, k, device=DEV, generator=g)
    x[:, torch.randperm(k, device=DEV, generator=g)[: max(1, k // 200)]] *= 20.0
    x = x.to(torch.bfloat16)
    signs = (torch.randint(0, 2, (k,), device=DEV, generator=g) * 2 - 1).to(torch.int8)
    xq, a_codes, a_meta = ops.hif4_quantize(x, levels="123", signs=signs, rot_block=64, want_codes=True)
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    b_codes, b_meta, _ = ops.hif4_pack_weight(w, levels="123")
    wq = ops.hif4_dequantize(b_codes, b_meta, k)
    return xq, a_codes, a_meta, wq, b_codes, b_meta


SHAPES = [
    (512, 512, 256),      # first: one wave, a few K blocks
    (300, 520, 768),      # ragged M and N
    (64, 1024, 4096),     # M below one pair tile
    (8192, 4096, 4096),   # q_proj / o_proj (config 2)
    (8192, 1024, 4096),   # k_proj / v_proj
    (8192, 12288, 4096),  # gate_proj / up_proj
    (8192, 4096, 12288),  # down_proj
]


@pytest.mark.parametrize("m,n,k", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
def test_packed_gemm_is_bit_identical_to_the_bf16_gemm(m: int, n: int, k: int) -> None:
    from faquant_b200 import _lib

    ops = _ops()
    _lib.device_status(reset=True)
    xq, a_codes, a_meta, wq, b_codes, b_meta = _operands(m, n, k, seed=m + n + k)
    ref = ops.gemm_bf16(xq, wq)
    packed = ops.w4a4_gemm((a_codes, a_meta), b_codes, b_meta)
    qdq_a = ops.w4a4_gemm(xq, b_codes, b_meta)
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    assert np.array_equal(_bits(packed), _bits(ref))
    assert np.array_equal(_bits(qdq_a), _bits(ref))


def test_bias_residual_and_scale_extremes() -> None:
    """Bias and residual in the epilogue; blocks of zeros (scale clamp 2^-48), of tiny and
    of huge values (the 49152 clamp), and negative values that round to -0.0."""
    from faquant_b200 import _lib

    ops = _ops()
    m, n, k = 384, 640, 512
    g = torch.Generator(device=DEV).manual_seed(11)
    x = torch.randn(m, k, device=DEV, generator=g)
    x[0] = 0.0
    x[1, :64] = 0.0
    x[2] *= 1e-30
    x[3] *= 1e6
    x[4, :64] = torch.linspace(-1e-3, 1.0, 64, device=DEV)  # small negatives -> -0.0 codes
    x[5, 64:128] = -1e-12
    x[5, 127] = 2.0
    x = x.to(torch.bfloat16)
    xq, a_codes, a_meta = ops.hif4_quantize(x, levels="123", want_codes=True)
    w = torch.randn(n, k, device=DEV, generator=g) * 0.02
    w[7] = 0.0
    w[8] *= 1e4
    w = w.to(torch.bfloat16)
    b_codes, b_meta, _ = ops.hif4_pack_weight(w, levels="123")
    wq = ops.hif4_dequantize(b_codes, b_meta, k)
    bias = (torch.randn(n, device=DEV, generator=g) * 0.1).to(torch.bfloat16)
    res = torch.randn(m, n, device=DEV, generator=g).to(torch.bfloat16)
    _lib.device_status(reset=True)
    ref = ops.gemm_bf16(xq, wq, bias, residual=res)
    got = ops.w4a4_gemm((a_codes, a_meta), b_codes, b_meta, bias, residual=res)
    plain_ref = ops.gemm_bf16(xq, wq)
    plain = ops.w4a4_gemm((a_codes, a_meta), b_codes, b_meta)
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    assert np.array_equal(_bits(got), _bits(ref))
    assert np.array_equal(_bits(plain), _bits(plain_ref))


def test_two_level_variants_and_gptq_metadata() -> None:
    """Two-level scales (lv2 only, lv3 only) and a weight packed from GPTQ metadata."""
    from conftest import load_golden

    ops = _ops()
    for levels in ("12", "13"):
        g = torch.Generator(device=DEV).manual_seed(21)
        x = torch.randn(256, 512, device=DEV, generator=g).to(torch.bfloat16)
        w = (torch.randn(256, 512, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
        xq, a_codes, a_meta = ops.hif4_quantize(x, levels=levels, want_codes=True)
        b_codes, b_meta, _ = ops.hif4_pack_weight(w, levels=levels)
        wq = ops.hif4_dequantize(b_codes, b_meta, 512)
        assert np.array_equal(_bits(ops.w4a4_gemm((a_codes, a_meta), b_codes, b_meta)),
                              _bits(ops.gemm_bf16(xq, wq)))
    gp = load_golden("gptq")
    w = torch.from_numpy(gp["w"].view(np.int16)).view(torch.bfloat16).to(DEV)
    scale, lv2, lv3 = (torch.from_numpy(gp[name]) for name in ("scale", "lv2", "lv3"))
    b_codes, b_meta, bad = ops.hif4_pack_weight(w, scale=scale, lv2=lv2, lv3=lv3)
    assert bad == 0
    x = torch.randn(300, w.shape[1], device=DEV).to(torch.bfloat16)
    xq, a_codes, a_meta = ops.hif4_quantize(x, levels="123", want_codes=True)
    assert np.array_equal(_bits(ops.w4a4_gemm((a_codes, a_meta), b_codes, b_meta)), _bits(ops.gemm_bf16(xq, w)))


def test_bad_arguments_are_rejected() -> None:
    ops = _ops()
    codes = torch.zeros(64, 48, dtype=torch.uint8, device=DEV)  # k = 96: not whole blocks
    meta = torch.zeros(64, 1, dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError):
        ops.w4a4_gemm((codes, meta), codes, meta)
    # whole blocks but meta rows of 12 bytes: the TMA loads need k % 256 == 0
    codes = torch.zeros(64, 96, dtype=torch.uint8, device=DEV)
    meta = torch.zeros(64, 3, dtype=torch.int32, device=DEV)
    with pytest.raises(NotImplementedError):
        ops.w4a4_gemm((codes, meta), codes, meta)


def test_fake_quant_linear_with_packed_weights(monkeypatch) -> None:
    """``FakeQuantLinear`` holding only the packed weight gives the bits of the bf16-weight
    module (config-2 q_proj shape, HiSQ1024 rotation, bias); its state_dict carries the
    reference's bf16 ``weight``; a packed module loaded from it reproduces the weight."""
    from faquant_b200.hisq_rotation import derive_hisq_rotation
    from faquant_b200.quantization import FakeQuantLinear

    k, n = 4096, 1024
    rot = derive_hisq_rotation("model.layers.0.self_attn.q_proj", k, seed=17, block_size=1024)
    g = torch.Generator(device=DEV).manual_seed(31)
    lin = torch.nn.Linear(k, n, bias=True, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(n, k, device=DEV, generator=g) * 0.02)
        lin.bias.copy_(torch.randn(n, device=DEV, generator=g) * 0.1)
    kw = dict(quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64, symmetric=True,
              clip_ratio=1.0, input_rotation_signs=rot.signs.to(DEV), input_rotation_permutation=rot.permutation.to(DEV),
              input_rotation_block_size=1024)
    plain, packed = FakeQuantLinear(lin, **kw), FakeQuantLinear(lin, packed_weights=True, **kw)
    assert packed.packed and packed.weight is None and not plain.packed
    assert torch.equal(packed.dequantized_weight(), plain.weight)
    x = torch.randn(3, 700, k, device=DEV, generator=g).to(torch.bfloat16)
    xs = torch.randn(2, 100, k, device=DEV, generator=g).to(torch.bfloat16)
    import faquant_b200.quantization as fq

    with torch.no_grad():
        for rows in (0, 1 << 30):  # weight expanded + bf16 GEMM, then the packed GEMM
            monkeypatch.setattr(fq, "PACKED_EXPAND_MIN_ROWS", rows)
            assert np.array_equal(_bits(packed(x)), _bits(plain(x)))
            assert np.array_equal(_bits(packed(xs)), _bits(plain(xs)))
    monkeypatch.undo()
    sd = packed.state_dict()
    assert torch.equal(sd["weight"], plain.weight) and "weight_codes" not in sd
    # the saved metadata is the reference's RTN fit of the source weight (hif4.py:142-219)
    from oracle import hif4 as oh

    _, ref_meta = oh.hif4_encode(lin.weight.detach().float().cpu().numpy(), "123")
    assert np.array_equal(packed.weight_meta.cpu().numpy().view(np.uint32), ref_meta)
    assert sd["weight_hif4_scale_lv3_exponent"].shape == (n, k // 64, 16)
    other = FakeQuantLinear(lin, packed_weights=True, **kw)
    other.load_state_dict(sd)
    # the same metadata and values (a weight of -0.0 comes back as +0: equal values)
    assert torch.equal(other.weight_meta, packed.weight_meta)
    assert torch.equal(other.dequantized_weight(), plain.weight)
    with torch.no_grad():
        assert np.array_equal(_bits(other(x)), _bits(plain(x)))
    # a bf16 grid weight without its metadata cannot be refitted exactly in general
    plain_sd = plain.state_dict()
    try:
        other.load_state_dict(plain_sd)
        assert torch.equal(other.dequantized_weight(), plain.weight)
    except RuntimeError as e:
        assert "refit" in str(e)


@pytest.mark.parametrize("rows,k", [(1000, 4096), (37, 192), (4096, 12288)])
def test_fast_bf16_expansion_matches_the_decoder(rows: int, k: int) -> None:
    """faq_hif4_dequantize's bf16 path for whole blocks (hif4_expand32_bf16, the packed
    GEMM's expansion) against its generic per-value decoder (fp32 output, exact in bf16):
    the same bits, negative zero codes included, over random codes and meta words spanning
    the E6M2 code range and every lv2/lv3 pattern."""
    from faquant_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(rows + k)
    codes = torch.randint(0, 256, (rows, k // 2), device=DEV, generator=g, dtype=torch.int32).to(torch.uint8)
    scale = torch.randint(0, 256, (rows, k // 64), device=DEV, generator=g, dtype=torch.int64)  # every E6M2 code
    bits = torch.randint(0, 1 << 24, (rows, k // 64), device=DEV, generator=g, dtype=torch.int64) << 8
    word = bits | scale  # < 2^32: as int32 with the same bits
    meta = (word - ((word >> 31) << 32)).to(torch.int32)
    fast = ops.hif4_dequantize(codes, meta, k, dtype=torch.bfloat16)
    ref = ops.hif4_dequantize(codes, meta, k, dtype=torch.float32).to(torch.bfloat16)
    assert np.array_equal(_bits(fast), _bits(ref))


@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (3, 1000, 4096), (8, 1024, 12288), (9, 2304, 4096),
                                   (16, 5120, 25600), (16, 17, 256)])
def test_small_row_kernel_matches_fp64(m: int, n: int, k: int) -> None:
    """faq_w4a4_gemm_qdq_a with m <= 16 (the small-row kernel: the weight streamed packed
    into mma.sync fragments, K split over eight warps, a fixed-order sum) against the product
    of the dequantized operands in fp64, with bias and residual; the same bits on a second
    run; within bf16 output rounding of the tiled bf16 GEMM on the same operands."""
    from faquant_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    a, _, _ = ops.hif4_quantize(x, levels="123")
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    bc, bm, _ = ops.hif4_pack_weight(w, levels="123")
    wd = ops.hif4_dequantize(bc, bm, k)
    bias = (torch.randn(n, device=DEV, generator=g) * 0.1).to(torch.bfloat16)
    res = torch.randn(m, n, device=DEV, generator=g).to(torch.bfloat16)
    y = ops.w4a4_gemm(a, bc, bm, bias=bias, residual=res)
    y2 = ops.w4a4_gemm(a, bc, bm, bias=bias, residual=res)
    assert np.array_equal(_bits(y), _bits(y2))
    pre = a.double() @ wd.double().T + bias.double()
    ref = pre + res.double()
    # the output is bf16(bf16(sum + bias) + residual): the first rounding may land one ulp
    # away from the exact sum's (fp32 sums in another order), the second is half an ulp
    scale = pre.abs() + res.double().abs() + 1e-30
    assert bool(((y.double() - ref).abs() <= 2.0 ** -7 * scale).all())
    tiled = ops.gemm_bf16(a, wd, bias=bias, residual=res)
    assert bool(((y.double() - tiled.double()).abs() <= 2.0 ** -6 * scale).all())


def test_packed_module_few_rows_streams_the_packed_weight() -> None:
    """A packed FakeQuantLinear called with at most PACKED_SMALL_ROWS rows (decode) runs the
    small-row kernel; it agrees with the bf16-weight module within bf16 output rounding."""
    from faquant_b200.quantization import PACKED_SMALL_ROWS, FakeQuantLinear

    k, n = 4096, 4096
    g = torch.Generator(device=DEV).manual_seed(5)
    lin = torch.nn.Linear(k, n, bias=True, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(n, k, device=DEV, generator=g) * 0.02)
        lin.bias.copy_(torch.randn(n, device=DEV, generator=g) * 0.1)
    kw = dict(quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64, symmetric=True,
              clip_ratio=1.0)
    plain, packed = FakeQuantLinear(lin, **kw), FakeQuantLinear(lin, packed_weights=True, **kw)
    for rows in (1, 4, PACKED_SMALL_ROWS):
        x = torch.randn(rows, k, device=DEV, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            yp, yb = packed(x).double(), plain(x).double()
        assert bool(((yp - yb).abs() <= 2.0 ** -7 * yb.abs() + 1e-30).all())  # one bf16 ulp at most
