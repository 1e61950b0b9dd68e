"""GPU parity of K3 (tcgen05 GEMM), K4 (Q/K/V preparation) and K5 (HiF4 attention).

Tolerances:
- GEMM: the kernel rounds an fp32 accumulation to bf16, so against the exact
  (fp64) product of the HiF4 operands each element is within half a bf16 ulp plus
  fp32 accumulation-order error: |y - ref| <= 2^-8 |ref| + 1e-4 * max|ref|.
- Attention: P = exp(s - max) uses the hardware ex2 where the reference uses CPU
  exp, so P differs by ulps and a P value can cross a HiF4 rounding boundary;
  outputs must agree within ATT_REL_FRO (relative Frobenius) and ATT_MAX_ABS.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from inputs import ATTENTION_CASES, attention_inputs, sha
from oracle import attention as oatt
from oracle import hif4 as oh

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATT_REL_FRO = 5e-3
ATT_MAX_ABS = 6e-2


def _ops():
    from faquant_b200 import ops

    return ops


def _hif4_operand(rows: int, cols: int, seed: int, scale: float = 1.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g) * scale
    return torch.from_numpy(oh.fake_quantize(x.numpy())).to(torch.bfloat16)


@pytest.mark.parametrize("m,n,k,bias", [(128, 256, 64, False), (300, 520, 200, True), (1000, 1000, 1024, True),
                                        (2048, 4096, 4096, False), (64, 48, 256, True), (1, 8, 64, False)])
def test_gemm_matches_fp64(m: int, n: int, k: int, bias: bool) -> None:
    ops = _ops()
    a = _hif4_operand(m, k, 1).to(DEV)
    b = _hif4_operand(n, k, 2, 0.02).to(DEV)
    bvec = (torch.randn(n, generator=torch.Generator().manual_seed(3)) * 0.1).to(torch.bfloat16).to(DEV) if bias else None
    y = ops.gemm_bf16(a, b, bvec)
    ref = a.double() @ b.double().T
    if bvec is not None:
        ref = ref + bvec.double()
    err = (y.double() - ref).abs()
    bound = 2.0**-8 * ref.abs() + 1e-4 * ref.abs().max()
    assert bool((err <= bound).all()), float((err - bound).max())


_ONE_CTA_CHILD = """
import sys
import torch
sys.path[:0] = sys.argv[2:4]
from faquant_b200 import ops
cases = torch.load(sys.argv[1])
torch.save([ops.gemm_bf16(a.cuda(), b.cuda(), None if c is None else c.cuda()).cpu() for a, b, c in cases],
           sys.argv[1] + ".out")
"""


def test_gemm_cta_pairs_equal_one_cta(tmp_path) -> None:
    """Shapes with a full 256 x 256 tile run on CTA pairs (tcgen05.mma.cta_group::2, each
    CTA holding half of A and half of B); FAQ_GEMM_ONE_SM=1 keeps the one-CTA kernel.
    Both sum the same products in the same K order: the same bits, ragged tiles, K tails
    and bias included."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    ops = _ops()
    shapes = [(300, 520, 200, True), (257, 257, 72, False), (1000, 1000, 1024, True), (2048, 4096, 4096, False),
              (8192, 1024, 4096, False), (512, 768, 8, True)]
    cases, ours = [], []
    for i, (m, n, k, bias) in enumerate(shapes):
        a = _hif4_operand(m, k, 10 + i)
        b = _hif4_operand(n, k, 20 + i, 0.02)
        c = (torch.randn(n, generator=torch.Generator().manual_seed(i)) * 0.1).to(torch.bfloat16) if bias else None
        cases.append((a, b, c))
        ours.append(ops.gemm_bf16(a.to(DEV), b.to(DEV), None if c is None else c.to(DEV)).cpu())
    path = tmp_path / "gemm_cases.pt"
    torch.save(cases, path)
    root = Path(__file__).resolve().parents[1]
    subprocess.run([sys.executable, "-c", _ONE_CTA_CHILD, str(path), str(root / "faquant-public_b200"), str(root)],
                   check=True, env=dict(os.environ, FAQ_GEMM_ONE_SM="1"), timeout=600)
    theirs = torch.load(str(path) + ".out")
    for (m, n, k, _), a, b in zip(shapes, ours, theirs):
        assert torch.equal(a, b), (m, n, k)


def test_gemm_sm_target_keeps_the_bits() -> None:
    """faq_set_gemm_sm_target (fewer SMs for the persistent grids, so collectives find free
    SMs) changes only which CTA computes a tile: the bf16 GEMM (pairs and one-CTA shapes)
    and the packed W4A4 GEMM give the same bits at 2, 17, 100 SMs and at every SM."""
    ops = _ops()
    cases = [(2048, 4096, 1024), (300, 520, 256), (8192, 1024, 512)]
    try:
        for i, (m, n, k) in enumerate(cases):
            a = _hif4_operand(m, k, 40 + i).to(DEV)
            b = _hif4_operand(n, k, 50 + i, 0.02).to(DEV)
            ac, am = ops.hif4_quantize(a, want_codes=True)[1:]
            bc, bm, _ = ops.hif4_pack_weight(b)
            ops.set_gemm_sm_target(0)
            ref, ref_p = ops.gemm_bf16(a, b), ops.w4a4_gemm((ac, am), bc, bm)
            for sms in (2, 17, 100, 1000):
                ops.set_gemm_sm_target(sms)
                assert torch.equal(ops.gemm_bf16(a, b), ref), (m, n, k, sms)
                assert torch.equal(ops.w4a4_gemm((ac, am), bc, bm), ref_p), (m, n, k, sms)
    finally:
        ops.set_gemm_sm_target(0)
    with pytest.raises(Exception):
        ops.set_gemm_sm_target(-1)


@pytest.mark.parametrize("m,n,k", [(300, 520, 200), (1000, 1000, 1024), (33, 48, 64), (2048, 4096, 512)])
def test_gemm_residual_epilogue_is_the_separate_bf16_add(m: int, n: int, k: int) -> None:
    """y = bf16(bf16(a b^T + bias) + residual): the same bits as the GEMM followed by the
    eager bf16 add, on both GEMM kernels' shapes, ragged tiles and a strided residual."""
    ops = _ops()
    a = _hif4_operand(m, k, 30).to(DEV)
    b = _hif4_operand(n, k, 31, 0.02).to(DEV)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(32)) * 0.1).to(torch.bfloat16).to(DEV)
    wide = (torch.randn(m, n + 24, generator=torch.Generator().manual_seed(33)) * 3).to(torch.bfloat16).to(DEV)
    for residual in (wide[:, :n].contiguous(), wide[:, :n]):  # contiguous and strided (ldr = n + 24)
        fused = ops.gemm_bf16(a, b, bias, residual=residual)
        assert torch.equal(fused, residual + ops.gemm_bf16(a, b, bias))


def test_gemm_strided_and_tail_k() -> None:
    ops = _ops()
    a_full = _hif4_operand(200, 136, 4).to(DEV)
    a = a_full[:, :128]  # lda 136
    b = _hif4_operand(72, 128, 5).to(DEV)
    y = ops.gemm_bf16(a, b)
    ref = a.double() @ b.double().T
    assert torch.allclose(y.double(), ref, rtol=2**-8, atol=1e-3)
    a2 = _hif4_operand(33, 100, 6).to(DEV)  # k % 8 != 0 -> zero padded
    b2 = _hif4_operand(40, 100, 7).to(DEV)
    y2 = ops.gemm_bf16(a2, b2)
    assert torch.allclose(y2.double(), a2.double() @ b2.double().T, rtol=2**-8, atol=1e-3)


def test_qk_prep_matches_reference_fixture() -> None:
    ops = _ops()
    g = load_golden("qk_prep")
    q = torch.from_numpy(g["q"].view(np.int16)).view(torch.bfloat16).to(DEV)
    k = torch.from_numpy(g["k"].view(np.int16)).view(torch.bfloat16).to(DEV)
    scale = torch.from_numpy(g["scale"]).to(DEV)
    offset = torch.from_numpy(g["offset"]).to(DEV)
    qo, _, _ = ops.qk_prep(q, levels=None, rotate=True, smooth_scale=scale, smooth_mode="mul")
    ko, _, _ = ops.qk_prep(k, levels=None, rotate=True, smooth_scale=scale, smooth_mode="div", key_offset=offset)
    assert np.array_equal(qo.cpu().view(torch.int16).numpy().view(np.uint16), g["q_out"])
    assert np.array_equal(ko.cpu().view(torch.int16).numpy().view(np.uint16), g["k_out"])
    # with HiF4 along head_dim: equals the oracle's QDQ of the transformed operand, codes too
    qq, codes, meta = ops.qk_prep(q, levels="123", rotate=True, smooth_scale=scale, smooth_mode="mul",
                                  want_codes=True)
    expect = oh.fake_quantize(oh.bf16_to_f32(g["q_out"]), "123")
    assert np.array_equal(qq.cpu().view(torch.int16).numpy().view(np.uint16), oh.f32_to_bf16_bits(expect))
    oc, om = oh.hif4_encode(oh.bf16_to_f32(g["q_out"]).reshape(-1, 128), "123")
    assert np.array_equal(codes.cpu().numpy(), oc)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), om)


def test_qk_prep_strided_fp32_input_and_per_head_scale() -> None:
    ops = _ops()
    rng = np.random.default_rng(9)
    x = torch.from_numpy(rng.standard_normal((2, 50, 3, 128)).astype(np.float32)).to(DEV).transpose(1, 2)  # [B,H,S,D]
    s = torch.from_numpy(rng.uniform(0.5, 2, (3, 128)).astype(np.float32)).to(DEV)
    out, _, _ = ops.qk_prep(x, levels="13", rotate=True, smooth_scale=s, smooth_mode="div")
    xt = x.cpu().numpy()
    qf = (xt / s.cpu().numpy()[None, :, None, :]).astype(np.float32)
    from oracle.rotation import hadamard

    expect = oh.fake_quantize(oh.bf16_round(hadamard(qf)), "13")
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), oh.f32_to_bf16_bits(expect))


@pytest.mark.parametrize("d", [128, 64])
def test_qk_prep_hadamard_rounding_over_many_magnitudes(d) -> None:
    """bf16(Hadamard(x) / sqrt(d)) bit for bit over ~2M fp32 values whose magnitudes span
    ~70 binades, with zeros, -0.0, values near the bottom of the normal range and a row
    that overflows to infinity: the head_dim scaling takes a reciprocal product except
    next to a bf16 rounding boundary, where it divides."""
    ops = _ops()
    rng = np.random.default_rng(21)
    n = (1 << 21) // d
    x = (rng.standard_normal((n, d)) * np.exp2(rng.integers(-40, 30, (n, 1)))).astype(np.float32)
    x[0] = 0.0
    x[1] = -0.0
    x[2, ::2] = -0.0
    x[3] = (rng.standard_normal(d) * 2.0**-120).astype(np.float32)
    x[4] = 0.0
    x[4, :2] = 3.0e38  # one pair overflows: +-inf and zeros downstream, no inf - inf
    got = ops.qk_prep(torch.from_numpy(x).to(DEV).view(1, 1, n, d), levels=None, rotate=True)[0]
    from oracle.rotation import hadamard

    with np.errstate(over="ignore"):
        expect = oh.f32_to_bf16_bits(oh.bf16_round(hadamard(x)))
    assert np.array_equal(got.cpu().view(torch.int16).numpy().view(np.uint16).reshape(n, d), expect)


def test_ex2_is_monotone_on_this_device() -> None:
    """K5 takes each HiF4 group's scale from ex2 of the group's largest score, which is
    the largest P only if ex2.approx.ftz never decreases: checked over every float in
    [-inf, 1] (about 3.2e9 values)."""
    import ctypes

    from faquant_b200 import _lib

    bad = ctypes.c_uint64(1)
    _lib.call("faq_selftest_ex2_monotone", ctypes.byref(bad), torch.cuda.current_stream().cuda_stream)
    assert bad.value == 0


def _attention_gpu(q, k, v, *, causal, normalizer, qk_quant, pv_quant, levels="123"):
    ops = _ops()
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    if qk_quant:
        qd, _, _ = ops.qk_prep(qd, levels=levels, rotate=False)
        kd, _, _ = ops.qk_prep(kd, levels=levels, rotate=False)
    if pv_quant:
        vd, _, _ = ops.qk_prep(vd, levels=levels, rotate=False)
    return ops.hif4_attention(qd, kd, vd, causal=causal, p_levels=levels if pv_quant else None,
                              quantized_normalizer=normalizer == "quantized_same")


def _check_close(out: torch.Tensor, ref: np.ndarray) -> tuple[float, float]:
    o = out.float().cpu().numpy()
    err = o - ref
    rel = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
    mx = float(np.abs(err).max())
    assert rel <= ATT_REL_FRO and mx <= ATT_MAX_ABS, (rel, mx)
    return rel, mx


@pytest.mark.parametrize("case", ATTENTION_CASES, ids=[c[0] for c in ATTENTION_CASES])
def test_attention_matches_reference_fixture(case) -> None:
    g = load_golden("attention")
    tag, b, h, kv, sq, sk, causal, normalizer, qk, pv, seed = case
    q, k, v = attention_inputs(b, h, kv, sq, sk, seed)
    assert str(g[f"{tag}_in_sha"]) == sha(q) + sha(k) + sha(v)
    out = _attention_gpu(q, k, v, causal=causal, normalizer=normalizer, qk_quant=qk, pv_quant=pv)
    _check_close(out, oh.bf16_to_f32(g[f"{tag}_out"]))


@pytest.mark.parametrize("causal,normalizer,levels", [(True, "quantized_same", "123"), (False, "unquantized", "123"),
                                                      (True, "unquantized", "12")])
def test_attention_matches_oracle_mid_size(causal: bool, normalizer: str, levels: str) -> None:
    q, k, v = attention_inputs(1, 8, 2, 1000, 1000, 77)
    out = _attention_gpu(q, k, v, causal=causal, normalizer=normalizer, qk_quant=True, pv_quant=True, levels=levels)
    ref = oatt.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=causal,
                         normalizer=normalizer, levels={"q": levels, "k": levels, "p": levels, "v": levels})
    _check_close(out, ref)


def test_attention_unit_values_are_exact_under_p_reordering() -> None:
    # simulated_flash_attention tests :653-688: with P-Reordering the numerator and the
    # denominator are sums of the same quantized P, so V = c gives exactly c. HiF4 itself
    # maps 1.0 to 0.9375 (scale 0.15625, code 6 with both micro-exponents), so the
    # QDQ'd V = 1 gives exactly 0.9375 and an unquantized V = 1 gives exactly 1.
    ops = _ops()
    q, k, _ = attention_inputs(1, 4, 2, 300, 300, 88)
    ones = torch.ones(1, 2, 300, 128, dtype=torch.bfloat16, device=DEV)
    qd, _, _ = ops.qk_prep(q.to(DEV), levels="123", rotate=True)
    kd, _, _ = ops.qk_prep(k.to(DEV), levels="123", rotate=True)
    out = ops.hif4_attention(qd, kd, ones, causal=True, p_levels="123", quantized_normalizer=True)
    assert torch.equal(out.float().cpu(), torch.ones(1, 300, 4, 128))
    vq, _, _ = ops.qk_prep(ones, levels="123", rotate=False)
    c = float(oh.fake_quantize(np.ones((1, 64), np.float32))[0, 0])
    assert c == 0.9375 and float(vq[0, 0, 0, 0]) == c
    out = ops.hif4_attention(qd, kd, vq, causal=True, p_levels="123", quantized_normalizer=True)
    assert torch.equal(out.float().cpu(), torch.full((1, 300, 4, 128), c))


def test_bounded_wait_reports_timeout_status() -> None:
    from faquant_b200 import _lib

    ops = _ops()
    _lib.device_status(reset=True)
    ops.selftest_wait_timeout(50_000_000)  # 50 ms on an mbarrier nothing arrives at
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) & _lib.FAQ_STATUS_TIMEOUT
    assert _lib.device_status() == 0
