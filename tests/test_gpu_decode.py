"""GPU tests of K6, the HiF4 decode attention (faq_hif4_decode_attention), through the C ABI.

Operands are HiF4 Q/K/V prepared on the GPU (K4); the oracle's tiled simulator runs the
same semantics on them (operands_quantized). Decode is the reference's attention call
with a few query positions at the end of a long cache, so the cases cover GQA groups of
4 and 8, MHA, several query positions, caches shorter than a tile and not a multiple of
128, several splits, and the three P modes (HiF4 P with P-Reordering, raw normalizer,
unquantized P)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
ATT_REL_FRO = 5e-3
ATT_MAX_ABS = 6e-2

CASES = [  # (b, hq, hkv, sq, sk)
    (1, 8, 2, 1, 1000),
    (2, 4, 4, 3, 300),
    (1, 32, 8, 1, 2500),
    (1, 16, 2, 2, 4096),
    (3, 4, 1, 1, 5),
]


def _operands(b, hq, hkv, sq, sk, seed):
    from faquant_b200 import ops

    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, hq, sq, 128, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(b, hkv, sk, 128, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(b, hkv, sk, 128, generator=g).to(torch.bfloat16).to(DEV)
    return (ops.qk_prep(q, levels="123", rotate=True)[0], ops.qk_prep(k, levels="123", rotate=True)[0],
            ops.qk_prep(v, levels="123", rotate=False)[0])


def _close(got: torch.Tensor, ref: np.ndarray) -> None:
    o = got.float().cpu().numpy()
    err = o - ref
    rel = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
    assert rel <= ATT_REL_FRO and float(np.abs(err).max()) <= ATT_MAX_ABS, rel


@pytest.mark.parametrize("mode", ["quantized_same", "raw", "p_unquantized"])
@pytest.mark.parametrize("case", CASES, ids=[f"b{c[0]}_h{c[1]}_{c[2]}_sq{c[3]}_sk{c[4]}" for c in CASES])
def test_decode_matches_oracle(case, mode) -> None:
    from faquant_b200 import ops

    b, hq, hkv, sq, sk = case
    q, k, v = _operands(b, hq, hkv, sq, sk, seed=sk + sq)
    p_levels = None if mode == "p_unquantized" else "123"
    out = ops.hif4_decode_attention(q, k, v, p_levels=p_levels, quantized_normalizer=mode == "quantized_same")
    assert out.shape == (b, sq, hq, 128)
    ref = oatt.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), causal=True,
                         pv_quant=mode != "p_unquantized",
                         normalizer="quantized_same" if mode == "quantized_same" else "unquantized",
                         operands_quantized=True)
    _close(out, ref)


def test_decode_agrees_with_the_prefill_kernel() -> None:
    from faquant_b200 import ops

    q, k, v = _operands(1, 32, 8, 1, 2500, seed=7)
    dec = ops.hif4_decode_attention(q, k, v).float().cpu().numpy()
    pre = ops.hif4_attention(q, k, v, causal=True).float().cpu().numpy()
    assert np.linalg.norm(dec - pre) <= ATT_REL_FRO * np.linalg.norm(pre)


def test_back_to_back_calls_share_one_workspace() -> None:
    """Passes 2 and 3 start before the pass they follow has finished (programmatic
    dependent launch) and read only what they may before they wait; calls queued back to
    back on one stream with one workspace and one output buffer, no host sync between
    them, give the same bits as the same calls made one at a time."""
    from faquant_b200 import ops

    shapes = [(1, 32, 8, 1, 32768), (1, 32, 8, 1, 700), (2, 8, 2, 3, 9000), (1, 32, 8, 1, 32768)]
    inputs = [_operands(*s, seed=20 + i) for i, s in enumerate(shapes)]
    one_at_a_time = []
    for q, k, v in inputs:
        one_at_a_time.append(ops.hif4_decode_attention(q, k, v).clone())
        torch.cuda.synchronize()
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=DEV)
    queued = [ops.hif4_decode_attention(q, k, v, workspace=ws).clone() for q, k, v in inputs for _ in range(3)]
    torch.cuda.synchronize()
    for i, ref in enumerate(one_at_a_time):
        for j in range(3):
            assert torch.equal(queued[3 * i + j], ref)


def test_decode_rejects_bad_calls() -> None:
    from faquant_b200 import _lib, ops

    q, k, v = _operands(1, 64, 1, 1, 200, seed=1)  # 64 rows per kv head > 32
    with pytest.raises(ValueError):
        ops.hif4_decode_attention(q, k, v)
    q, k, v = _operands(1, 8, 2, 1, 200, seed=2)
    ws = torch.empty(16, dtype=torch.uint8, device=DEV)
    out = torch.empty(1, 1, 8, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):  # workspace smaller than faq_hif4_decode_workspace_bytes
        _lib.call("faq_hif4_decode_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, 8, 2, 1, 200, 128,
                  q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), v.stride(0),
                  v.stride(1), v.stride(2), 128**-0.5, 123, 1, out.data_ptr(), out.stride(0), out.stride(1),
                  out.stride(2), ws.data_ptr(), 16, torch.cuda.current_stream().cuda_stream)
    assert _lib.load().faq_hif4_decode_workspace_bytes(1, 8, 3, 1, 200, 128) == 0  # 8 % 3 != 0
