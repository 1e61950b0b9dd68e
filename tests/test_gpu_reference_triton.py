"""GPU parity with the reference's own GPU kernel, from a committed fixture.

The reference's only GPU kernel is the Triton HiF4 flash attention of its Wan2.2 path,
reached through ``make_flash_attention`` (``src/faquant/wan22_attention.py:134-228``:
the head_dim Hadamard of ``rotate_heads``, HiF4 QDQ of Q/K/V, Triton attention with HiF4
P). ``tests/golden/make_triton_golden.py`` ran it on a B200 (with the reference
importable there) and stored its outputs for both normalizer modes, with the SHA-256 of
the HiF4 operands it computed. This test rebuilds the inputs from the same CPU generator,
checks that this package's K4 produces exactly those operands, and runs this package's
drop-in ``make_flash_attention`` (K4 + K5) on them: the outputs must agree within the
attention tolerance (the two kernels evaluate exp2 with different instructions and
round P at different points). It needs no reference install at run time.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
SEQ, HEADS, SEED = 1000, 3, 5  # the fixture's inputs (make_triton_golden.py)


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def _inputs():
    g = torch.Generator().manual_seed(SEED)
    return tuple(torch.randn(1, SEQ, HEADS, 128, generator=g).to(torch.bfloat16) for _ in range(3))


def _rel(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_k4_operands_are_the_references() -> None:
    from faquant_b200 import ops

    g = load_golden("wan_triton")
    q, k, v = _inputs()
    assert str(g["in_sha"]) == _sha(q) + _sha(k) + _sha(v)
    ours = [ops.qk_prep(t.to(DEV).transpose(1, 2), levels="123", rotate=rot)[0].transpose(1, 2)
            for t, rot in ((q, True), (k, True), (v, False))]
    assert "".join(_sha(t) for t in ours) == str(g["operand_sha"])


@pytest.mark.parametrize("quantized_normalizer", [False, True])
def test_flash_attention_matches_the_reference_triton_kernel(quantized_normalizer: bool) -> None:
    from faquant_b200.wan22 import faquant_qdq, make_flash_attention

    g = load_golden("wan_triton")
    q, k, v = (t.to(DEV) for t in _inputs())
    attend = make_flash_attention(faquant_qdq("123"), quantized_normalizer=quantized_normalizer, qk_rotation=True)
    ours = attend(q, k, v, softmax_scale=128**-0.5)
    assert ours.shape == (1, SEQ, HEADS, 128) and ours.dtype == torch.bfloat16
    theirs = torch.from_numpy(g[f"out_{int(quantized_normalizer)}"].view(np.int16)).view(torch.bfloat16).float()
    got = ours.float().cpu()
    assert _rel(got.numpy(), theirs.numpy()) <= 5e-3
    assert float((got - theirs).abs().max()) <= 6e-2
