"""The allocation-free decode entry point, faq_hif4_decode_attention_static.

Some callers cannot allocate device memory -- a serving runtime that plans all of its
memory at start-up and forbids allocations while it serves, or a host hot path where
cudaMalloc would synchronize the device. For them the decode call keeps its scratch in a
16 MiB array inside the library instead of a caller workspace. These tests call it
through the C ABI on a larger problem, a smaller one, then the larger one again (the calls
share that array, so the third call starts from the second call's leftovers), and check
that each result equals the workspace entry point's bit for bit: both run the same three
kernels on the same inputs, only the scratch address differs. They also check that a
problem needing more scratch is refused. The file is collected last so that a run stopping
at the first failure has run everything else."""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
STATIC_SCRATCH_BYTES = 16 << 20  # FAQ_DECODE_STATIC_SCRATCH_BYTES in include/faquant_b200.h


def _operands(b, hq, hkv, sq, sk, seed):
    from faquant_b200 import ops

    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, hq, sq, 128, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(b, hkv, sk, 128, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(b, hkv, sk, 128, generator=g).to(torch.bfloat16).to(DEV)
    return (ops.qk_prep(q, levels="123", rotate=True)[0], ops.qk_prep(k, levels="123", rotate=True)[0],
            ops.qk_prep(v, levels="123", rotate=False)[0])


def _static_call(q, k, v, out) -> None:
    from faquant_b200 import _lib

    b, hq, sq, d = q.shape
    hkv, sk = k.shape[1], k.shape[2]
    _lib.call("faq_hif4_decode_attention_static", q.data_ptr(), k.data_ptr(), v.data_ptr(), b, hq, hkv, sq, sk, d,
              q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1),
              v.stride(2), ctypes.c_float(d**-0.5).value, 123, 1, out.data_ptr(), out.stride(0), out.stride(1),
              out.stride(2), torch.cuda.current_stream(DEV).cuda_stream)


def test_static_scratch_decode_matches_the_workspace_entry_point_twice() -> None:
    from faquant_b200 import ops

    large, small = ((1, 32, 8, 1, 2500), 3), ((2, 8, 2, 3, 700), 4)
    for case, seed in (large, small, large):
        q, k, v = _operands(*case, seed=seed)
        out = torch.full((case[0], case[3], case[1], 128), float("nan"), dtype=torch.bfloat16, device=DEV)
        _static_call(q, k, v, out)
        ref = ops.hif4_decode_attention(q, k, v)
        torch.cuda.synchronize(DEV)
        assert torch.isfinite(ref.float()).all()
        assert torch.equal(out, ref)


def test_static_scratch_refuses_a_problem_larger_than_its_array() -> None:
    from faquant_b200 import _lib

    assert _lib.load().faq_hif4_decode_workspace_bytes(8, 32, 8, 1, 65536, 128) > STATIC_SCRATCH_BYTES
    q = torch.zeros(8, 32, 1, 128, dtype=torch.bfloat16, device=DEV)
    kv = torch.zeros(8, 8, 65536, 128, dtype=torch.bfloat16, device=DEV)
    out = torch.empty(8, 1, 32, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError, match="16 MiB"):
        _static_call(q, kv, kv, out)
