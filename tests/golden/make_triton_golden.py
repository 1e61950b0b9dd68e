"""Generate ``wan_triton.npz``: outputs of the reference's own GPU kernel.

The reference's only GPU kernel is the Triton HiF4 flash attention of its Wan2.2 path
(``src/faquant/wan22_attention.py:134-183``), reached through its drop-in
``make_flash_attention`` (``:195-228``: ``rotate_heads`` over head_dim, the HiF4 QDQ of
``wan22_hif4.faquant_qdq``, then ``hif4_attention``). It needs a GPU, so this script runs
on a GPU box where the reference is importable -- from ``FAQUANT_REFERENCE_SRC`` (its
``src`` directory) or from an offline pip install under ``baseline/_ref`` -- and writes
the fixture into the directory given as its argument::

    python tests/golden/make_triton_golden.py gpurun_out/

The inputs come from the torch CPU generator (seed 5, so the tests rebuild them and check
their SHA-256); the fixture stores the reference's outputs for both normalizer modes as
bf16 bits, plus the SHA-256 of the HiF4 Q/K/V operands the reference computed, which the
test compares with this package's own operands.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
SEQ, HEADS, SEED = 1000, 3, 5


def reference_path() -> Path:
    src = os.environ.get("FAQUANT_REFERENCE_SRC")
    if src:
        return Path(src)
    return HERE.parents[1] / "baseline" / "_ref"


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def inputs():
    """q, k, v [1, SEQ, HEADS, 128] bf16 ~N(0,1): Wan's [B, L, H, D] flash_attention layout."""
    g = torch.Generator().manual_seed(SEED)
    return tuple(torch.randn(1, SEQ, HEADS, 128, generator=g).to(torch.bfloat16) for _ in range(3))


def main() -> None:
    out_dir = Path(sys.argv[1] if len(sys.argv) > 1 else ".")
    sys.path.insert(0, str(reference_path()))
    from faquant.wan22_attention import make_flash_attention, rotate_heads
    from faquant.wan22_hif4 import faquant_qdq

    q, k, v = (t.cuda() for t in inputs())
    qdq = faquant_qdq("123")
    operands = [qdq(rotate_heads(q)), qdq(rotate_heads(k)), qdq(v)]
    arrays = {"in_sha": np.array(sha(q) + sha(k) + sha(v)),
              "operand_sha": np.array("".join(sha(t) for t in operands))}
    for normalizer in (False, True):
        attend = make_flash_attention(qdq, quantized_normalizer=normalizer, qk_rotation=True)
        out = attend(q, k, v, softmax_scale=128**-0.5)
        torch.cuda.synchronize()
        arrays[f"out_{int(normalizer)}"] = out.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    out_dir.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out_dir / "wan_triton.npz", **arrays)
    print(f"wrote {out_dir / 'wan_triton.npz'}")


if __name__ == "__main__":
    main()
