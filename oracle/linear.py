"""``FakeQuantLinear`` forward restated in numpy (test infrastructure).

Restates ``src/faquant/quantization.py:199-277`` for ``quant_format="hif4"``:
optional input scale (in the input dtype), optional HiSQ rotation
(``oracle.rotation.rotate_input``), HiF4 fake quantization of the activations
(``hif4.py:376``), then ``F.linear`` against HiF4-grid weights. The GEMM here is
the fp32 fake-quant product ``Xq @ Wq.T`` of the exactly-dequantized operands,
the quantity the CUDA GEMM is compared with inside a tolerance.
"""

from __future__ import annotations

import numpy as np

from . import hif4
from .rotation import F32, round_to, rotate_input


def quantize_activations(
    x: np.ndarray,
    *,
    levels: str = "123",
    dtype: str = "bf16",
    input_scale: np.ndarray | None = None,
    signs: np.ndarray | None = None,
    permutation: np.ndarray | None = None,
    block: int | None = None,
) -> np.ndarray:
    """Activation path of ``FakeQuantLinear.forward`` up to (excluding) ``F.linear``."""
    x = np.asarray(x, dtype=F32)
    if input_scale is not None:
        x = round_to(x * np.asarray(input_scale, dtype=F32), dtype)
    if signs is not None:
        perm = np.arange(x.shape[-1]) if permutation is None else permutation
        x = rotate_input(x, signs, perm, block, dtype)
    return hif4.fake_quantize(x, levels)


def quantize_weight_rtn(w: np.ndarray, levels: str = "123") -> np.ndarray:
    """RTN weight quantization of ``FakeQuantLinear.__init__`` (quantization.py:169-184)."""
    return hif4.fake_quantize(np.asarray(w, dtype=F32), levels)


def fake_quant_linear(
    x: np.ndarray,
    w_quantized: np.ndarray,
    bias: np.ndarray | None = None,
    **kwargs,
) -> np.ndarray:
    """fp32 ``Xq @ Wq.T (+ bias)`` of the fake-quantized activations."""
    xq = quantize_activations(x, **kwargs)
    y = xq.reshape(-1, xq.shape[-1]) @ np.asarray(w_quantized, dtype=F32).T
    if bias is not None:
        y = y + np.asarray(bias, dtype=F32)
    return y.reshape(*xq.shape[:-1], -1).astype(F32)
