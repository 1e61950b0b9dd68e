"""Input rotations restated in numpy (test infrastructure; see ``oracle/__init__.py``).

- ``hadamard`` restates ``hadamard_transform`` (``src/faquant/rotation.py:14-29``):
  butterfly stages of stride 1, 2, 4, ..., n/2, each producing ``(l + r, l - r)``,
  then one fp32 division by ``fp32(sqrt(n))``. The division is a correctly
  rounded fp32 divide, as torch's CPU ``tensor / python_float`` is; it is exact
  for n = 4^j.
- ``block_hadamard`` restates ``chunked_block_hadamard_transform``
  (``rotation.py:117-135``): independent transforms of consecutive blocks.
- ``rotate_input`` restates the rotation block of ``FakeQuantLinear.forward``
  (``src/faquant/quantization.py:200-221``): ``x * signs`` in fp32, gather by the
  permutation, block Hadamard, then one rounding to the input dtype.
"""

from __future__ import annotations

import math

import numpy as np

from .hif4 import F32, bf16_round


def hadamard(x: np.ndarray) -> np.ndarray:
    """Normalized Walsh-Hadamard transform over the last axis, fp32."""
    x = np.asarray(x, dtype=F32)
    n = x.shape[-1]
    if n <= 0 or n & (n - 1):
        raise ValueError(f"Hadamard dimension must be a power of two, got {n}")
    shape = x.shape
    out = x.reshape(-1, n)
    stride = 1
    while stride < n:
        work = out.reshape(-1, n // (2 * stride), 2, stride)
        left = work[:, :, 0, :]
        right = work[:, :, 1, :]
        out = np.concatenate((left + right, left - right), axis=2).reshape(-1, n)
        stride *= 2
    return (out / F32(math.sqrt(n))).astype(F32).reshape(shape)


def block_hadamard(x: np.ndarray, block: int) -> np.ndarray:
    x = np.asarray(x, dtype=F32)
    if block <= 0 or block & (block - 1) or x.shape[-1] % block:
        raise ValueError(f"dimension {x.shape[-1]} must be divisible by power-of-two block={block}")
    return hadamard(x.reshape(-1, block)).reshape(x.shape)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_round(x)
    if dtype == "f32":
        return np.asarray(x, dtype=F32)
    raise ValueError(f"unsupported dtype {dtype!r}")


def rotate_input(
    x: np.ndarray,
    signs: np.ndarray,
    permutation: np.ndarray,
    block: int | None,
    dtype: str = "bf16",
) -> np.ndarray:
    """``FakeQuantLinear`` input rotation; ``x`` holds values of ``dtype`` as fp32."""
    work = np.asarray(x, dtype=F32) * np.asarray(signs, dtype=F32)
    work = np.take(work, np.asarray(permutation, dtype=np.int64), axis=-1)
    if block is not None:
        work = block_hadamard(work, block)
    return round_to(work, dtype)
