"""HiF4 quantizer restated in numpy (test infrastructure; see ``oracle/__init__.py``).

Restates ``src/faquant/hif4.py`` of the reference:

- ``_e6m2_scale`` (hif4.py:91-115): ``s = bf16(max * bf16(1/d))``, clamped to
  ``[2^-48, 49152]``, rounded half-to-even onto the E6M2 grid, ``rec = bf16(1/s)``;
- ``fit_hif4_compact_parameters`` (hif4.py:142-219): the per-8 (lv2) and per-4
  (lv3) one-bit exponents for the level variants ``123``, ``12`` and ``13``;
- ``quantize_hif4_with_parameters`` (hif4.py:254-271):
  ``m = min(floor(|x| * qm * 4 + 0.5), 7)``, ``y = sign(x) * m/4 * ds``;
- ``_group_for_hif4`` / ``fake_quantize_hif4`` (hif4.py:345-390): zero padding
  of the last axis to a multiple of 64.

Every step is IEEE fp32 arithmetic with one rounding, exactly as the
reference's eager torch ops, so results are bit-identical. The packed-code
view (``hif4_encode``) is this project's own storage format, defined in the
C header ``include/faquant_b200.h``.
"""

from __future__ import annotations

import numpy as np

BLOCK = 64
F32 = np.float32
SCALE_MIN = F32(2.0**-48)
SCALE_MAX = F32(49152.0)
LEVELS = ("123", "12", "13")


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=F32)
    bits = x.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(F32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.nan
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen raw bf16 bit patterns (uint16) to fp32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (RNE) and return the raw uint16 bit patterns."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def _divisor_reciprocal(levels: str) -> np.float32:
    # hif4.py:102 -- bf16(1/7) for the official format, bf16(1/3.5) otherwise.
    divisor = 7.0 if levels == "123" else 3.5
    return bf16_round(np.array([F32(1.0) / F32(divisor)], dtype=F32))[0]


def _floor_log2(s: np.ndarray) -> np.ndarray:
    # s is a positive normal fp32 value: its exponent field is floor(log2(s)).
    return ((s.view(np.uint32) >> 23) & 0xFF).astype(np.int32) - 127


def e6m2_scale(maximum: np.ndarray, levels: str = "123") -> tuple[np.ndarray, np.ndarray]:
    """E6M2 base scale and bf16 reciprocal from a block maximum (hif4.py:91-115)."""
    maximum = np.asarray(maximum, dtype=F32)
    scale = bf16_round(maximum * _divisor_reciprocal(levels))
    scale = np.clip(scale, SCALE_MIN, SCALE_MAX).astype(F32)
    exponent = _floor_log2(scale)
    scaled = np.ldexp(scale, 2 - exponent).astype(F32)  # exact, in [4, 8)
    scale = np.ldexp(np.rint(scaled), exponent - 2).astype(F32)  # half-to-even
    reciprocal = bf16_round(F32(1.0) / scale)
    return scale, reciprocal


def fit_compact(blocks: np.ndarray, levels: str = "123") -> dict[str, np.ndarray]:
    """Compact HiF4 metadata of fp32 blocks shaped ``[..., 64]`` (hif4.py:142-219).

    Returns ``scale``/``reciprocal`` shaped ``[...]``, ``lv2`` shaped ``[..., 8]``
    and ``lv3`` shaped ``[..., 8, 2]`` (exponents 0/1 as int8).
    """
    if levels not in LEVELS:
        raise ValueError(f"levels must be one of {LEVELS}, got {levels!r}")
    blocks = np.asarray(blocks, dtype=F32)
    if blocks.shape[-1] != BLOCK:
        raise ValueError("HiF4 fitting needs a final axis of 64")
    magnitude = np.abs(blocks).reshape(*blocks.shape[:-1], 8, 2, 4)
    max_lv3 = magnitude.max(axis=-1)
    max_lv2 = max_lv3.max(axis=-1)
    max_lv1 = max_lv2.max(axis=-1)
    scale, reciprocal = e6m2_scale(max_lv1, levels)
    rec2 = reciprocal[..., None]
    rec3 = reciprocal[..., None, None]
    if levels == "123":
        lv2 = (max_lv2 * rec2 >= F32(4.0)).astype(np.int8)
        threshold = np.where(lv2 > 0, F32(4.0), F32(2.0))[..., None]
        lv3 = (max_lv3 * rec3 >= threshold).astype(np.int8)
    elif levels == "12":
        lv2 = (max_lv2 * rec2 >= F32(2.0)).astype(np.int8)
        lv3 = np.zeros(max_lv3.shape, dtype=np.int8)
    else:
        lv2 = np.zeros(max_lv2.shape, dtype=np.int8)
        lv3 = (max_lv3 * rec3 >= F32(2.0)).astype(np.int8)
    return {"scale": scale, "reciprocal": reciprocal, "lv2": lv2, "lv3": lv3}


def _expand(compact: dict[str, np.ndarray], shape: tuple[int, ...]) -> tuple[np.ndarray, np.ndarray]:
    """Per-value quant multiplier and dequant scale (hif4.py:222-243)."""
    exponent = compact["lv2"][..., None].astype(np.int32) + compact["lv3"].astype(np.int32)
    qm = np.ldexp(compact["reciprocal"][..., None, None], -exponent).astype(F32)
    ds = np.ldexp(compact["scale"][..., None, None], exponent).astype(F32)
    qm = np.broadcast_to(qm[..., None], (*qm.shape, 4)).reshape(shape)
    ds = np.broadcast_to(ds[..., None], (*ds.shape, 4)).reshape(shape)
    return qm, ds


def codes_from_blocks(blocks: np.ndarray, compact: dict[str, np.ndarray]) -> np.ndarray:
    """Element magnitudes ``m`` in 0..7 (hif4.py:268-269)."""
    qm, _ = _expand(compact, blocks.shape)
    y = (np.abs(blocks).astype(F32) * qm).astype(F32) * F32(4.0)
    t = (y + F32(0.5)).astype(F32)
    return np.minimum(np.floor(t), F32(7.0)).astype(np.uint8)


def dequant_blocks(blocks_sign_negative: np.ndarray, m: np.ndarray, compact: dict[str, np.ndarray]) -> np.ndarray:
    _, ds = _expand(compact, m.shape)
    magnitude = (m.astype(F32) / F32(4.0)) * ds
    return np.where(blocks_sign_negative, -magnitude, magnitude).astype(F32)


def group(x: np.ndarray) -> tuple[np.ndarray, int]:
    """Zero-pad the last axis to a multiple of 64 and split it (hif4.py:345-357)."""
    x = np.asarray(x, dtype=F32)
    size = x.shape[-1]
    if size == 0:
        raise ValueError("HiF4 does not support an empty axis")
    pad = (-size) % BLOCK
    if pad:
        x = np.concatenate([x, np.zeros((*x.shape[:-1], pad), dtype=F32)], axis=-1)
    return x.reshape(*x.shape[:-1], -1, BLOCK), size


def fake_quantize(x: np.ndarray, levels: str = "123") -> np.ndarray:
    """HiF4 quantize-dequantize of fp32 values along the last axis (hif4.py:376-390).

    Returns fp32; every result is exactly representable in bf16.
    """
    blocks, size = group(x)
    compact = fit_compact(blocks, levels)
    m = codes_from_blocks(blocks, compact)
    out = dequant_blocks(blocks < 0, m, compact)
    return out.reshape(*out.shape[:-2], -1)[..., :size]


def hif4_encode(x: np.ndarray, levels: str = "123") -> tuple[np.ndarray, np.ndarray]:
    """Packed HiF4 codes of fp32 rows ``[R, K]``, in this project's storage format.

    - ``codes``: uint8 ``[R, K64/2]``; value ``2i`` in the low nibble, ``2i+1`` in
      the high nibble; nibble = ``sign << 3 | m`` with ``sign = x < 0``;
    - ``meta``: uint32 ``[R, K64/64]``; bits 0-7 the E6M2 scale code
      ``(e + 48) << 2 | (mantissa_quarter - 4)``, bits 8-15 the eight lv2 bits,
      bits 16-31 the sixteen lv3 bits (sub-block ``j`` of 4 values at bit ``16+j``).
    """
    x = np.asarray(x, dtype=F32)
    if x.ndim != 2:
        raise ValueError("hif4_encode expects a 2-D array")
    blocks, _ = group(x)
    compact = fit_compact(blocks, levels)
    m = codes_from_blocks(blocks, compact)
    nib = (m | ((blocks < 0).astype(np.uint8) << 3)).reshape(x.shape[0], -1)
    codes = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    scale = compact["scale"]
    e = _floor_log2(scale)
    quarter = np.ldexp(scale, 2 - e).astype(np.int32)  # 4..7
    scale_code = ((e + 48) << 2) | (quarter - 4)
    lv2_bits = np.zeros(scale.shape, dtype=np.uint32)
    for j in range(8):
        lv2_bits |= compact["lv2"][..., j].astype(np.uint32) << j
    lv3_flat = compact["lv3"].reshape(*scale.shape, 16)
    lv3_bits = np.zeros(scale.shape, dtype=np.uint32)
    for j in range(16):
        lv3_bits |= lv3_flat[..., j].astype(np.uint32) << j
    meta = (scale_code.astype(np.uint32) | (lv2_bits << 8) | (lv3_bits << 16)).astype(np.uint32)
    return codes, meta


def hif4_decode(codes: np.ndarray, meta: np.ndarray, k: int) -> np.ndarray:
    """Inverse of ``hif4_encode``: fp32 ``[R, k]`` dequantized values."""
    rows = codes.shape[0]
    nib = np.empty((rows, codes.shape[1] * 2), dtype=np.uint8)
    nib[:, 0::2] = codes & 0xF
    nib[:, 1::2] = codes >> 4
    m = (nib & 7).astype(F32).reshape(rows, -1, 8, 2, 4)
    neg = (nib >> 3).astype(bool).reshape(m.shape)
    scale_code = (meta & 0xFF).astype(np.int32)
    e = (scale_code >> 2) - 48
    scale = np.ldexp(F32(1.0) + F32(0.25) * (scale_code & 3).astype(F32), e).astype(F32)
    lv2 = np.stack([(meta >> (8 + j)) & 1 for j in range(8)], axis=-1).astype(np.int32)
    lv3 = np.stack([(meta >> (16 + j)) & 1 for j in range(16)], axis=-1).astype(np.int32)
    lv3 = lv3.reshape(*meta.shape, 8, 2)
    ds = np.ldexp(scale[..., None, None], lv2[..., None] + lv3).astype(F32)[..., None]
    magnitude = (m / F32(4.0)) * ds
    out = np.where(neg, -magnitude, magnitude).astype(F32)
    return out.reshape(rows, -1)[:, :k]
