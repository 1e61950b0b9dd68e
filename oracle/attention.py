"""HiF4 QK/PV attention restated in numpy (test infrastructure).

- ``qk_pretransform`` restates the post-RoPE block of ``qwen3._attention_forward``
  (``src/faquant/qwen3.py:101-130``) and Wan's ``self_forward`` +
  ``rotate_heads`` (``src/faquant/wan22_attention.py:186-192, 257-259``): one fp32
  excursion ``k - offset``, ``q * s``, ``k / s`` (true division), a Hadamard over
  ``head_dim`` and a single rounding to bf16.
- ``attention`` restates ``simulated_flash_attention_forward``
  (``src/faquant/simulated_flash_attention.py:457-909``) for HiF4 operands with
  no attention mask: K/V QDQ before the GQA repeat (``:588-611``), Q QDQ
  (``:613-619``), fp32 scores times ``scale`` (``:723-727``), bottom-right causal
  masking (``_streaming_mask :371-427``), online softmax with ``exp`` against the
  running max that includes the current key tile (``:788-799``), HiF4 QDQ of P
  along the keys of each key tile in groups of 64 with a zero-padded tail
  (``:800-805``, ``_fake_quantize_tail :292-338``), the denominator from the
  unquantized P or, under ``quantized_same`` (P-Reordering), from the quantized P
  (``:824-834``), fp32 PV (``:848-850``) and ``acc / denominator`` cast to bf16
  (``:870-884``). Fully-future key tiles are skipped, which the reference shows to
  be bitwise identical to processing them (``:676-699``).
"""

from __future__ import annotations

import numpy as np

from . import hif4
from .hif4 import F32, bf16_round
from .rotation import hadamard


def qk_pretransform(
    q: np.ndarray,
    k: np.ndarray,
    *,
    smooth_scale: np.ndarray | None = None,
    key_offset: np.ndarray | None = None,
    rotate: bool = True,
) -> tuple[np.ndarray, np.ndarray]:
    """Post-RoPE Q/K transform; ``q [B,H,S,D]``, ``k [B,KV,S,D]``; bf16 values as fp32.

    ``smooth_scale`` is ``[D]`` (shared) or ``[H, D]`` (per head, Wan);
    ``key_offset`` is ``[KV, D]``.
    """
    qf = np.asarray(q, dtype=F32)
    kf = np.asarray(k, dtype=F32)
    if key_offset is not None:
        kf = (kf - np.asarray(key_offset, dtype=F32)[None, :, None, :]).astype(F32)
    if smooth_scale is not None:
        s = np.asarray(smooth_scale, dtype=F32)
        if s.ndim == 1:
            qs, ks = s, s
        else:
            qs = s[None, :, None, :]
            ks = s[None, :, None, :]
        qf = (qf * qs).astype(F32)
        kf = (kf / ks).astype(F32)
    if rotate:
        qf = hadamard(qf)
        kf = hadamard(kf)
    return bf16_round(qf), bf16_round(kf)


def _qdq_tail(x: np.ndarray, levels: str) -> np.ndarray:
    return hif4.fake_quantize(x, levels)


def attention(
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    *,
    causal: bool = True,
    scale: float | None = None,
    qk_quant: bool = True,
    pv_quant: bool = True,
    normalizer: str = "quantized_same",
    query_chunk: int = 256,
    key_chunk: int = 128,
    levels: dict[str, str] | None = None,
    return_f32: bool = False,
    operands_quantized: bool = False,
    query_positions: np.ndarray | None = None,
    full_queries: int | None = None,
) -> np.ndarray:
    """Tiled HiF4 attention; ``q [B,H,Sq,D]``, ``k/v [B,KV,Sk,D]`` -> ``[B,Sq,H,D]``.

    ``operands_quantized``: Q/K/V are already HiF4 operands (a kernel's K4 output) and
    are used as given (re-fitting HiF4 values is not idempotent); P is still quantized
    when ``pv_quant``.

    ``query_positions``: the position of each query row in the full query sequence of
    ``n`` rows, whose causal offset is ``sk - n`` -- i.e. the key index of row i's
    diagonal is ``query_positions[i] + sk - n``; pass ``n`` as ``full_queries``. Every
    output row depends only on its own query and on all keys (the key tiling, the
    running max and P's HiF4 groups are per row), so a subset of rows computed this way
    equals those rows of the full computation; tests use it to check sampled rows of
    sequences too long for the whole oracle."""
    if normalizer not in ("unquantized", "quantized_same"):
        raise ValueError(f"unsupported normalizer {normalizer!r}")
    lv = {"q": "123", "k": "123", "p": "123", "v": "123"}
    lv.update(levels or {})
    q = np.asarray(q, dtype=F32)
    k = np.asarray(k, dtype=F32)
    v = np.asarray(v, dtype=F32)
    b, h, sq, d = q.shape
    kv, sk = k.shape[1], k.shape[2]
    if h % kv:
        raise ValueError("query heads must be divisible by key/value heads")
    rep = h // kv
    scale = F32(scale if scale is not None else d**-0.5)
    qo = _qdq_tail(q, lv["q"]) if qk_quant and not operands_quantized else q
    ko = _qdq_tail(k, lv["k"]) if qk_quant and not operands_quantized else k
    vo = _qdq_tail(v, lv["v"]) if pv_quant and not operands_quantized else v
    ko = np.repeat(ko, rep, axis=1)
    vo = np.repeat(vo, rep, axis=1)
    out = np.zeros((b, h, sq, d), dtype=F32)
    if query_positions is None:
        diag = np.arange(sq) + (sk - sq)
    else:
        diag = np.asarray(query_positions, dtype=np.int64) + (sk - full_queries)
        if diag.shape != (sq,):
            raise ValueError("query_positions needs one position per query row")
    for qs in range(0, sq, query_chunk):
        qe = min(qs + query_chunk, sq)
        rows = qe - qs
        qt = qo[:, :, qs:qe]
        run_max = np.full((b, h, rows, 1), -np.inf, dtype=F32)
        denom = np.zeros((b, h, rows, 1), dtype=F32)
        acc = np.zeros((b, h, rows, d), dtype=F32)
        qpos = diag[qs:qe]
        for ks in range(0, sk, key_chunk):
            ke = min(ks + key_chunk, sk)
            if causal and ks > qpos.max():
                continue
            scores = (qt @ np.swapaxes(ko[:, :, ks:ke], -1, -2)).astype(F32) * scale
            if causal:
                allowed = np.arange(ks, ke)[None, :] <= qpos[:, None]
                scores = np.where(allowed, scores, -np.inf).astype(F32)
            block_max = scores.max(axis=-1, keepdims=True)
            new_max = np.maximum(run_max, block_max)
            with np.errstate(invalid="ignore"):
                prev = np.where(np.isfinite(run_max), np.exp(run_max - new_max), F32(0)).astype(F32)
                probs = np.where(np.isfinite(scores), np.exp(scores - new_max), F32(0)).astype(F32)
            pq = _qdq_tail(probs, lv["p"]) if pv_quant else probs
            source = pq if normalizer == "quantized_same" else probs
            denom = (prev * denom + source.sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)
            acc = (prev * acc + (pq @ vo[:, :, ks:ke]).astype(F32)).astype(F32)
            run_max = new_max
        tiny = np.finfo(F32).tiny
        with np.errstate(invalid="ignore", divide="ignore"):
            normalized = np.where(denom > 0, acc / np.maximum(denom, tiny), F32(0)).astype(F32)
        out[:, :, qs:qe] = normalized
    out = np.swapaxes(out, 1, 2)
    return out if return_f32 else bf16_round(out)


def attention_flops(heads: int, sq: int, sk: int, d: int, causal: bool, batch: int = 1) -> float:
    """Algorithmic QK^T + PV FLOPs: 4 * d per valid (query, key) pair."""
    if causal:
        offset = sk - sq
        pairs = sum(max(0, min(sk, q + offset + 1)) for q in range(sq)) if sq < 4096 else _causal_pairs(sq, sk)
    else:
        pairs = sq * sk
    return 4.0 * d * heads * batch * pairs


def _causal_pairs(sq: int, sk: int) -> float:
    offset = sk - sq
    start = max(0, -offset)  # queries with no valid key contribute 0
    first = start + offset + 1
    last = sq - 1 + offset + 1
    n = sq - start
    return n * (first + last) / 2.0

