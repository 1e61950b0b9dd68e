"""HiF4 QK/PV attention backend: the drop-in for ``faquant.simulated_flash_attention``.

``simulated_flash_attention_forward`` keeps the reference's HF attention-backend
contract (``src/faquant/simulated_flash_attention.py:457-909``): it takes
``(module, query [B,H,S,D], key [B,KV,S,D], value, attention_mask, dropout, scaling,
sliding_window, softcap, **kwargs)``, reads the same ``module.faquant_*`` runtime
attributes, updates ``module.faquant_simulated_attention_stats`` with the same
counters, and returns ``(out [B,S,H,D], None)``. The work is two launches per
operand of the C-ABI library: K4 (HiF4 QDQ of Q, K, V along head_dim, levels per
operand from the same environment variables as ``hif4.py:13-43``) and K5 (the
tcgen05 flash attention with HiF4 P and the chosen normalizer).

Supported, as in every configuration the reference deploys: HiF4 operands in
groups of 64 (or no operand quantization), head_dim 128, key chunk 128 (the P
groups and the running-max schedule of the simulator), any query chunk (rows are
independent), causal bottom-right or non-causal, GQA, and an attention mask that
is ``None`` or an all-valid 2-D mask (which the reference itself reduces to
``None`` for prefill, ``:531-546``). Everything else raises ``NotImplementedError``
(no CPU fallback): padding masks, sliding windows, softcap, non-HiF4 formats.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import ops

SIMULATED_ATTENTION_IMPLEMENTATION = "faquant_simulated"
B200_ATTENTION_IMPLEMENTATION = "faquant_b200"
PV_NORMALIZER_MODES = ("unquantized", "quantized_same")
_QUANTIZED_OPERANDS = ("q", "k", "p", "v")


def new_simulated_attention_stats() -> dict[str, int]:
    """Zeroed counters, the same keys as the reference (``simulated_flash_attention.py:18-33``)."""
    stats = {"calls": 0, "qk_tiles": 0, "pv_tiles": 0, "qk_quantized_tiles": 0, "pv_quantized_tiles": 0}
    for operand in _QUANTIZED_OPERANDS:
        stats[f"{operand}_quant_calls"] = 0
        stats[f"{operand}_quantized_values"] = 0
        stats[f"{operand}_quant_blocks"] = 0
        stats[f"{operand}_quant_padding_values"] = 0
    return stats


def _hif4_kwargs(kwargs: dict | None, what: str) -> bool:
    """True when ``kwargs`` describe HiF4 group-64 operands; raise for other formats."""
    if kwargs is None:
        return False
    fmt = kwargs.get("quant_format", "int")
    if fmt != "hif4":
        raise NotImplementedError(f"{what}: faquant_b200 implements HiF4 attention operands only, got {fmt!r}")
    if kwargs.get("group_size", 64) not in (64, -1) or kwargs.get("bits", 4) != 4:
        raise NotImplementedError(f"{what}: HiF4 operands need bits=4 and group_size=64")
    return True


def _record(stats, operand, vectors, width, group, repeats):
    groups = math.ceil(width / group)
    stats[f"{operand}_quant_calls"] += repeats
    stats[f"{operand}_quantized_values"] += vectors * width * repeats
    stats[f"{operand}_quant_blocks"] += vectors * groups * repeats
    stats[f"{operand}_quant_padding_values"] += vectors * (groups * group - width) * repeats


def _tile_schedule(sq: int, sk: int, query_chunk: int, key_chunk: int, causal: bool):
    """(query tile rows, active key tiles) per query-tile group, as the simulator walks them."""
    out = []
    full = sq // query_chunk
    groups = []
    if full:
        groups.append((0, query_chunk, full))
    if full * query_chunk < sq:
        groups.append((full * query_chunk, sq - full * query_chunk, 1))
    offset = sk - sq
    for start, rows, count in groups:
        for key_start in range(0, sk, key_chunk):
            active_start = 0
            if causal:
                active_start = max(0, min(count, (key_start - offset - start) // rows))
            active = count - active_start
            if active:
                out.append((rows, active, min(key_chunk, sk - key_start)))
    return out


def _update_stats(module, b, h, kv, sq, sk, d, query_chunk, key_chunk, causal, qk_quant, pv_quant) -> None:
    """The simulator's geometry counters (``simulated_flash_attention.py:187-211, 637-866``)."""
    stats = getattr(module, "faquant_simulated_attention_stats", None)
    if stats is None:
        return
    schedule = _tile_schedule(sq, sk, query_chunk, key_chunk, causal)
    tiles = sum(active for _, active, _ in schedule)
    group = 64
    if qk_quant:
        full = sq // query_chunk
        if full:
            _record(stats, "q", b * h * query_chunk, d, group, full)
        if full * query_chunk < sq:
            _record(stats, "q", b * h * (sq - full * query_chunk), d, group, 1)
    for rows, active, kt in schedule:
        if qk_quant:
            _record(stats, "k", b * h * kt, d, group, active)
        if pv_quant:
            _record(stats, "p", b * h * rows, kt, group, active)
            _record(stats, "v", b * h * kt, d, group, active)
    stats["calls"] += 1
    stats["qk_tiles"] += tiles
    stats["pv_tiles"] += tiles
    if qk_quant:
        stats["qk_quantized_tiles"] += tiles
    if pv_quant:
        stats["pv_quantized_tiles"] += tiles


DECODE_MAX_QUERIES = 16  # query positions up to which a causal call runs the decode kernel


def _cached_decode_quantize(module, tensor: torch.Tensor, operand: str, enabled: bool, query_length: int):
    """K/V HiF4 operands with the reference's append cache (``_cached_decode_quantize``,
    ``simulated_flash_attention.py:243-289``): HiF4 groups run along head_dim only, so a
    decode step quantizes just the appended position and concatenates it to the cached
    operand -- identical to re-quantizing the whole cache."""
    name = f"faquant_{operand}_matmul_qdq_cache"
    if not enabled:
        setattr(module, name, None)
        return tensor.to(torch.bfloat16)
    cached = getattr(module, name, None)
    can_append = (
        query_length == 1
        and isinstance(cached, torch.Tensor)
        and cached.device == tensor.device
        and cached.dtype == torch.bfloat16
        and cached.shape[:-2] == tensor.shape[:-2]
        and cached.shape[-1] == tensor.shape[-1]
        and cached.shape[-2] + 1 == tensor.shape[-2]
    )
    levels = ops.default_levels(operand)
    if can_append:
        tail = ops.qk_prep(tensor[..., cached.shape[-2]:, :], levels=levels, rotate=False)[0]
        quantized = torch.cat((cached, tail), dim=-2)
    else:
        quantized = ops.qk_prep(tensor, levels=levels, rotate=False)[0]
    setattr(module, name, quantized)
    return quantized


def simulated_flash_attention_forward(
    module: torch.nn.Module,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    attention_mask: Optional[torch.Tensor],
    dropout: float = 0.0,
    scaling: Optional[float] = None,
    sliding_window: Optional[int] = None,
    softcap: Optional[float] = None,
    **kwargs: object,
) -> tuple[torch.Tensor, None]:
    """Tiled HiF4 flash attention on B200; the reference's backend contract."""
    if dropout:
        raise ValueError("simulated FlashAttention only supports dropout=0 inference")
    if softcap is not None:
        raise NotImplementedError("softcap is not implemented by faquant_b200")
    if sliding_window is not None:
        raise NotImplementedError("sliding windows are not implemented by faquant_b200")
    if kwargs.get("output_attentions", False):
        raise ValueError("simulated FlashAttention does not materialize attention weights")
    if query.ndim != 4 or key.ndim != 4 or value.ndim != 4:
        raise ValueError("simulated FlashAttention expects rank-4 Q/K/V tensors")
    if key.shape != value.shape:
        raise ValueError("simulated FlashAttention requires matching K/V shapes")
    if query.shape[0] != key.shape[0] or query.shape[-1] != key.shape[-1]:
        raise ValueError("simulated FlashAttention received incompatible Q/K shapes")
    if any(kwargs.get(n) is not None for n in ("cu_seq_lens_q", "cu_seq_lens_k", "max_length_q", "max_length_k")):
        raise NotImplementedError("packed cu_seqlens are not supported")
    valid_key_length = key.shape[-2]
    if attention_mask is not None:
        valid_key_length = min(valid_key_length, attention_mask.shape[-1])
    cache_position = kwargs.get("cache_position")
    if isinstance(cache_position, torch.Tensor) and cache_position.numel():
        valid_key_length = min(valid_key_length, int(cache_position.max().item()) + 1)
    if valid_key_length < key.shape[-2]:
        key = key[:, :, :valid_key_length]
        value = value[:, :, :valid_key_length]
    b, h, sq, d = query.shape
    _, kv, sk, _ = key.shape
    if h % kv:
        raise ValueError("query heads must be divisible by key/value heads")
    if any(size == 0 for size in query.shape) or sk == 0:
        raise ValueError("simulated FlashAttention does not support zero dimensions")
    if attention_mask is not None:
        if attention_mask.ndim == 2 and bool(torch.all(attention_mask[:, -sk:]).item()):
            attention_mask = None  # the reference's all-valid prefill normalization
        else:
            raise NotImplementedError("padding / 4-D attention masks are not implemented by faquant_b200")
    scale = float(scaling if scaling is not None else d**-0.5)
    query_chunk = int(module.faquant_attention_query_chunk_size)
    key_chunk = int(module.faquant_attention_key_chunk_size)
    if key_chunk != 128:
        raise NotImplementedError("faquant_b200 attention runs key tiles of 128 (faquant_attention_key_chunk_size)")
    quant_kwargs = module.faquant_matmul_quant_kwargs
    qk_kwargs = getattr(module, "faquant_qk_matmul_quant_kwargs", quant_kwargs)
    pv_kwargs = getattr(module, "faquant_pv_matmul_quant_kwargs", quant_kwargs)
    qk_quant = bool(module.faquant_qk_matmul_quant)
    pv_quant = bool(module.faquant_pv_matmul_quant)
    if qk_quant:
        _hif4_kwargs(qk_kwargs, "QK operands")
    if pv_quant:
        _hif4_kwargs(pv_kwargs, "PV operands")
    mode = getattr(module, "faquant_pv_normalizer_mode", "unquantized")
    if mode not in PV_NORMALIZER_MODES:
        raise ValueError(f"unsupported pv_normalizer_mode {mode!r}; expected one of {PV_NORMALIZER_MODES}")
    requested = kwargs.get("is_causal")
    causal = bool(getattr(module, "is_causal", True) if requested is None else requested)
    if d != 128:
        raise NotImplementedError("faquant_b200 attention needs head_dim 128")

    qo = ops.qk_prep(query, levels=ops.default_levels("q"), rotate=False)[0] if qk_quant else query.to(torch.bfloat16)
    ko = _cached_decode_quantize(module, key, "k", qk_quant, sq)
    vo = _cached_decode_quantize(module, value, "v", pv_quant, sq)
    p_levels = ops.default_levels("p") if pv_quant else None
    if causal and sq <= DECODE_MAX_QUERIES and (h // kv) * sq <= 32:
        # a decode step: K6 spreads the cache over the GPU with the same semantics
        out = ops.hif4_decode_attention(qo, ko, vo, scale=scale, p_levels=p_levels,
                                        quantized_normalizer=mode == "quantized_same")
    else:
        out = ops.hif4_attention(qo, ko, vo, scale=scale, causal=causal, p_levels=p_levels,
                                 quantized_normalizer=mode == "quantized_same")
    _update_stats(module, b, h, kv, sq, sk, d, query_chunk, key_chunk, causal, qk_quant, pv_quant)
    return (out if out.dtype == query.dtype else out.to(query.dtype)), None


def register_simulated_attention_backend(name: str = B200_ATTENTION_IMPLEMENTATION) -> None:
    """Register the backend with transformers (``simulated_flash_attention.py:214-228``)."""
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS, flash_attention_mask
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    ALL_ATTENTION_FUNCTIONS.register(name, simulated_flash_attention_forward)
    ALL_MASK_ATTENTION_FUNCTIONS.register(name, flash_attention_mask)
