"""Quantized prefill, then BF16 greedy decode: the generation loop of the reference's
LongBench evaluation (``eval_longbench._prefill_quant_decode_bf16_generate``,
src/faquant/workflows/eval_longbench.py:495-576).

The prompt runs through the HiF4 model -- in chunks when the model carries
``_faquant_prefill_chunk_tokens`` (a multiple of the attention's 256-query tile keeps every
attention tile and every token-local quantizer exactly as in one pass; the attention
backend of this package runs chunked prefill bit-identically) -- keeping only the last
position's logits. The first token is the argmax of those logits; the K/V QDQ copies
kept for quantized decode appends (``faquant_k_matmul_qdq_cache`` /
``faquant_v_matmul_qdq_cache`` on each attention module) are then released, and the
remaining tokens come greedily from the BF16 model stored as
``_faquant_bf16_decode_model``, which continues on the same K/V cache.

Only batch 1, greedy, one beam, as in the reference; the others raise ``ValueError``.
Both models follow the Hugging Face calling convention (keyword ``input_ids``,
``past_key_values``, ``cache_position``, ``use_cache``, ``return_dict``; the prefill model
also ``logits_to_keep``) and return an object with ``logits`` and ``past_key_values``.
"""

from __future__ import annotations

import torch


def _stopped(stopping_criteria, sequence: torch.Tensor, scores: torch.Tensor) -> bool:
    """eval_longbench.py:495-501: a criteria object may answer with a tensor (all rows
    must agree to stop) or a plain bool."""
    if stopping_criteria is None:
        return False
    verdict = stopping_criteria(sequence, scores)
    if isinstance(verdict, torch.Tensor):
        return bool(verdict.all().item())
    return bool(verdict)


def _eos_ids(model, generation_kwargs: dict) -> set[int]:
    eos = generation_kwargs.get("eos_token_id", model.generation_config.eos_token_id)
    if eos is None:
        return set()
    return {int(eos)} if isinstance(eos, int) else {int(token) for token in eos}


def release_decode_qdq_caches(model) -> None:
    """Drop every attention module's K/V HiF4 append cache (only quantized decode
    appends use them; BF16 decode would otherwise hold a second K/V cache)."""
    for layer in model.model.layers:
        layer.self_attn.faquant_k_matmul_qdq_cache = None
        layer.self_attn.faquant_v_matmul_qdq_cache = None


@torch.inference_mode()
def prefill_quant_decode_bf16_generate(
    model,
    *,
    input_ids: torch.Tensor,
    max_length: int,
    stopping_criteria=None,
    **generation_kwargs,
) -> torch.Tensor:
    """``input_ids [1, S]`` -> ``[1, S + generated]`` (see the module docstring)."""
    if input_ids.shape[0] != 1:
        raise ValueError("prefill-only quantization requires batch size 1")
    if generation_kwargs.get("do_sample", False):
        raise ValueError("prefill-only quantization currently supports greedy decode")
    if int(generation_kwargs.get("num_beams", 1)) != 1:
        raise ValueError("prefill-only quantization currently supports one beam")

    decode_model = model.__dict__["_faquant_bf16_decode_model"]
    length = input_ids.shape[-1]
    chunk = int(model.__dict__.get("_faquant_prefill_chunk_tokens") or length)
    device = input_ids.device

    cache, outputs = None, None
    for begin in range(0, length, chunk):
        end = min(begin + chunk, length)
        outputs = model(input_ids=input_ids[:, begin:end], past_key_values=cache,
                        cache_position=torch.arange(begin, end, device=device), use_cache=True,
                        return_dict=True, logits_to_keep=1)
        cache = outputs.past_key_values
    release_decode_qdq_caches(model)

    scores = outputs.logits[:, -1, :]
    next_token = scores.argmax(dim=-1, keepdim=True)
    sequence = torch.cat((input_ids, next_token), dim=-1)
    eos_ids = _eos_ids(model, generation_kwargs)
    while sequence.shape[-1] < max_length:
        if int(next_token.item()) in eos_ids or _stopped(stopping_criteria, sequence, scores):
            break
        position = torch.tensor([cache.get_seq_length()], device=device, dtype=torch.long)
        outputs = decode_model(input_ids=next_token, past_key_values=cache, cache_position=position,
                               use_cache=True, return_dict=True)
        cache = outputs.past_key_values
        scores = outputs.logits[:, -1, :]
        next_token = scores.argmax(dim=-1, keepdim=True)
        sequence = torch.cat((sequence, next_token), dim=-1)
    return sequence
