"""Qwen3 attention adapter on B200: the post-RoPE Q/K transform and the patched forward.

Mirrors ``qwen3._attention_forward`` (``src/faquant/qwen3.py:56-172``) with the same
``module.faquant_*`` attribute contract (installed by the reference's
``install_qwen3_attention_adapter :175-279`` and ``apply_qwen3_qk_smooth_scales
:282-346``): q/k/v projections, q_norm/k_norm, RoPE, then one fp32 excursion for
``k - offset``, Smooth-QK ``q * s`` / ``k / s`` and the Hadamard over head_dim with a
single bf16 rounding -- here one K4 launch per operand -- then the HiF4 attention
backend (``faquant_b200.attention``) and ``o_proj``.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ops
from .attention import simulated_flash_attention_forward


def qk_pretransform(module, query_states: torch.Tensor, key_states: torch.Tensor):
    """Post-RoPE Q/K transform of ``qwen3.py:92-130`` on ``[B, H, S, D]`` tensors."""
    smooth = getattr(module, "faquant_qk_smooth_scale", None)
    delta = getattr(module, "faquant_qk_smooth_delta", None)
    if delta is not None:
        if smooth is None:
            raise RuntimeError("Smooth-QK delta requires a frozen base scale")
        smooth = smooth * delta.float().exp()
    offset = getattr(module, "faquant_qk_key_offset", None)
    rotate = bool(getattr(module, "faquant_qk_rotation", False))
    if smooth is None and offset is None and not rotate:
        return query_states, key_states
    head_dim = query_states.shape[-1]
    block = getattr(module, "faquant_qk_rotation_block_size", None)
    if rotate and block not in (None, head_dim):
        raise NotImplementedError("a block Hadamard narrower than head_dim is not implemented by faquant_b200")
    if query_states.dtype != torch.bfloat16 or key_states.dtype != torch.bfloat16:
        raise NotImplementedError("the fused Q/K transform rounds to bf16; bf16 Q/K are required")
    if offset is not None:
        offset = offset.reshape(key_states.shape[1], head_dim)
    q, _, _ = ops.qk_prep(query_states, levels=None, rotate=rotate, smooth_scale=smooth,
                          smooth_mode=None if smooth is None else "mul")
    k, _, _ = ops.qk_prep(key_states, levels=None, rotate=rotate, smooth_scale=smooth,
                          smooth_mode=None if smooth is None else "div", key_offset=offset)
    return q, k


def attention_forward(
    self,
    hidden_states: torch.Tensor,
    position_embeddings: tuple[torch.Tensor, torch.Tensor],
    attention_mask: Optional[torch.Tensor],
    past_key_values=None,
    cache_position: Optional[torch.LongTensor] = None,
    **kwargs,
):
    """Drop-in for ``Qwen3Attention.forward`` as patched by the reference (``qwen3.py:56-172``)."""
    from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb

    legacy = kwargs.pop("past_key_value", None)
    if past_key_values is None:
        past_key_values = legacy
    input_shape = hidden_states.shape[:-1]
    hidden_shape = (*input_shape, -1, self.head_dim)
    query_states = self.q_norm(self.q_proj(hidden_states).view(hidden_shape)).transpose(1, 2)
    key_states = self.k_norm(self.k_proj(hidden_states).view(hidden_shape)).transpose(1, 2)
    value_states = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
    cos, sin = position_embeddings
    query_states, key_states = apply_rotary_pos_emb(query_states, key_states, cos, sin)
    query_states, key_states = qk_pretransform(self, query_states, key_states)
    if getattr(self, "faquant_attention_input_quant", False):
        quant_kwargs = self.faquant_core_quant_kwargs
        if quant_kwargs.get("quant_format") != "hif4":
            raise NotImplementedError("faquant_b200 implements HiF4 attention-input quantization only")
        query_states = ops.qk_prep(query_states, levels=ops.default_levels("act"), rotate=False)[0]
        key_states = ops.qk_prep(key_states, levels=ops.default_levels("act"), rotate=False)[0]
        value_states = ops.qk_prep(value_states, levels=ops.default_levels("act"), rotate=False)[0]
    if past_key_values is not None:
        cache_kwargs = {"sin": sin, "cos": cos, "cache_position": cache_position}
        key_states, value_states = past_key_values.update(key_states, value_states, self.layer_idx, cache_kwargs)
    kernel = getattr(self, "faquant_attention_kernel", "simulated")
    if kernel == "simulated":  # the HiF4 attention of this package
        kwargs["cache_position"] = cache_position
        interface = simulated_flash_attention_forward
    elif kernel == "native":  # the model's own attention on the transformed Q/K (qwen3.py:147-152)
        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
        from transformers.models.qwen3.modeling_qwen3 import eager_attention_forward

        impl = self.config._attn_implementation
        interface = eager_attention_forward if impl == "eager" else ALL_ATTENTION_FUNCTIONS[impl]
    else:
        raise NotImplementedError("the differentiable (training) attention kernel is not part of faquant_b200")
    attn_output, attn_weights = interface(
        self, query_states, key_states, value_states, attention_mask, dropout=0.0, scaling=self.scaling,
        sliding_window=getattr(self, "sliding_window", None), **kwargs)
    attn_output = attn_output.reshape(*input_shape, -1).contiguous()
    if getattr(self, "faquant_attention_output_quant", False) and not getattr(self.o_proj, "faquant_quantizes_input", False):
        attn_output = ops.hif4_quantize(attn_output, levels=ops.default_levels("act"))[0]
    return self.o_proj(attn_output), attn_weights
