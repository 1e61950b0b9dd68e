"""Wan2.2 DiT drop-ins on B200: HiF4 W4A4 block Linears and HiF4 flash attention.

Mirrors ``src/faquant/wan22_hif4.py`` (``faquant_qdq :35``, ``HiF4Linear :51-92``,
``quantize_dit_blocks :121-148``) and ``src/faquant/wan22_attention.py``
(``hif4_attention :165-183``, ``rotate_heads :186-192``, ``make_flash_attention
:195-228``, ``patch_attention_modules :231-272``). ``input_qdq`` callables made by
``faquant_qdq`` run on the K1 kernel (with an optional fused block-Hadamard reader
rotation, the ``rbhn_r64`` composition of BASELINE config 4); any other callable is
called as given. The Triton kernel of the reference is replaced by K5 (non-causal,
all batch elements in one launch).
"""

from __future__ import annotations

import contextvars
from typing import Callable, Mapping

import torch
from torch import nn

from . import ops

KEY_TILE = 128
BLOCK_LINEARS = (
    "self_attn.q", "self_attn.k", "self_attn.v", "self_attn.o",
    "cross_attn.q", "cross_attn.k", "cross_attn.v", "cross_attn.o",
    "ffn.0", "ffn.2",
)
_BF16_ATTENTION = contextvars.ContextVar("faquant_b200_bf16_attention", default=False)


class _HiF4QDQ:
    """A HiF4 ``input_qdq`` callable that the module can fuse with its rotation."""

    def __init__(self, levels: str, rotation: tuple[torch.Tensor, torch.Tensor | None, int] | None = None):
        ops.levels_code(levels)
        self.levels = levels
        self.rotation = rotation

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        signs, perm, block = self.rotation if self.rotation is not None else (None, None, 0)
        return ops.hif4_quantize(x, levels=self.levels, signs=signs, permutation=perm, rot_block=block)[0]


def faquant_qdq(levels: str, *, signs: torch.Tensor | None = None, permutation: torch.Tensor | None = None,
                block: int | None = None) -> Callable[[torch.Tensor], torch.Tensor]:
    """HiF4 QDQ along the last axis (``wan22_hif4.py:35-36``); optional fused input rotation."""
    rotation = None if signs is None else (signs, permutation, int(block or 0))
    return _HiF4QDQ(levels, rotation)


class HiF4Linear(nn.Module):
    """HiF4 W4A4 Linear (``wan22_hif4.py:51-92``): HiF4-grid bf16 weight, per-call input QDQ, tcgen05 GEMM."""

    def __init__(self, linear: nn.Linear, *, weight_qdq: Callable[[torch.Tensor], torch.Tensor],
                 input_qdq: Callable[[torch.Tensor], torch.Tensor], device: torch.device | str,
                 chunk_elements: int = 1 << 26, weight: torch.Tensor | None = None) -> None:
        super().__init__()
        self.in_features, self.out_features = linear.in_features, linear.out_features
        source = linear.weight.detach()
        if weight is None:
            quantized = weight_qdq(source.to(device=device, dtype=torch.float32))
        elif weight.shape != source.shape:
            raise ValueError(f"HiF4 weight of shape {tuple(weight.shape)} for a Linear of {tuple(source.shape)}")
        else:
            quantized = weight.to(device=device, dtype=torch.float32)
        stored = quantized.to(source.dtype)
        if not torch.equal(stored.float(), quantized):
            raise RuntimeError(f"HiF4 weight is not exactly representable in {source.dtype}")
        self.weight = nn.Parameter(stored.to(source.device), requires_grad=False)
        self.bias = None if linear.bias is None else nn.Parameter(linear.bias.detach().clone(), requires_grad=False)
        self.input_qdq = input_qdq
        self.chunk_rows = max(1, chunk_elements // self.in_features)
        self.collector: Callable[[nn.Module, torch.Tensor, int], None] | None = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        rows = x.reshape(-1, self.in_features)
        w = self.weight if self.weight.dtype == torch.bfloat16 else self.weight.to(torch.bfloat16)
        if self.collector is None and isinstance(self.input_qdq, _HiF4QDQ):
            # one K1 launch over all rows: the chunking bounds fp32 temporaries in the
            # reference and has no effect on the values
            xq = self.input_qdq(rows)
            y = ops.gemm_bf16(xq if xq.dtype == torch.bfloat16 else xq.to(torch.bfloat16), w, self.bias)
            return self._out(y, x).reshape(*x.shape[:-1], self.out_features)
        out = None
        for start in range(0, rows.shape[0], self.chunk_rows):
            part = self.input_qdq(rows[start:start + self.chunk_rows])
            if self.collector is not None:
                self.collector(self, part, start)
            y = ops.gemm_bf16(part.to(torch.bfloat16), w, self.bias)
            if out is None:
                out = y.new_empty(rows.shape[0], y.shape[-1])
            out[start:start + part.shape[0]] = y
        return self._out(out, x).reshape(*x.shape[:-1], self.out_features)

    @staticmethod
    def _out(y: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        # F.linear under the bf16 autocast of WanT2V.generate returns bf16 (wan22_hif4.py:13-14)
        if torch.is_autocast_enabled("cuda") or x.dtype == y.dtype:
            return y
        return y.to(x.dtype)


@torch.no_grad()
def quantize_dit_blocks(model: nn.Module, *, weight_qdq: Callable, input_qdq: Callable,
                        device: torch.device | str = "cuda", weights: Mapping[str, torch.Tensor] | None = None) -> int:
    """Replace the block Linears of one WanModel (``wan22_hif4.py:121-148``)."""
    count = 0
    for index, block in enumerate(model.blocks):
        for path in BLOCK_LINEARS:
            parent_name, _, child = path.rpartition(".")
            parent = block.get_submodule(parent_name)
            linear = getattr(parent, child)
            if type(linear) is not nn.Linear:
                raise TypeError(f"{path} is {type(linear).__name__}, not nn.Linear")
            given = None if weights is None else weights[f"blocks.{index}.{path}"]
            setattr(parent, child, HiF4Linear(linear, weight_qdq=weight_qdq, input_qdq=input_qdq, device=device,
                                              weight=given))
            count += 1
    left = [n for n, m in model.named_modules() if n.startswith("blocks.") and type(m) is nn.Linear]
    if left:
        raise RuntimeError(f"block Linears left unquantized: {left[:8]}")
    return count


def hif4_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, softmax_scale: float | None = None,
                   quantize_p: bool = True, quantized_normalizer: bool = False, block_m: int = 128,
                   num_warps: int = 8, num_stages: int = 1, p_levels: str = "123") -> torch.Tensor:
    """Non-causal attention of ``[L, H, D]`` bf16 tensors (Q/K/V already quantized); bf16 out.

    Same arguments as ``wan22_attention.hif4_attention`` (:165-183); ``block_m``,
    ``num_warps`` and ``num_stages`` were Triton launch knobs and are accepted and ignored.
    The P quantizer is three-level, as the reference's in-kernel ``_hif4_qdq_128``.
    """
    lq, heads, dim = q.shape
    if dim != 128 or k.shape != v.shape or tuple(k.shape[1:]) != (heads, dim):
        raise ValueError("hif4_attention expects [L, H, 128] q and matching k/v")
    out = ops.hif4_attention(q.unsqueeze(0).transpose(1, 2), k.unsqueeze(0).transpose(1, 2),
                             v.unsqueeze(0).transpose(1, 2), scale=softmax_scale, causal=False,
                             p_levels=p_levels if quantize_p else None, quantized_normalizer=quantized_normalizer)
    return out[0]


def rotate_heads(x: torch.Tensor, chunk_rows: int = 1 << 16) -> torch.Tensor:
    """Normalized Hadamard over head_dim in fp32, one bf16 rounding (``wan22_attention.py:186-192``)."""
    shape = x.shape
    flat = x.reshape(1, 1, -1, shape[-1])
    out, _, _ = ops.qk_prep(flat, levels=None, rotate=True)
    return out.reshape(shape)


def make_flash_attention(input_qdq: Callable[[torch.Tensor], torch.Tensor], *, quantized_normalizer: bool = False,
                         qk_rotation: bool = False, fallback: Callable | None = None) -> Callable:
    """Drop-in for ``wan.modules.attention.flash_attention`` with HiF4 Q/K/P/V (``:195-228``)."""

    def flash_attention(q, k, v, q_lens=None, k_lens=None, dropout_p=0., softmax_scale=None, q_scale=None,
                        causal=False, window_size=(-1, -1), deterministic=False, dtype=torch.bfloat16, version=None):
        if fallback is not None and _BF16_ATTENTION.get():
            return fallback(q, k, v, q_lens=q_lens, k_lens=k_lens, dropout_p=dropout_p, softmax_scale=softmax_scale,
                            q_scale=q_scale, causal=causal, window_size=window_size, deterministic=deterministic,
                            dtype=dtype, version=version)
        if dropout_p != 0 or q_scale is not None or causal or tuple(window_size) != (-1, -1):
            raise NotImplementedError("HiF4 flash_attention supports the Wan self/cross-attention call only")
        lq, lk, out_dtype = q.size(1), k.size(1), q.dtype
        for lens, full in ((q_lens, lq), (k_lens, lk)):
            if lens is not None and any(int(n) != full for n in lens.tolist()):
                raise NotImplementedError("variable sequence lengths are not supported")
        # [B, L, H, D] -> [B, H, L, D] views; K4 fuses the rotation, the bf16 cast and the QDQ
        qh, kh, vh = (t.transpose(1, 2) for t in (q, k, v))
        if isinstance(input_qdq, _HiF4QDQ) and input_qdq.rotation is None:
            lv = input_qdq.levels
            qd = ops.qk_prep(qh, levels=lv, rotate=qk_rotation)[0]
            kd = ops.qk_prep(kh, levels=lv, rotate=qk_rotation)[0]
            vd = ops.qk_prep(vh, levels=lv, rotate=False)[0]
        else:
            if qk_rotation:
                qh = ops.qk_prep(qh, levels=None, rotate=True)[0]
                kh = ops.qk_prep(kh, levels=None, rotate=True)[0]
            qd, kd, vd = (input_qdq(t.to(dtype)).to(torch.bfloat16) for t in (qh, kh, vh))
        out = ops.hif4_attention(qd, kd, vd, scale=softmax_scale, causal=False, p_levels="123",
                                 quantized_normalizer=quantized_normalizer)
        return out.type(out_dtype)

    return flash_attention


def patch_attention_modules(model_module, collector: Callable | None = None) -> None:
    """Per-module Smooth-QK / bf16 fallback for ``wan.modules.model`` (``wan22_attention.py:231-272``)."""
    rope_apply = model_module.rope_apply

    def attend(module, *args, **kwargs):
        token = _BF16_ATTENTION.set(bool(getattr(module, "faquant_attention_bf16", False)))
        try:
            return model_module.flash_attention(*args, **kwargs)
        finally:
            _BF16_ATTENTION.reset(token)

    def self_forward(self, x, seq_lens, grid_sizes, freqs):
        b, s, n, d = *x.shape[:2], self.num_heads, self.head_dim
        q = self.norm_q(self.q(x)).view(b, s, n, d)
        k = self.norm_k(self.k(x)).view(b, s, n, d)
        v = self.v(x).view(b, s, n, d)
        q, k = rope_apply(q, grid_sizes, freqs), rope_apply(k, grid_sizes, freqs)
        if collector is not None:
            collector(self, q, k)
        scale = getattr(self, "faquant_qk_smooth_scale", None)
        if scale is not None:
            q, k = q * scale, k / scale
        x = attend(self, q=q, k=k, v=v, k_lens=seq_lens, window_size=self.window_size)
        return self.o(x.flatten(2))

    def cross_forward(self, x, context, context_lens):
        b, n, d = x.size(0), self.num_heads, self.head_dim
        q = self.norm_q(self.q(x)).view(b, -1, n, d)
        k = self.norm_k(self.k(context)).view(b, -1, n, d)
        v = self.v(context).view(b, -1, n, d)
        x = attend(self, q, k, v, k_lens=context_lens)
        return self.o(x.flatten(2))

    model_module.WanSelfAttention.forward = self_forward
    model_module.WanCrossAttention.forward = cross_forward
