"""HiF4 W4A4 Linear: the drop-in for ``faquant.quantization`` on B200.

Mirrors ``src/faquant/quantization.py``: ``fake_quantize`` (:30-94),
``FakeQuantLinear`` (:97-277) with the same constructor arguments, buffers and
``state_dict`` keys, ``replace_linear_with_fake_quant`` (:300-375) and
``quantize_qwen3_linears`` (:378-408). The forward pass is two launches of the
C-ABI library: K1 (input scale, HiSQ signs/permutation/block Hadamard, HiF4
quantization, bit-exact with the reference) and K3 (tcgen05 GEMM on the
exactly-dequantized bf16 operands). With packed weights (``packed_weights=True``, or
``FAQ_PACKED_WEIGHTS=1`` in the environment for modules built through the reference's
installers) the module holds only the 4.5-bit packed weight: up to
``PACKED_SMALL_ROWS`` input rows (decode) the small-row kernel streams it packed into
register-fragment MMAs (``faq_w4a4_gemm_qdq_a``); from ``PACKED_EXPAND_MIN_ROWS`` rows
(by default every larger call) the weight is expanded to bf16 in a transient buffer at HBM
speed (``faq_hif4_dequantize``) and K3 runs on it, with the output bits of the bf16 path;
in between K1 writes the activation's packed codes and the GEMM expands both operands in
shared memory (``faq_w4a4_gemm``, the same bits too). A quarter of the weight bytes held.
Only ``quant_format="hif4"`` is implemented;
every other format, and the QAD-only clamp/companding knobs, raise
``NotImplementedError`` -- there is no CPU fallback.
"""

from __future__ import annotations

import torch
from torch import nn

import os

from . import ops

HIF4_BLOCK_SIZE = 64
# Input rows from which a packed module expands its weight to bf16 and runs the bf16 GEMM
# instead of the packed GEMM (faq_w4a4_gemm). The expansion reads 0.5625 and writes 2
# bytes per weight value, then K3 runs near the bf16 tensor peak, about twice the packed
# GEMM's rate at prefill sizes; at small row counts the packed GEMM's 256 x 256 tiles
# leave most SMs idle. Measured through the module on the config-2 projection shapes at
# 64 .. 2048 rows, expansion was never slower (down_proj at 64 rows: 124 us against 196),
# so every call expands; raise it to route small calls to the packed GEMM.
PACKED_EXPAND_MIN_ROWS = 0
# Up to this many input rows a packed module runs the small-row kernel (faq_w4a4_gemm_qdq_a
# with m <= 16): the weight is read in its 4.5-bit form and expanded in registers, so a
# decode step reads 0.5625 bytes per weight value instead of 2 (bf16 weights) or 4.5
# (expansion to bf16 and back). Its sums run in another order than the bf16 GEMM's: the
# same values up to fp32 rounding of the accumulation, not bit for bit.
PACKED_SMALL_ROWS = 16


def _packed_weights_default() -> bool:
    return os.environ.get("FAQ_PACKED_WEIGHTS", "0") == "1"


def _is_pow2(n: int) -> bool:
    return n > 0 and n & (n - 1) == 0


def fake_quantize(
    x: torch.Tensor,
    *,
    quant_format: str = "int",
    bits: int = 4,
    group_size: int = -1,
    symmetric: bool = True,
    clip_ratio: float = 1.0,
    hif4_levels: str | None = None,
) -> torch.Tensor:
    """HiF4 quantize-dequantize on the device (``quantization.py:30-57`` argument rules)."""
    if quant_format != "hif4":
        raise NotImplementedError(f"faquant_b200 implements quant_format='hif4' only, got {quant_format!r}")
    if bits != 4:
        raise ValueError("HiF4 requires bits=4")
    if group_size not in (-1, HIF4_BLOCK_SIZE):
        raise ValueError("HiF4 requires group_size=64 (or -1 for direct use)")
    if not symmetric:
        raise ValueError("HiF4 does not support asymmetric quantization")
    if clip_ratio != 1.0:
        raise ValueError("HiF4 direct-cast does not support clipping")
    qdq, _, _ = ops.hif4_quantize(x, levels=hif4_levels or ops.default_levels("act"))
    return qdq


def _quantize_weight_on_device(weight: torch.Tensor, levels: str) -> torch.Tensor:
    """RTN HiF4 of a weight (``quantization.py:174-184``), computed on a CUDA device."""
    source = weight.detach()
    device = source.device if source.is_cuda else torch.device("cuda", torch.cuda.current_device())
    qdq, _, _ = ops.hif4_quantize(source.to(device), levels=levels)
    return qdq.to(device=weight.device, dtype=weight.dtype)


class FakeQuantLinear(nn.Module):
    """Linear layer with dynamic HiF4 input and HiF4-grid weights, on tcgen05."""

    faquant_quantizes_input = True

    def __init__(
        self,
        linear: nn.Linear,
        *,
        quant_format: str = "int",
        bits: int,
        weight_group_size: int,
        activation_group_size: int,
        symmetric: bool,
        clip_ratio: float,
        quantize_weight: bool = True,
        online_hadamard: bool = False,
        online_hadamard_block_size: int | None = None,
        input_scale: torch.Tensor | None = None,
        input_rotation_signs: torch.Tensor | None = None,
        input_rotation_permutation: torch.Tensor | None = None,
        input_rotation_block_size: int | None = None,
        weight_override: torch.Tensor | None = None,
        activation_min: float | None = None,
        activation_max: float | None = None,
        activation_compand_log_scale: torch.Tensor | None = None,
        packed_weights: bool | None = None,
    ) -> None:
        super().__init__()
        if quant_format != "hif4":
            raise NotImplementedError(f"faquant_b200 implements quant_format='hif4' only, got {quant_format!r}")
        if bits != 4 or weight_group_size not in (-1, 64) or activation_group_size not in (-1, 64):
            raise ValueError("HiF4 requires bits=4 and group_size=64")
        if not symmetric or clip_ratio != 1.0:
            raise ValueError("HiF4 is symmetric and does not support clipping")
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.quant_format = quant_format
        self.bits = bits
        self.activation_group_size = activation_group_size
        self.symmetric = symmetric
        self.clip_ratio = clip_ratio
        self.online_hadamard = online_hadamard
        self.online_hadamard_block_size = online_hadamard_block_size
        self.register_buffer("input_scale", None if input_scale is None else input_scale.detach().float().clone())
        self.register_buffer(
            "input_rotation_signs",
            None if input_rotation_signs is None else input_rotation_signs.detach().to(torch.int8).clone(),
        )
        self.register_buffer(
            "input_rotation_permutation",
            None if input_rotation_permutation is None else input_rotation_permutation.detach().long().clone(),
        )
        self.input_rotation_block_size = input_rotation_block_size
        self.register_buffer(
            "activation_min", None if activation_min is None else torch.as_tensor(activation_min).detach().float().clone()
        )
        self.register_buffer(
            "activation_max", None if activation_max is None else torch.as_tensor(activation_max).detach().float().clone()
        )
        self.register_buffer(
            "activation_compand_log_scale",
            None if activation_compand_log_scale is None else activation_compand_log_scale.detach().float().clone(),
        )
        weight = linear.weight.detach() if weight_override is None else weight_override.detach()
        self._gemm_weight: torch.Tensor | None = None
        # packed weight (non-persistent: the state_dict keeps the reference's bf16 `weight`)
        self.register_buffer("weight_codes", None, persistent=False)
        self.register_buffer("weight_meta", None, persistent=False)
        packed = _packed_weights_default() if packed_weights is None else packed_weights
        if packed and self._pack(weight, source=quantize_weight):
            # only the packed form is kept; `weight` reads back as None
            self.register_parameter("weight", None)
        else:
            if quantize_weight:
                weight = _quantize_weight_on_device(weight, ops.default_levels("weight"))
            weight = weight.to(dtype=linear.weight.dtype)
            with torch.inference_mode(False):
                weight = weight.detach().clone()
            self.weight = nn.Parameter(weight, requires_grad=False)
        if linear.bias is None:
            self.register_parameter("bias", None)
        else:
            with torch.inference_mode(False):
                self.bias = nn.Parameter(linear.bias.detach().clone(), requires_grad=False)

    # ---------------------------------------------------------------- packed weights
    def _pack(self, weight: torch.Tensor, *, source: bool) -> bool:
        """Store ``weight`` in the packed format (K2). ``source`` (RTN): ``weight`` is the
        unquantized weight and the packed form is its RTN quantization, bit-identical to
        the reference's (quantization.py:169-184). Otherwise ``weight`` is already on the
        HiF4 grid without its metadata: it is refitted and kept packed only when the
        packed form reproduces every value (RTN is not idempotent in general). False when
        the weight stays in bf16 (k not a multiple of 256, or values not reproduced)."""
        n, k = weight.shape
        if k % 256:
            return False
        device = weight.device if weight.is_cuda else torch.device("cuda", torch.cuda.current_device())
        codes, meta, changed = ops.hif4_pack_weight(weight.detach().to(device), levels=ops.default_levels("weight"))
        if not source and changed:
            return False
        self.weight_codes, self.weight_meta = codes, meta
        self._gemm_weight = None
        return True

    @property
    def packed(self) -> bool:
        return self.weight_codes is not None

    def use_packed(self, codes: torch.Tensor, meta: torch.Tensor) -> None:
        """Switch to packed storage with an exact packed form produced elsewhere (for
        example K2 with a checkpoint's GPTQ metadata); the bf16 weight is released."""
        if codes.shape != (self.out_features, self.in_features // 2) or meta.shape != (
                self.out_features, self.in_features // 64):
            raise ValueError("packed weight shape does not match the layer")
        if self.in_features % 256:
            raise NotImplementedError("the packed GEMM needs in_features % 256 == 0")
        self.weight_codes, self.weight_meta = codes, meta
        self._gemm_weight = None
        self.register_parameter("weight", None)

    def hif4_metadata(self) -> dict[str, torch.Tensor]:
        """The packed weight's compact HiF4 metadata in the reference's checkpoint leaves
        (qad_checkpoint.py:43-48, the fields of CompactHiF4Parameters, hif4.py:68-79):
        scale and reciprocal fp32 [n, k/64], lv2 int8 [n, k/64, 8], lv3 int8 [n, k/64, 16]."""
        meta = self.weight_meta.to(torch.int64) & 0xFFFFFFFF
        code = meta & 0xFF
        scale = (1.0 + (code & 3).double() / 4.0) * torch.exp2(((code >> 2) - 48).double())
        scale = scale.float()
        bits2 = torch.arange(8, device=meta.device)
        bits3 = torch.arange(16, device=meta.device)
        return {
            "weight_hif4_scale": scale,
            "weight_hif4_reciprocal": (1.0 / scale).to(torch.bfloat16).float(),
            "weight_hif4_scale_lv2_exponent": ((meta[..., None] >> (8 + bits2)) & 1).to(torch.int8),
            "weight_hif4_scale_lv3_exponent": ((meta[..., None] >> (16 + bits3)) & 1).to(torch.int8),
        }

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        super()._save_to_state_dict(destination, prefix, keep_vars)
        if self.packed:
            # the reference's layout of a HiF4 checkpoint (qad_checkpoint.py:43-48): the
            # weight on the HiF4 grid in bf16 plus its compact metadata, from which the
            # packed form is rebuilt exactly on load
            destination[prefix + "weight"] = self.dequantized_weight()
            for leaf, value in self.hif4_metadata().items():
                destination[prefix + leaf] = value

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        key = prefix + "weight"
        leaves = ("weight_hif4_scale", "weight_hif4_reciprocal", "weight_hif4_scale_lv2_exponent",
                  "weight_hif4_scale_lv3_exponent")
        if self.packed and key in state_dict:
            w = state_dict[key]
            fields = [state_dict.get(prefix + leaf) for leaf in leaves]
            if all(f is not None for f in fields):
                n, k = w.shape
                dev = self.weight_codes.device
                codes, meta, bad = ops.hif4_pack_weight(
                    w.to(dev), levels=ops.default_levels("weight"), scale=fields[0].reshape(n, k // 64).to(dev),
                    lv2=fields[2].reshape(n, k // 64, 8), lv3=fields[3].reshape(n, k // 64, 16))
                if bad:
                    error_msgs.append(f"{key}: {bad} values are not on the grid of their HiF4 metadata")
                else:
                    self.weight_codes, self.weight_meta = codes, meta
            elif not self._pack(w, source=False):
                error_msgs.append(f"{key}: no HiF4 metadata, and a refit does not reproduce the weight; load it "
                                  "into a module without packed weights")
            state_dict = {k: v for k, v in state_dict.items() if k != key and k[len(prefix):] not in leaves}
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)

    def _rotation(self) -> tuple[torch.Tensor | None, torch.Tensor | None, int]:
        if self.activation_min is not None or self.activation_max is not None:
            raise NotImplementedError("activation clamping (QAD) is not implemented by faquant_b200")
        if self.activation_compand_log_scale is not None:
            raise NotImplementedError("activation companding (QAD) is not implemented by faquant_b200")
        if self.input_rotation_signs is not None:
            if self.online_hadamard:
                raise NotImplementedError("an input rotation followed by an online Hadamard is not implemented")
            block = self.input_rotation_block_size
            return self.input_rotation_signs, self.input_rotation_permutation, 0 if block is None else int(block)
        if self.online_hadamard:
            block = self.online_hadamard_block_size or self.in_features
            if not _is_pow2(block):
                raise NotImplementedError("the 12*2^n generalized Hadamard is not implemented; use a power of two")
            device = self.weight_codes.device if self.packed else self.weight.device
            ones = torch.ones(self.in_features, dtype=torch.int8, device=device)
            return ones, None, int(block)
        return None, None, 0

    def _operand_weight(self) -> torch.Tensor:
        if self.packed:
            return ops.hif4_dequantize(self.weight_codes, self.weight_meta, self.in_features)
        w = self.weight
        if w.dtype == torch.bfloat16:
            return w
        cached = self._gemm_weight
        if cached is None or cached.device != w.device or cached.shape != w.shape:
            # HiF4 values are exact in bf16 (<= 6 significant bits)
            cached = w.detach().to(torch.bfloat16)
            self._gemm_weight = cached
        return cached

    def dequantized_weight(self) -> torch.Tensor:
        """The weight on the HiF4 grid as the GEMM sees it, in bf16 (exact)."""
        return self._operand_weight()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("faquant_b200.FakeQuantLinear runs on CUDA tensors only")
        signs, perm, block = self._rotation()
        # the reference moves its rotation buffers to the input's device per call (quantization.py:208-209)
        if signs is not None and signs.device != x.device:
            signs = signs.to(x.device)
        if perm is not None and perm.device != x.device:
            perm = perm.to(x.device)
        scale = self.input_scale
        if scale is not None and scale.device != x.device:
            scale = scale.to(x.device)
        shape = x.shape
        rows = x.numel() // shape[-1]
        if self.packed and x.dtype == torch.bfloat16 and 0 < rows <= PACKED_SMALL_ROWS:
            # a few rows (decode): the weight streams packed into the small-row kernel
            qdq, _, _ = ops.hif4_quantize(x.reshape(-1, shape[-1]), levels=ops.default_levels("act"),
                                          input_scale=scale, signs=signs, permutation=perm, rot_block=block)
            y = ops.w4a4_gemm(qdq, self.weight_codes, self.weight_meta, self.bias)
            return y.reshape(*shape[:-1], self.out_features)
        if self.packed and x.dtype == torch.bfloat16 and rows < PACKED_EXPAND_MIN_ROWS:
            _, codes, meta = ops.hif4_quantize(x.reshape(-1, shape[-1]), levels=ops.default_levels("act"),
                                               input_scale=scale, signs=signs, permutation=perm, rot_block=block,
                                               want_qdq=False, want_codes=True)
            y = ops.w4a4_gemm((codes, meta), self.weight_codes, self.weight_meta, self.bias)
            return y.reshape(*shape[:-1], self.out_features)
        qdq, _, _ = ops.hif4_quantize(
            x.reshape(-1, shape[-1]),
            levels=ops.default_levels("act"),
            input_scale=scale,
            signs=signs,
            permutation=perm,
            rot_block=block,
        )
        a = qdq if qdq.dtype == torch.bfloat16 else qdq.to(torch.bfloat16)  # exact
        y = ops.gemm_bf16(a, self._operand_weight(), self.bias)
        y = y.reshape(*shape[:-1], self.out_features)
        return y if y.dtype == x.dtype else y.to(x.dtype)


def replace_linear_with_fake_quant(parent: nn.Module, name: str, config: object, *, weights_prequantized: bool) -> None:
    """Swap ``parent.<name>`` for a ``FakeQuantLinear`` reading its ``faquant_*`` attributes."""
    linear = getattr(parent, name)
    if isinstance(linear, FakeQuantLinear):
        return
    online_hadamard = bool(getattr(linear, "faquant_online_hadamard", False))
    online_hadamard_block_size = getattr(linear, "faquant_online_hadamard_block_size", None)
    if online_hadamard:
        linear = linear.module
    if not isinstance(linear, nn.Linear):
        raise TypeError(f"{parent.__class__.__name__}.{name} is not nn.Linear")
    weight_override = getattr(linear, "faquant_weight_override", None)
    replacement = FakeQuantLinear(
        linear,
        quant_format=config.quant_format,
        bits=config.bits,
        weight_group_size=config.weight_group_size,
        activation_group_size=config.activation_group_size,
        symmetric=config.symmetric,
        clip_ratio=config.clip_ratio,
        quantize_weight=not weights_prequantized,
        online_hadamard=online_hadamard,
        online_hadamard_block_size=online_hadamard_block_size,
        input_scale=getattr(linear, "faquant_input_scale", None),
        input_rotation_signs=getattr(linear, "faquant_input_rotation_signs", None),
        input_rotation_permutation=getattr(linear, "faquant_input_rotation_permutation", None),
        input_rotation_block_size=getattr(linear, "faquant_input_rotation_block_size", None),
        weight_override=None if weights_prequantized else weight_override,
        activation_min=getattr(linear, "faquant_activation_min", None),
        activation_max=getattr(linear, "faquant_activation_max", None),
        activation_compand_log_scale=getattr(linear, "faquant_activation_compand_log_scale", None),
    )
    for attr in ("faquant_hif4_qat_parameters", "faquant_hif4_qat_master"):
        value = getattr(linear, attr, None)
        if value is not None:
            setattr(replacement, attr, value)
    setattr(parent, name, replacement)


@torch.inference_mode()
def quantize_qwen3_linears(model: nn.Module, config: object, *, weights_prequantized: bool = False,
                           exempt: frozenset[tuple[int, str]] = frozenset()) -> None:
    """Install HiF4 W4A4 on the Qwen3 projections (``quantization.py:378-408``)."""
    target = config.quant_target
    if target == "none":
        return
    for index, layer in enumerate(model.model.layers):
        if target in ("attention", "all"):
            for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
                if (index, name) not in exempt:
                    replace_linear_with_fake_quant(layer.self_attn, name, config, weights_prequantized=weights_prequantized)
        if target in ("ffn", "all"):
            for name in ("gate_proj", "up_proj", "down_proj"):
                if (index, name) not in exempt:
                    replace_linear_with_fake_quant(layer.mlp, name, config, weights_prequantized=weights_prequantized)
