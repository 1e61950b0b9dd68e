"""Step-0 QAD checkpoint ingestion into HiF4 inference linears, verified on the GPU.

Reference: ``qad_checkpoint.load_qad_inference_checkpoint``
(src/faquant/qad_checkpoint.py:272-385) with the metadata leaves of :43-48. A step-0
checkpoint holds, per quantized projection, the bf16 weight (already on the HiF4 grid)
and its compact metadata -- ``weight_hif4_scale`` and ``weight_hif4_reciprocal`` (fp32,
one per 64-value block), ``weight_hif4_scale_lv2_exponent`` (int8, per 8 values) and
``weight_hif4_scale_lv3_exponent`` (int8, per 4 values), the fields of
``CompactHiF4Parameters`` (hif4.py:68-79) -- in safetensors shards listed by
``model.safetensors.index.json``, with ``qad_init.json`` recording the HiF4 level variants.

The reference re-quantizes every weight with its metadata and reports the largest change
(``requantized_max_abs``, zero for a valid checkpoint). Here the same check runs in K2
(``faq_hif4_pack_weight`` with the recorded scale and exponents), which also produces
the 4.5-bit packed form; the largest change is measured on the packed form decoded back
(``faq_hif4_dequantize``), and the number of values the packed form does not reproduce
is counted (``requantized_mismatches``).

Unlike the reference, the model is not built here: ``model`` must already hold this
package's ``FakeQuantLinear`` modules (for example from ``quantize_qwen3_linears``) under
the checkpoint's module names.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import torch
from torch import nn

from . import ops
from .quantization import FakeQuantLinear

HIF4_METADATA_LEAVES = {
    "weight_hif4_scale": "scale",
    "weight_hif4_reciprocal": "reciprocal",
    "weight_hif4_scale_lv2_exponent": "scale_lv2_exponent",
    "weight_hif4_scale_lv3_exponent": "scale_lv3_exponent",
}
# artifacts of a trained (not step-0) QAD run, whose weights need the QAT skeleton
TRAINING_ARTIFACTS = ("training_receipt.json", "activation_companding.json", "activation_clipping.json")


@dataclass(frozen=True)
class QADInferenceLoadStats:
    linears: int
    requantized_max_abs: float
    missing_keys: tuple[str, ...]
    unexpected_keys: tuple[str, ...]
    requantized_mismatches: int = 0


@dataclass(frozen=True)
class PackedHiF4Weight:
    """A weight in the 4.5-bit layout of ``faq_hif4_pack_weight``."""

    codes: torch.Tensor  # uint8 [n, k / 2]
    meta: torch.Tensor   # int32 [n, k / 64]
    in_features: int


def check_receipt(checkpoint: str | Path, *, weight_levels: str = "123", act_levels: str | None = None) -> None:
    """The checks of qad_checkpoint.py:295-313: the recorded level variants must be the
    ones this process quantizes with, and no training artifact may be present."""
    checkpoint = Path(checkpoint)
    receipt = checkpoint / "qad_init.json"
    recorded = json.loads(receipt.read_text(encoding="utf-8")) if receipt.exists() else {}
    w_rec = recorded.get("hif4_scale_levels", "123")
    a_rec = recorded.get("hif4_act_scale_levels", w_rec)
    act_levels = weight_levels if act_levels is None else act_levels
    if (w_rec, a_rec) != (weight_levels, act_levels):
        raise ValueError(f"{checkpoint} was built with HiF4 scale levels {w_rec} (weights) / {a_rec} "
                         f"(activations), but this process runs {weight_levels} / {act_levels}")
    for artifact in TRAINING_ARTIFACTS:
        if (checkpoint / artifact).exists():
            raise ValueError(f"{checkpoint} has {artifact}; only step-0 initializations load without the QAT skeleton")


def iter_checkpoint_shards(checkpoint: str | Path, metadata: dict[str, dict[str, torch.Tensor]]):
    """Yield the model tensors of one shard at a time (the shards listed by the index, in
    order); the HiF4 metadata leaves are split off into ``metadata[module_name][field]``,
    which the caller keeps across shards. Only one shard's tensors are alive at a time, as
    in the reference's loader (qad_checkpoint.py:340-356), so the host peak is one shard
    plus the small metadata, not the whole model."""
    from safetensors import safe_open

    checkpoint = Path(checkpoint)
    index = json.loads((checkpoint / "model.safetensors.index.json").read_text(encoding="utf-8"))
    for shard in sorted(set(index["weight_map"].values())):
        state: dict[str, torch.Tensor] = {}
        with safe_open(str(checkpoint / shard), framework="pt", device="cpu") as tensors:
            for key in tensors.keys():
                module_name, _, leaf = key.rpartition(".")
                if leaf in HIF4_METADATA_LEAVES:
                    metadata.setdefault(module_name, {})[HIF4_METADATA_LEAVES[leaf]] = tensors.get_tensor(key)
                else:
                    state[key] = tensors.get_tensor(key)
        yield state
        del state


def read_checkpoint(checkpoint: str | Path) -> tuple[dict[str, torch.Tensor], dict[str, dict[str, torch.Tensor]]]:
    """``(state, metadata)``: every tensor of the shards listed by the index, with the HiF4
    metadata leaves split off into ``metadata[module_name][field]`` (all shards at once;
    the loader below goes shard by shard)."""
    state: dict[str, torch.Tensor] = {}
    metadata: dict[str, dict[str, torch.Tensor]] = {}
    for shard_state in iter_checkpoint_shards(checkpoint, metadata):
        state.update(shard_state)
    return state, metadata


@torch.no_grad()
def load_qad_inference_checkpoint(
    model: nn.Module,
    checkpoint: str | Path,
    *,
    levels: str = "123",
    packed_out: dict[str, PackedHiF4Weight] | None = None,
    pack: bool = False,
) -> QADInferenceLoadStats:
    """Load a step-0 QAD checkpoint into ``model``'s ``FakeQuantLinear`` modules and verify
    every weight against its metadata on the GPU (see the module docstring). With
    ``packed_out`` the packed weights are stored there by module name; with ``pack`` every
    exactly packed weight replaces the module's bf16 weight (``FakeQuantLinear.use_packed``),
    so the model keeps 4.5 bits per weight in HBM."""
    check_receipt(checkpoint, weight_levels=levels)
    expected = set(model.state_dict())
    metadata: dict[str, dict[str, torch.Tensor]] = {}
    loaded: set[str] = set()
    unexpected: set[str] = set()
    # one shard at a time: copy it into the model, then drop it before opening the next
    for state in iter_checkpoint_shards(checkpoint, metadata):
        result = model.load_state_dict(state, strict=False)
        loaded.update(state)
        unexpected.update(result.unexpected_keys)
        del state, result

    max_abs, mismatches, linears = 0.0, 0, 0
    for name, module in model.named_modules():
        if not isinstance(module, FakeQuantLinear):
            continue
        fields = metadata.pop(name, None)
        if fields is None or len(fields) != len(HIF4_METADATA_LEAVES):
            raise RuntimeError(f"{checkpoint} has no complete HiF4 metadata for {name}")
        module._gemm_weight = None  # the weight was replaced: drop any cached GEMM operand
        weight = module.weight
        if not weight.is_cuda:
            raise RuntimeError("load the checkpoint into a model on the GPU (the check runs in K2)")
        n, k = weight.shape
        groups = k // 64
        device = weight.device
        scale = fields["scale"].to(device=device, dtype=torch.float32).reshape(n, groups)
        reciprocal = fields["reciprocal"].to(device=device, dtype=torch.float32).reshape(n, groups)
        # the reciprocal is bf16(1 / scale) by construction (hif4.py:114); K2 derives it
        if not torch.equal(reciprocal, (1.0 / scale).to(torch.bfloat16).float()):
            raise RuntimeError(f"{name}: weight_hif4_reciprocal is not bf16(1 / weight_hif4_scale)")
        lv2 = fields["scale_lv2_exponent"].reshape(n, groups, 8)
        lv3 = fields["scale_lv3_exponent"].reshape(n, groups, 16)
        codes, meta, bad = ops.hif4_pack_weight(weight, levels=levels, scale=scale, lv2=lv2, lv3=lv3)
        decoded = ops.hif4_dequantize(codes, meta, k, dtype=torch.float32)
        max_abs = max(max_abs, float((decoded - weight.float()).abs().max()))
        mismatches += bad
        linears += 1
        if packed_out is not None:
            packed_out[name] = PackedHiF4Weight(codes=codes, meta=meta, in_features=k)
        if pack and bad == 0 and k % 256 == 0:
            module.use_packed(codes, meta)
    if metadata:
        raise RuntimeError(f"HiF4 metadata for modules that are not quantized: {sorted(metadata)[:4]}")
    return QADInferenceLoadStats(linears=linears, requantized_max_abs=max_abs,
                                 missing_keys=tuple(sorted(expected - loaded)),
                                 unexpected_keys=tuple(sorted(unexpected)), requantized_mismatches=mismatches)
