"""Step-0 QAD checkpoint ingestion on the GPU (faquant_b200.checkpoint against
qad_checkpoint.load_qad_inference_checkpoint, qad_checkpoint.py:272-385): grid weights
with their metadata load into FakeQuantLinear modules with zero re-quantization change,
pack to the same values, and a checkpoint whose metadata does not describe its weights
is reported (the planted mistake is in the checkpoint written on the CPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from torch import nn

from checkpoint_fixture import LINEARS, write_checkpoint

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _model() -> nn.Module:
    from faquant_b200.quantization import FakeQuantLinear

    root = nn.Module()
    layer = nn.Module()
    for name, (n, k) in LINEARS.items():
        lin = nn.Linear(k, n, bias=False, device=DEV, dtype=torch.bfloat16)
        setattr(layer, name.rsplit(".", 1)[1],
                FakeQuantLinear(lin, quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64,
                                symmetric=True, clip_ratio=1.0, quantize_weight=False))
    layers = nn.ModuleDict({"0": layer})
    root.layers = layers
    root.norm = nn.Module()
    root.norm.weight = nn.Parameter(torch.zeros(512, device=DEV, dtype=torch.bfloat16), requires_grad=False)
    return root


def test_step0_checkpoint_loads_verified_and_packed(tmp_path) -> None:
    from faquant_b200 import ops
    from faquant_b200.checkpoint import load_qad_inference_checkpoint

    weights = write_checkpoint(tmp_path)
    model = _model()
    packed = {}
    stats = load_qad_inference_checkpoint(model, tmp_path, packed_out=packed)
    assert stats.linears == 2 and stats.requantized_max_abs == 0.0 and stats.requantized_mismatches == 0
    assert stats.missing_keys == () and stats.unexpected_keys == ()
    modules = dict(model.named_modules())
    for name, w in weights.items():
        got = modules[name].weight.float().cpu().numpy()
        assert np.array_equal(got, w)
        p = packed[name]
        assert np.array_equal(ops.hif4_dequantize(p.codes, p.meta, p.in_features, torch.float32).cpu().numpy(), w)
    assert torch.equal(model.norm.weight.float().cpu(), torch.ones(512))


def test_metadata_that_does_not_describe_the_weights_is_reported(tmp_path) -> None:
    from faquant_b200.checkpoint import load_qad_inference_checkpoint

    write_checkpoint(tmp_path, corrupt_lv2=True)
    stats = load_qad_inference_checkpoint(_model(), tmp_path)
    assert stats.requantized_mismatches > 0 and stats.requantized_max_abs > 0.0
