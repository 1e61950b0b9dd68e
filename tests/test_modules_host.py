"""Host-side logic of the module layer (no GPU): argument validation that must fail
before any device work, the simulator's geometry counters, and the level variants
read from the reference's environment variables."""

from __future__ import annotations

import json
from types import SimpleNamespace

import pytest
import torch

from conftest import load_golden
from inputs import ATTENTION_CASES


def _module(causal: bool, normalizer: str, qk: bool, pv: bool, key_chunk: int = 128) -> SimpleNamespace:
    from faquant_b200.attention import new_simulated_attention_stats

    return SimpleNamespace(
        is_causal=causal,
        training=False,
        faquant_attention_query_chunk_size=256,
        faquant_attention_key_chunk_size=key_chunk,
        faquant_qk_matmul_quant=qk,
        faquant_pv_matmul_quant=pv,
        faquant_pv_normalizer_mode=normalizer,
        faquant_matmul_quant_kwargs={"quant_format": "hif4", "bits": 4, "group_size": 64, "symmetric": True,
                                     "clip_ratio": 1.0},
        faquant_simulated_attention_stats=new_simulated_attention_stats(),
    )


@pytest.mark.parametrize("case", ATTENTION_CASES, ids=[c[0] for c in ATTENTION_CASES])
def test_attention_stats_match_reference(case) -> None:
    """The per-operand counters equal the ones the reference simulator recorded."""
    from faquant_b200.attention import _update_stats

    g = load_golden("attention")
    tag, b, h, kv, sq, sk, causal, normalizer, qk, pv, seed = case
    module = _module(causal, normalizer, qk, pv)
    _update_stats(module, b, h, kv, sq, sk, 128, 256, 128, causal, qk, pv)
    expected = json.loads(bytes(g[f"{tag}_stats"]).decode())
    assert module.faquant_simulated_attention_stats == expected


def test_attention_backend_rejects_unsupported_calls_before_device_work() -> None:
    from faquant_b200.attention import simulated_flash_attention_forward

    q = torch.zeros(1, 2, 4, 128)
    k = torch.zeros(1, 2, 4, 128)
    mod = _module(True, "quantized_same", True, True)
    with pytest.raises(NotImplementedError, match="softcap"):
        simulated_flash_attention_forward(mod, q, k, k, None, softcap=30.0)
    with pytest.raises(NotImplementedError, match="sliding"):
        simulated_flash_attention_forward(mod, q, k, k, None, sliding_window=8)
    with pytest.raises(ValueError, match="dropout"):
        simulated_flash_attention_forward(mod, q, k, k, None, dropout=0.1)
    with pytest.raises(NotImplementedError, match="key tiles of 128"):
        simulated_flash_attention_forward(_module(True, "quantized_same", True, True, key_chunk=64), q, k, k, None)
    int_mod = _module(True, "quantized_same", True, True)
    int_mod.faquant_matmul_quant_kwargs = {"bits": 4, "group_size": 4, "symmetric": True, "clip_ratio": 1.0}
    with pytest.raises(NotImplementedError, match="HiF4"):
        simulated_flash_attention_forward(int_mod, q, k, k, None)
    bad = _module(True, "bogus", True, True)
    with pytest.raises(ValueError, match="normalizer"):
        simulated_flash_attention_forward(bad, q, k, k, None)
    with pytest.raises(NotImplementedError, match="mask"):
        mask = torch.ones(1, 4, dtype=torch.bool)
        mask[0, 0] = False
        simulated_flash_attention_forward(mod, q, k, k, mask)


def test_fake_quant_linear_rejects_other_formats_without_a_gpu() -> None:
    from faquant_b200.quantization import FakeQuantLinear, fake_quantize

    lin = torch.nn.Linear(64, 8, bias=False)
    with pytest.raises(NotImplementedError, match="hif4"):
        FakeQuantLinear(lin, quant_format="int", bits=4, weight_group_size=64, activation_group_size=64,
                        symmetric=True, clip_ratio=1.0)
    with pytest.raises(ValueError, match="group"):
        FakeQuantLinear(lin, quant_format="hif4", bits=4, weight_group_size=128, activation_group_size=64,
                        symmetric=True, clip_ratio=1.0)
    with pytest.raises(NotImplementedError):
        fake_quantize(torch.zeros(2, 64), quant_format="mxfp8e4m3", bits=8, group_size=32)
    # prequantized weights need no device: the module is built on the host
    mod = FakeQuantLinear(lin, quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64,
                          symmetric=True, clip_ratio=1.0, quantize_weight=False,
                          input_rotation_signs=torch.ones(64, dtype=torch.int8),
                          input_rotation_permutation=torch.arange(64), input_rotation_block_size=64)
    assert set(mod.state_dict()) == {"weight", "input_rotation_signs", "input_rotation_permutation"}
    with pytest.raises(RuntimeError, match="CUDA"):
        mod(torch.zeros(2, 64))


def test_levels_follow_the_reference_environment(monkeypatch) -> None:
    from faquant_b200 import ops

    monkeypatch.setenv("FAQUANT_HIF4_SCALE_LEVELS", "12")
    monkeypatch.delenv("FAQUANT_HIF4_ACT_SCALE_LEVELS", raising=False)
    monkeypatch.setenv("FAQUANT_HIF4_ATTN_SCALE_LEVELS", "13")
    monkeypatch.setenv("FAQUANT_HIF4_ATTN_OPERAND_LEVELS", "p=123,v=123")
    assert ops.default_levels("weight") == "12"
    assert ops.default_levels("act") == "12"
    assert ops.default_levels("q") == "13" and ops.default_levels("k") == "13"
    assert ops.default_levels("p") == "123" and ops.default_levels("v") == "123"
    monkeypatch.setenv("FAQUANT_HIF4_SCALE_LEVELS", "99")
    with pytest.raises(ValueError):
        ops.default_levels("weight")
