"""GPU test of the Hugging Face path end to end on a small random Qwen3: HiF4 W4A4 on every
projection (quantize_qwen3_linears, FakeQuantLinear), the patched Qwen3 attention forward
(qwen3.attention_forward: q/k norm, RoPE, the post-RoPE Hadamard) on the HiF4 attention
backend registered with transformers, the HF K/V cache, chunked prefill, and the hand-off
to a BF16 copy of the model for greedy decode (generate.prefill_quant_decode_bf16_generate,
after eval_longbench.py:505-576)."""

from __future__ import annotations

import types
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
PROMPT = 600  # three 256-query chunks, the last one ragged
NEW = 6


def _tiny_qwen3():
    from transformers import Qwen3Config, Qwen3ForCausalLM

    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, max_position_embeddings=4096,
                      tie_word_embeddings=False)
    torch.manual_seed(0)
    return Qwen3ForCausalLM(cfg).to(device=DEV, dtype=torch.bfloat16).eval()


def _adapter(model, kernel: str):
    """The patched Qwen3 attention on every layer: post-RoPE Hadamard over head_dim, then
    the HiF4 backend (kernel "simulated") or the model's own attention ("native")."""
    from faquant_b200.qwen3 import attention_forward

    for layer in model.model.layers:
        attn = layer.self_attn
        attn.faquant_attention_kernel = kernel
        attn.faquant_qk_rotation = True
        attn.forward = types.MethodType(attention_forward, attn)
    return model


def _hif4(model):
    from faquant_b200.attention import (B200_ATTENTION_IMPLEMENTATION, new_simulated_attention_stats,
                                        register_simulated_attention_backend)
    from faquant_b200.quantization import quantize_qwen3_linears

    register_simulated_attention_backend()
    model.set_attn_implementation(B200_ATTENTION_IMPLEMENTATION)
    quantize_qwen3_linears(model, SimpleNamespace(quant_target="all", quant_format="hif4", bits=4,
                                                  weight_group_size=64, activation_group_size=64, symmetric=True,
                                                  clip_ratio=1.0))
    for layer in model.model.layers:
        attn = layer.self_attn
        attn.faquant_attention_query_chunk_size = 256
        attn.faquant_attention_key_chunk_size = 128
        attn.faquant_qk_matmul_quant = True
        attn.faquant_pv_matmul_quant = True
        attn.faquant_pv_normalizer_mode = "quantized_same"
        attn.faquant_matmul_quant_kwargs = {"quant_format": "hif4", "bits": 4, "group_size": 64,
                                            "symmetric": True, "clip_ratio": 1.0}
        attn.faquant_simulated_attention_stats = new_simulated_attention_stats()
    return _adapter(model, "simulated")


@torch.inference_mode()
def test_quantized_prefill_then_bf16_decode_on_qwen3() -> None:
    """One-pass prefill of the HiF4 model plus greedy decode of the BF16 model on its cache
    give the tokens the workflow gives with 256-token prefill chunks."""
    from faquant_b200.generate import prefill_quant_decode_bf16_generate
    from faquant_b200.quantization import FakeQuantLinear

    # the BF16 decode model is built as the reference builds it (eval_longbench.py:427-470):
    # the same weights and the same Q/K transform (the shared cache holds transformed keys),
    # the model's own attention, no quantization
    quant, bf16, plain = _hif4(_tiny_qwen3()), _adapter(_tiny_qwen3(), "native"), _tiny_qwen3()
    assert all(isinstance(layer.mlp.down_proj, FakeQuantLinear) for layer in quant.model.layers)
    assert not any(isinstance(m, FakeQuantLinear) for m in bf16.modules())
    prompt = torch.randint(0, 512, (1, PROMPT), generator=torch.Generator().manual_seed(1)).to(DEV)
    # the Hadamard is orthonormal: with it on Q and K the BF16 model matches the plain one
    # up to the bf16 rounding of the rotated operands
    a = bf16(input_ids=prompt, logits_to_keep=8).logits.float()
    b = plain(input_ids=prompt, logits_to_keep=8).logits.float()
    assert float((a - b).norm() / b.norm()) <= 2e-2

    # the whole prompt in one pass: its last logits give the first token, and its cache
    # (HF keeps the bf16 K/V; the HiF4 operands are made inside the attention call)
    one = quant(input_ids=prompt, use_cache=True, return_dict=True, logits_to_keep=1)
    assert torch.isfinite(one.logits).all()
    first = int(one.logits[0, -1].argmax())
    cache, token, expect = one.past_key_values, torch.tensor([[first]], device=DEV), [first]
    for _ in range(NEW - 1):  # greedy BF16 decode on that cache
        step = bf16(input_ids=token, past_key_values=cache,
                    cache_position=torch.tensor([cache.get_seq_length()], device=DEV), use_cache=True,
                    return_dict=True)
        cache, token = step.past_key_values, step.logits[:, -1].argmax(-1, keepdim=True)
        expect.append(int(token))

    # the workflow: chunked prefill (256-token chunks are bit-identical to one pass), the
    # QDQ append caches released, then the BF16 model
    quant.__dict__["_faquant_bf16_decode_model"] = bf16
    quant.__dict__["_faquant_prefill_chunk_tokens"] = 256
    out = prefill_quant_decode_bf16_generate(quant, input_ids=prompt, max_length=PROMPT + NEW, eos_token_id=[])
    assert torch.equal(out[:, :PROMPT], prompt)
    assert out[0, PROMPT:].tolist() == expect
    for layer in quant.model.layers:
        assert layer.self_attn.faquant_k_matmul_qdq_cache is None
        assert layer.self_attn.faquant_v_matmul_qdq_cache is None
    stats = quant.model.layers[0].self_attn.faquant_simulated_attention_stats
    assert stats and max(stats.values()) > 0  # the HiF4 backend ran
