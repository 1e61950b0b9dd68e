"""Host tests of the quantized-prefill / BF16-decode generation loop
(faquant_b200.generate, after eval_longbench.py:495-576 and the reference's
tests/test_prefill_decode.py): chunked prompt feeding with cache positions, the first
token from the prefill logits, release of the K/V QDQ append caches, BF16 greedy decode at
the cache length, and the stops (EOS, max_length, a stopping criteria)."""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from faquant_b200.generate import prefill_quant_decode_bf16_generate

VOCAB = 6


class Cache:
    def __init__(self) -> None:
        self.length = 0

    def get_seq_length(self) -> int:
        return self.length


def _logits(token: int) -> torch.Tensor:
    out = torch.zeros(1, 1, VOCAB)
    out[0, -1, token] = 1.0
    return out


class BF16Decoder:
    """Emits the tokens of `script` in turn, recording each call's cache position."""

    def __init__(self, script: list[int]) -> None:
        self.script = list(script)
        self.positions: list[list[int]] = []
        self.inputs: list[list[list[int]]] = []

    def __call__(self, *, input_ids, past_key_values, cache_position, use_cache, return_dict):
        assert use_cache and return_dict
        assert cache_position.tolist() == [past_key_values.length]
        self.positions.append(cache_position.tolist())
        self.inputs.append(input_ids.tolist())
        past_key_values.length += 1
        return SimpleNamespace(logits=_logits(self.script.pop(0)), past_key_values=past_key_values)


class QuantPrefill:
    """The HiF4 model: answers `first` after the whole prompt, records the chunks."""

    def __init__(self, first: int, decode_script: list[int], chunk: int | None = None, eos=5) -> None:
        self.generation_config = SimpleNamespace(eos_token_id=eos)
        self.__dict__["_faquant_bf16_decode_model"] = BF16Decoder(decode_script)
        self.__dict__["_faquant_prefill_chunk_tokens"] = chunk
        attn = SimpleNamespace(faquant_k_matmul_qdq_cache=object(), faquant_v_matmul_qdq_cache=object())
        self.model = SimpleNamespace(layers=[SimpleNamespace(self_attn=attn), SimpleNamespace(self_attn=attn)])
        self.first = first
        self.chunks: list[list[list[int]]] = []

    def __call__(self, *, input_ids, past_key_values, cache_position, use_cache, return_dict, logits_to_keep):
        assert use_cache and return_dict and logits_to_keep == 1
        cache = past_key_values if past_key_values is not None else Cache()
        assert cache_position.tolist() == list(range(cache.length, cache.length + input_ids.shape[1]))
        self.chunks.append(input_ids.tolist())
        cache.length += input_ids.shape[1]
        return SimpleNamespace(logits=_logits(self.first), past_key_values=cache)

    @property
    def decoder(self) -> BF16Decoder:
        return self.__dict__["_faquant_bf16_decode_model"]


def test_one_pass_prefill_then_bf16_decode_until_eos() -> None:
    model = QuantPrefill(first=3, decode_script=[2, 5, 1])
    out = prefill_quant_decode_bf16_generate(model, input_ids=torch.tensor([[1, 4]]), max_length=10)
    assert out.tolist() == [[1, 4, 3, 2, 5]]  # stops after emitting EOS (5)
    assert model.chunks == [[[1, 4]]]
    assert model.decoder.positions == [[2], [3]]
    assert model.decoder.inputs == [[[3]], [[2]]]
    for layer in model.model.layers:
        assert layer.self_attn.faquant_k_matmul_qdq_cache is None
        assert layer.self_attn.faquant_v_matmul_qdq_cache is None


def test_chunked_prefill_feeds_the_prompt_in_order() -> None:
    model = QuantPrefill(first=3, decode_script=[5], chunk=2)
    out = prefill_quant_decode_bf16_generate(model, input_ids=torch.tensor([[1, 2, 4, 0, 2]]), max_length=10)
    assert out.tolist() == [[1, 2, 4, 0, 2, 3, 5]]
    assert model.chunks == [[[1, 2]], [[4, 0]], [[2]]]
    assert model.decoder.positions == [[5]]


def test_first_token_eos_and_max_length_stop_decoding() -> None:
    model = QuantPrefill(first=5, decode_script=[])
    assert prefill_quant_decode_bf16_generate(model, input_ids=torch.tensor([[1]]), max_length=9).tolist() == [[1, 5]]
    assert model.decoder.positions == []
    model = QuantPrefill(first=3, decode_script=[2, 2, 2, 2], eos=[5, 0])
    out = prefill_quant_decode_bf16_generate(model, input_ids=torch.tensor([[1, 1]]), max_length=5)
    assert out.tolist() == [[1, 1, 3, 2, 2]]
    assert len(model.decoder.positions) == 2
    model = QuantPrefill(first=3, decode_script=[2])
    out = prefill_quant_decode_bf16_generate(model, input_ids=torch.tensor([[1, 1]]), max_length=9, eos_token_id=3)
    assert out.tolist() == [[1, 1, 3]]  # the call's eos_token_id overrides the config's


def test_stopping_criteria_tensor_and_bool() -> None:
    calls = []

    def stop_after_two(sequence, scores):
        calls.append(sequence.shape[-1])
        return torch.tensor([sequence.shape[-1] >= 4])

    model = QuantPrefill(first=3, decode_script=[2, 2, 2])
    out = prefill_quant_decode_bf16_generate(model, input_ids=torch.tensor([[1, 1]]), max_length=9,
                                             stopping_criteria=stop_after_two)
    assert out.tolist() == [[1, 1, 3, 2]]
    assert calls == [3, 4]
    model = QuantPrefill(first=3, decode_script=[2])
    out = prefill_quant_decode_bf16_generate(model, input_ids=torch.tensor([[1]]), max_length=9,
                                             stopping_criteria=lambda s, sc: True)
    assert out.tolist() == [[1, 3]]


@pytest.mark.parametrize("kwargs", [dict(do_sample=True), dict(num_beams=2)])
def test_rejects_sampling_and_beams(kwargs) -> None:
    model = QuantPrefill(first=3, decode_script=[])
    with pytest.raises(ValueError):
        prefill_quant_decode_bf16_generate(model, input_ids=torch.tensor([[1]]), max_length=4, **kwargs)


def test_rejects_batches() -> None:
    model = QuantPrefill(first=3, decode_script=[])
    with pytest.raises(ValueError):
        prefill_quant_decode_bf16_generate(model, input_ids=torch.tensor([[1], [2]]), max_length=4)
