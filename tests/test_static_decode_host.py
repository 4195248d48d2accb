"""Host-side checks of the CUDA-graph decode runner (CPU): inputs it must
refuse before touching a GPU, as the reference's runner does
(static_decode.py:11-40)."""

import pytest
import torch


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=32, hidden_size=64, intermediate_size=128, num_hidden_layers=1,
                      num_attention_heads=2, num_key_value_heads=1, max_position_embeddings=64)
    return LlamaForCausalLM(cfg).eval()


@pytest.mark.parametrize("ids,new_tokens", [
    (torch.zeros(1, 4, dtype=torch.long), 2),      # host tensor
    (torch.zeros(4, dtype=torch.long), 2),         # not [batch, prefix]
    (torch.zeros(1, 4, dtype=torch.int32), 2),     # not int64
    (torch.zeros(1, 4, dtype=torch.long), 0),      # no tokens to generate
])
def test_runner_refuses_bad_inputs_before_any_device_work(ids, new_tokens):
    from probe_b200.static_decode import StaticDecodeRunner

    with pytest.raises(ValueError):
        StaticDecodeRunner(_tiny_llama(), ids, new_tokens)
