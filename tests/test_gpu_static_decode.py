"""CUDA-graph greedy decoding (GPU): replayed decode equals the eager steps and
Transformers' own greedy ``generate``.

Follows the reference's test (test_static_decode.py:14-51): a tiny random
Llama (2 layers, grouped-query attention) in bf16, first plain, then with
nonzero LoRAs on q_proj and v_proj served by this package's kernels through
the PEFT bridge; batches 1 and 2, 1 and 6 new tokens, changing prompts.  PEFT
is not installed here, so the LoRA layers are small modules carrying PEFT's
LoRA-Linear attributes (the bridge recognises those).
"""

import pytest
import torch
from torch import nn

pytestmark = pytest.mark.gpu
DEV = "cuda"


class _LoraOnLinear(nn.Module):
    """base_layer + scaling * lora_B(lora_A(x)), with PEFT LoRA-Linear attributes."""

    def __init__(self, base, r, alpha):
        super().__init__()
        self.base_layer = base
        dt, dev = base.weight.dtype, base.weight.device
        self.lora_A = nn.ModuleDict({"default": nn.Linear(base.in_features, r, bias=False).to(dev, dt)})
        self.lora_B = nn.ModuleDict({"default": nn.Linear(r, base.out_features, bias=False).to(dev, dt)})
        with torch.no_grad():
            self.lora_B["default"].weight.normal_(std=0.03)
        self.lora_dropout = nn.ModuleDict({"default": nn.Identity()})
        self.scaling = {"default": alpha / r}
        self.use_dora = {"default": False}
        self._active_adapter = "default"
        self.merged = False
        self.disable_adapters = False
        self.in_features, self.out_features = base.in_features, base.out_features

    @property
    def active_adapters(self):
        return [self._active_adapter]

    @property
    def weight(self):
        return self.base_layer.weight

    def forward(self, x):
        return self.base_layer(x) + self.lora_B["default"](self.lora_A["default"](x)) * self.scaling["default"]


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=64, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512,
                      bos_token_id=1, eos_token_id=2, pad_token_id=0)
    return LlamaForCausalLM(cfg).to(DEV, torch.bfloat16).eval()


@torch.inference_mode()
def test_static_decode_matches_eager_and_generate():
    from probe_b200 import enable_loraforge_peft
    from probe_b200.static_decode import StaticDecodeRunner

    torch.manual_seed(53)
    model = _tiny_llama()
    for adapted in (False, True):
        if adapted:
            for layer in model.model.layers:
                attn = layer.self_attn
                attn.q_proj = _LoraOnLinear(attn.q_proj, 3, 3)
                attn.v_proj = _LoraOnLinear(attn.v_proj, 3, 3)
            assert enable_loraforge_peft(model, enable_grouping=False) == 4
        for batch in (1, 2):
            ids = torch.randint(3, 64, (batch, 7), device=DEV)
            for count in (1, 6):
                runner = StaticDecodeRunner(model, ids, count)
                for _ in range(2):
                    ids.random_(3, 64)
                    want = model.generate(input_ids=ids, attention_mask=torch.ones_like(ids), do_sample=False,
                                          min_new_tokens=count, max_new_tokens=count, pad_token_id=0)
                    eager = runner(ids, replay=False)
                    got = runner(ids)
                    assert torch.equal(got, eager), (adapted, batch, count, "graph/eager")
                    assert torch.equal(got, want), (adapted, batch, count, "generate")
    # a longer prompt (prefill through the GEMM path), validated step by step
    ids = torch.randint(3, 64, (2, 129), device=DEV)
    runner = StaticDecodeRunner(model, ids, 6)
    for _ in range(2):
        ids.random_(3, 64)
        assert runner.validate(ids) == 0.0
        assert torch.equal(runner(ids), runner(ids, replay=False))


def test_static_decode_rejects_bad_inputs():
    from probe_b200.static_decode import StaticDecodeRunner

    model = _tiny_llama()
    with pytest.raises(ValueError):
        StaticDecodeRunner(model, torch.zeros(2, 0, dtype=torch.long, device=DEV), 3)
    with pytest.raises(ValueError):
        StaticDecodeRunner(model, torch.zeros(2, 4, dtype=torch.long, device=DEV), 0)
    runner = StaticDecodeRunner(model, torch.randint(3, 64, (1, 5), device=DEV), 2)
    with pytest.raises(ValueError):
        runner(torch.randint(3, 64, (1, 6), device=DEV))
