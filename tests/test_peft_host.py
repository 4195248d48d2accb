"""Host logic of the PEFT bridge (CPU): which modules are patched and grouped,
the plan cache, and that declined calls run PEFT's own forward unchanged."""

import torch
from torch import nn

from probe_b200 import peft_integration as pi


class _FakeLora(nn.Module):
    """A module carrying PEFT LoRA-Linear attributes (peft is not installed here)."""

    def __init__(self, base, r, alpha, dtype=torch.bfloat16):
        super().__init__()
        self.base_layer = base.to(dtype)
        self.lora_A = nn.ModuleDict({"default": nn.Linear(base.in_features, r, bias=False).to(dtype)})
        self.lora_B = nn.ModuleDict({"default": nn.Linear(r, base.out_features, bias=False).to(dtype)})
        self.lora_dropout = nn.ModuleDict({"default": nn.Dropout(0.1)})
        self.scaling = {"default": alpha / r}
        self.use_dora = {"default": False}
        self._active_adapter = "default"
        self.merged = False
        self.disable_adapters = False

    @property
    def active_adapters(self):
        return [self._active_adapter]

    def forward(self, x):
        a = self.lora_A["default"](self.lora_dropout["default"](x))
        return self.base_layer(x) + self.lora_B["default"](a) * self.scaling["default"]


class _Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.gate_proj = _FakeLora(nn.Linear(32, 48, bias=False), 4, 8)
        self.up_proj = _FakeLora(nn.Linear(32, 48, bias=False), 8, 8)
        self.down_proj = _FakeLora(nn.Linear(48, 32, bias=False), 4, 4)
        self.q_proj = _FakeLora(nn.Linear(32, 32, bias=True), 4, 4)
        self.k_proj = _FakeLora(nn.Linear(32, 16, bias=False), 4, 4)
        self.v_proj = _FakeLora(nn.Linear(32, 16, bias=True), 4, 4)


def test_patch_counts_and_groups():
    blk = _Block().eval()
    assert pi.is_lora_linear(blk.q_proj) and not pi.is_lora_linear(blk.q_proj.base_layer)
    assert pi.enable_loraforge_peft(blk, group_attention=True) == 6
    assert blk._loraforge_grouped_mlp_count == 1 and blk._loraforge_grouped_attention_count == 1
    w, down, up = blk._gate_up_packed
    assert w.shape == (96, 32) and down.shape == (12, 32) and up.shape == (96, 12)
    # block-diagonal up factor with each member's scale folded in
    assert torch.count_nonzero(up[:48, 4:]) == 0 and torch.count_nonzero(up[48:, :4]) == 0
    want = (blk.up_proj.lora_B["default"].weight.float() * blk.up_proj.scaling["default"]).to(torch.bfloat16)
    assert torch.equal(up[48:, 4:], want)
    assert pi.enable_loraforge_peft(blk) == 0  # patching twice is a no-op
    report = pi.peft_plan_report(blk)
    assert report["grouped_mlp_modules"] == 1 and report["grouped_attention_modules"] == 1


def test_declined_calls_run_peft_forward():
    blk = _Block().eval()
    ref = {n: getattr(blk, n).forward for n in ("down_proj", "gate_proj", "q_proj")}
    x = torch.randn(5, 32, dtype=torch.bfloat16)
    h = torch.randn(5, 48, dtype=torch.bfloat16)
    want = {"down_proj": ref["down_proj"](h), "gate_proj": ref["gate_proj"](x), "q_proj": ref["q_proj"](x)}
    pi.enable_loraforge_peft(blk, group_attention=True)
    # CPU activations: declined, PEFT's forward runs (grouped members fall back too)
    assert torch.equal(blk.down_proj(h), want["down_proj"])
    assert torch.equal(blk.gate_proj(x), want["gate_proj"])
    assert torch.equal(blk.q_proj(x), want["q_proj"])
    blk.train()  # training mode: PEFT's forward, dropout included
    torch.manual_seed(5)
    got = blk.down_proj(h)
    torch.manual_seed(5)
    assert torch.equal(got, ref["down_proj"](h))


def test_plan_cache_keeps_two_most_recent():
    cache = pi._PlanCache(size=2)
    calls = {k: object() for k in "abc"}
    for k in "ab":
        cache.store(k, calls[k])
    assert cache.lookup("a") is calls["a"]  # a becomes the most recent
    cache.store("c", calls["c"])            # evicts b
    assert cache.lookup("b") is None and cache.lookup("a") is calls["a"] and cache.lookup("c") is calls["c"]


def test_scaling_change_is_a_new_plan():
    blk = _Block().eval()
    pi.enable_loraforge_peft(blk, enable_grouping=False)
    x = torch.randn(3, 48, dtype=torch.bfloat16)
    blk.down_proj(x)
    k1 = blk.down_proj._loraforge_plans.last_key
    blk.down_proj.scaling["default"] = 0.0
    blk.down_proj(x)
    assert blk.down_proj._loraforge_plans.last_key != k1
