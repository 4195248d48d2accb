"""Inference-only PEFT integration (drop-in for peft_integration.py:1-479).

``enable_loraforge_peft(model)`` reroutes the forward of every PEFT LoRA
``Linear`` through this package's B200 kernels.  A module keeps PEFT's own
forward unless it has exactly one active adapter, no DoRA, an inactive
dropout, CUDA fp16/bf16 activations matching the base weight's dtype and an
``nn.Linear`` base -- the same set of modules the reference accepts
(peft_integration.py:41-63).  Calls with extra arguments, in training mode,
on merged weights or with adapters disabled also take PEFT's forward.

Plans.  Each patched module owns a :class:`_PlanCache`: a resolved callable
per (active adapters, row count, scaling, dtype, device), holding at most two
(a prefill shape and a decode shape, the usual pair), so a forward costs one
key comparison once warm.  Scaling is part of the key, so a ``set_scale``
between calls (a zero scale turns the module into its base linear) is seen.

Grouping.  Sibling projections that read the same input are served by ONE
packed linear (:class:`_SiblingGroup`): their base weights stacked along the
output, their down factors stacked along the rank and a block-diagonal up
factor with each member's scale folded in, so one shrink and one GEMM (or one
small-M launch) read x once for all of them.  ``enable_grouping`` packs a
transformer MLP's gate and up projections (the reference groups those for
decode, peft_integration.py:270-411); ``group_attention`` (or
``LORAFORGE_GROUPED_ATTN=1``) also packs an attention block's q, k and v.
``LORAFORGE_GROUPED_MLP=individual`` turns the MLP grouping off.

``peft`` itself is optional: modules are recognised by PEFT's LoRA Linear
attributes when the package is not importable.
"""

from __future__ import annotations

import os
import types
from collections import Counter, OrderedDict

import torch

from .fused_linear import MIN_GEMM_ROWS, build_plan

try:  # pragma: no cover - exercised only where peft is installed
    from peft.tuners.lora.layer import Linear as _PeftLoraLinear
except Exception:  # noqa: BLE001
    _PeftLoraLinear = None

_HALF = (torch.float16, torch.bfloat16)
_PEFT_ATTRS = ("lora_A", "lora_B", "scaling", "base_layer", "active_adapters")


def is_lora_linear(module) -> bool:
    """A PEFT LoRA Linear (or an object exposing the same attributes)."""
    if _PeftLoraLinear is not None and isinstance(module, _PeftLoraLinear):
        return True
    if "lora_A" not in module.__dict__.get("_modules", {}):
        return False
    return all(hasattr(module, attr) for attr in _PEFT_ATTRS)


def _dropout_is_identity(layer) -> bool:
    """In eval mode a Dropout passes x through whatever its p (and Identity always does)."""
    if isinstance(layer, torch.nn.Identity):
        return True
    return isinstance(layer, torch.nn.Dropout) and not layer.training


def _bypassed(module) -> bool:
    """States in which the module must run PEFT's own forward."""
    return module.training or bool(getattr(module, "merged", False)) or bool(getattr(module, "disable_adapters", False))


def _adapter_factors(module, adapter: str, dtype=None):
    """(A [r, K], B [N, r], scale) of ``adapter`` when the kernels can serve it, else None."""
    if adapter not in module.lora_A or adapter not in module.lora_B:
        return None
    if (getattr(module, "use_dora", None) or {}).get(adapter, False):
        return None
    if not isinstance(module.base_layer, torch.nn.Linear) or not _dropout_is_identity(module.lora_dropout[adapter]):
        return None
    a, b = module.lora_A[adapter].weight, module.lora_B[adapter].weight
    want = module.base_layer.weight.dtype if dtype is None else dtype
    if a.ndim != 2 or b.ndim != 2 or want not in _HALF or module.base_layer.weight.dtype != want:
        return None
    if a.dtype != want or b.dtype != want:
        return None
    return a, b, float(module.scaling[adapter])


def _as_rows(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    return x2 if x2.is_contiguous() else x2.contiguous()


# ------------------------------------------------------------------ plans
class _PlanCache:
    """Resolved forwards of one module, most recently used last, at most ``size``."""

    def __init__(self, size: int = 2):
        self.size = size
        self.entries: OrderedDict[tuple, object] = OrderedDict()
        self.last_key = None
        self.last_call = None

    def lookup(self, key):
        if key == self.last_key:
            return self.last_call
        call = self.entries.get(key)
        if call is not None:
            self.entries.move_to_end(key)
            self.last_key, self.last_call = key, call
        return call

    def store(self, key, call):
        self.entries[key] = call
        self.entries.move_to_end(key)
        while len(self.entries) > self.size:
            self.entries.popitem(last=False)
        self.last_key, self.last_call = key, call
        return call


def _plan_key(module, x: torch.Tensor, rows: int) -> tuple:
    return (tuple(module.active_adapters), rows, tuple(sorted(module.scaling.items())), x.dtype, x.device)


def _resolve(module, x: torch.Tensor, rows: int):
    """The forward for this key: a kernel plan, or PEFT's forward when declined."""
    declined = module._loraforge_original_forward
    adapters = list(module.active_adapters)
    if len(adapters) != 1 or not x.is_cuda or x.dtype not in _HALF:
        return declined
    factors = _adapter_factors(module, adapters[0], dtype=x.dtype)
    if factors is None:
        return declined
    a, b, scale = factors
    base = module.base_layer
    if a.shape[0] == 0 or scale == 0:
        module._loraforge_decode_choice = "base"
    else:
        module._loraforge_decode_choice = "decode" if rows < MIN_GEMM_ROWS else "gemm"
    plan = build_plan(_as_rows(x), base.weight, base.bias, a, b, scale)
    width = base.out_features

    def run(x):
        return plan(_as_rows(x)).reshape(*x.shape[:-1], width)

    return run


def _patched_forward(self, x: torch.Tensor, *args, **kwargs):
    """Inference forward of a patched PEFT LoRA Linear (peft_integration.py:199-232)."""
    if args or kwargs or _bypassed(self):
        return self._loraforge_original_forward(x, *args, **kwargs)
    rows = x.numel() // x.shape[-1]
    key = _plan_key(self, x, rows)
    cache = self._loraforge_plans
    call = cache.lookup(key)
    if call is None:
        call = cache.store(key, _resolve(self, x, rows))
    self._loraforge_plan = call
    return call(x)


# --------------------------------------------------------------- grouping
class _SiblingGroup:
    """Projections of one parent that read the same x, served by one packed linear.

    The first member called with a new x computes every member's output and
    keeps the others' for their own calls.  The key of that hand-off is x's
    storage address, shape and version counter, so an x written in place in
    between (or any other x) makes the member compute on its own.  Calls with
    extra arguments, other dtypes, several or disabled adapters or merged
    weights take the members' individual forwards.  So do 129..256-row calls
    whose summed rank exceeds 64: the one-launch split-K linear serving that
    row range takes ranks up to 64, and the individual projections measured
    faster than the packed one there.
    """

    def __init__(self, parent, names, members, adapter: str, tag: str):
        self.parent, self.names, self.members, self.adapter, self.tag = parent, names, members, adapter, tag
        ws = [m.base_layer.weight for m in members]
        self.dtype = ws[0].dtype
        self.widths = [w.shape[0] for w in ws]
        ranks = [m.lora_A[adapter].weight.shape[0] for m in members]
        self.rank = sum(ranks)
        device = ws[0].device
        self.weight = torch.cat([w.detach() for w in ws], dim=0).contiguous()
        self.down = torch.cat([m.lora_A[adapter].weight.detach() for m in members], dim=0).contiguous()
        self.up = torch.zeros((sum(self.widths), self.rank), device=device, dtype=self.dtype)
        self.bias = None
        if any(m.base_layer.bias is not None for m in members):
            self.bias = torch.zeros((sum(self.widths),), device=device, dtype=self.dtype)
        row = col = 0
        for m, width, r in zip(members, self.widths, ranks):
            scaled = m.lora_B[adapter].weight.detach().float() * float(m.scaling[adapter])
            self.up[row:row + width, col:col + r].copy_(scaled)
            if m.base_layer.bias is not None:
                self.bias[row:row + width].copy_(m.base_layer.bias.detach())
            row, col = row + width, col + r
        self.individual = [m.forward for m in members]
        self.plans: dict[int, object] = {}
        self.handoff_key = None
        self.handoff: dict[int, torch.Tensor] = {}

    @staticmethod
    def eligible(members, adapter: str, max_rank: int = 128) -> bool:
        factors = [_adapter_factors(m, adapter) for m in members]
        if any(f is None for f in factors) or any(list(m.active_adapters) != [adapter] for m in members):
            return False
        k = members[0].base_layer.weight.shape[1]
        dtype = members[0].base_layer.weight.dtype
        same = all(m.base_layer.weight.shape[1] == k and m.base_layer.weight.dtype == dtype for m in members)
        return same and sum(f[0].shape[0] for f in factors) <= max_rank

    def _packable(self, x, args, kwargs) -> bool:
        if args or kwargs or not x.is_cuda or x.dtype != self.dtype:
            return False
        return all(list(m.active_adapters) == [self.adapter] and not getattr(m, "merged", False)
                   and not getattr(m, "disable_adapters", False) for m in self.members)

    def call(self, index: int, x: torch.Tensor, *args, **kwargs):
        key = (x.data_ptr(), tuple(x.shape), x._version)
        if not args and not kwargs and key == self.handoff_key and index in self.handoff:
            return self.handoff.pop(index)
        self.handoff_key, self.handoff = None, {}
        if not self._packable(x, args, kwargs):
            return self.individual[index](x, *args, **kwargs)
        x2 = _as_rows(x)
        rows = x2.shape[0]
        if 128 < rows <= 256 and self.rank > 64:
            self.parent._loraforge_grouped_choices[rows] = "individual"
            return self.individual[index](x, *args, **kwargs)
        plan = self.plans.get(rows)
        if plan is None:
            plan = self.plans[rows] = build_plan(x2, self.weight, self.bias, self.down, self.up, 1.0)
            self.parent._loraforge_grouped_choices[rows] = "grouped"
        packed = plan(x2)
        outs, c0 = {}, 0
        for j, width in enumerate(self.widths):
            outs[j] = packed[:, c0:c0 + width].reshape(*x.shape[:-1], width)
            c0 += width
        mine = outs.pop(index)
        self.handoff_key, self.handoff = key, outs
        return mine

    def install(self) -> None:
        for i, m in enumerate(self.members):
            m._loraforge_individual_forward = self.individual[i]

            def forward(module, x, *args, _i=i, **kwargs):
                return self.call(_i, x, *args, **kwargs)

            m.forward = types.MethodType(forward, m)
        if "_loraforge_grouped_choices" not in self.parent.__dict__:
            self.parent._loraforge_grouped_choices = {}
            self.parent._loraforge_grouped_timings_us = {}


def _group_siblings(parent, names, tag: str) -> _SiblingGroup | None:
    """Pack ``parent``'s children ``names`` into one group if they qualify."""
    if parent.__dict__.get(f"_loraforge_grouped_{tag}", False):
        return None
    members = [parent._modules.get(nm) for nm in names]  # direct children only (PEFT wrappers delegate getattr)
    if any(m is None or not is_lora_linear(m) for m in members):
        return None
    active = list(members[0].active_adapters)
    if len(active) != 1 or not _SiblingGroup.eligible(members, active[0]):
        return None
    group = _SiblingGroup(parent, names, members, active[0], tag)
    group.install()
    setattr(parent, f"_loraforge_grouped_{tag}", True)
    return group


MLP_GROUP = ("gate_proj", "up_proj")
ATTENTION_GROUP = ("q_proj", "k_proj", "v_proj")


def _patch_grouped_mlp(mlp_module) -> bool:
    """Serve gate_proj and up_proj with one packed linear (peft_integration.py:270-411)."""
    group = _group_siblings(mlp_module, MLP_GROUP, "mlp")
    if group is None:
        return False
    mlp_module._gate_up_packed = (group.weight, group.down, group.up)
    return True


def _patch_grouped_siblings(parent, names, tag: str) -> bool:
    """Serve sibling projections ``names`` of ``parent`` with one packed linear.

    Used for an attention block's q, k and v (an extension: the reference
    groups only gate/up).  Output widths may differ (grouped-query attention).
    Measured at K = N = 4096, r = 16 per projection: 8192 rows 829 -> 824 us,
    16 rows 42.1 -> 39.7 us for the three projections.
    """
    group = _group_siblings(parent, names, tag)
    if group is None:
        return False
    setattr(parent, f"_{tag}_packed", (group.weight, group.down, group.up, group.bias))
    return True


# ------------------------------------------------------------ public API
def _cast_adapters(module) -> None:
    """Bring the active adapters' factors to the base weight's half dtype (PEFT
    often keeps them in fp32 for training)."""
    if not isinstance(module.base_layer, torch.nn.Linear):
        return
    target = module.base_layer.weight.dtype
    if target not in _HALF:
        return
    for adapter in module.active_adapters:
        for table in (module.lora_A, module.lora_B):
            if adapter in table:
                table[adapter].to(dtype=target)


def enable_loraforge_peft(model, enable_grouping: bool = True, cast_adapter_dtype: bool = True,
                          group_attention: bool | None = None) -> int:
    """Patch the model's PEFT LoRA Linear modules for inference; returns how many
    were patched (peft_integration.py:414-448).

    ``cast_adapter_dtype`` casts active adapter factors to the base dtype
    (pass False to keep PEFT's fp32 sidecars, which then take PEFT's forward).
    ``enable_grouping`` packs MLP gate/up pairs; ``group_attention`` (default:
    ``LORAFORGE_GROUPED_ATTN``, off) packs q/k/v.
    """
    patched = 0
    for module in list(model.modules()):
        if not is_lora_linear(module) or "_loraforge_original_forward" in module.__dict__:
            continue
        if cast_adapter_dtype:
            _cast_adapters(module)
        module._loraforge_original_forward = module.forward
        module._loraforge_plan = None
        module._loraforge_plans = _PlanCache()
        module.forward = types.MethodType(_patched_forward, module)
        patched += 1

    if enable_grouping and os.environ.get("LORAFORGE_GROUPED_MLP", "").strip().lower() != "individual":
        for m in list(model.modules()):
            _patch_grouped_mlp(m)
    if group_attention is None:
        group_attention = os.environ.get("LORAFORGE_GROUPED_ATTN", "").strip().lower() in ("1", "true", "yes")
    if group_attention:
        for m in list(model.modules()):
            _patch_grouped_siblings(m, ATTENTION_GROUP, "attention")
    # groups installed in the model so far (a repeated call counts earlier ones too)
    model._loraforge_grouped_mlp_count = sum(
        bool(m.__dict__.get("_loraforge_grouped_mlp")) for m in model.modules())
    model._loraforge_grouped_attention_count = sum(
        bool(m.__dict__.get("_loraforge_grouped_attention")) for m in model.modules())
    return patched


def peft_plan_report(model) -> dict:
    """Which path each patched module and group took (peft_integration.py:451-479)."""
    decode = Counter()
    decode_samples = []
    grouped = Counter()
    grouped_samples = []
    for module in model.modules():
        state = module.__dict__  # not getattr: PEFT wrappers delegate attribute lookups
        choice = state.get("_loraforge_decode_choice")
        if choice is not None:
            decode[choice] += 1
            decode_samples.append({"choice": choice, "timings_us": state.get("_loraforge_decode_timings_us", {})})
        timings = state.get("_loraforge_grouped_timings_us", {})
        for rows, how in state.get("_loraforge_grouped_choices", {}).items():
            grouped[how] += 1
            grouped_samples.append({"rows": rows, "choice": how, "timings_us": timings.get(rows, {})})
    return {
        "decode_choices": dict(decode),
        "grouped_mlp_modules": getattr(model, "_loraforge_grouped_mlp_count", 0),
        "grouped_attention_modules": getattr(model, "_loraforge_grouped_attention_count", 0),
        "decode_timing_samples": decode_samples,
        "grouped_mlp_choices": dict(grouped),
        "grouped_mlp_timing_samples": grouped_samples,
    }
