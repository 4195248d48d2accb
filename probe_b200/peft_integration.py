"""Inference-only PEFT integration (drop-in for peft_integration.py:1-479).

``enable_loraforge_peft(model)`` patches every PEFT LoRA ``Linear`` so that its
forward runs the B200 kernels of this package.  As in the reference, a module
is declined -- it keeps PEFT's own forward -- unless it has exactly one active
adapter, no DoRA, an inactive dropout, CUDA fp16/bf16 tensors of one dtype and
an ``nn.Linear`` base (peft_integration.py:41-63).  A plan is resolved once per
(adapter, row count, scaling, dtype, device) and the last two are kept
(peft_integration.py:199-232).

Grouping (``enable_grouping``): a transformer MLP's gate and up projections
read the same x.  Their weights are packed once into ``[W_gate; W_up]`` with a
block-diagonal ``[B_gate*s_g, 0; 0, B_up*s_u]`` sidecar, so one shrink and one
GEMM (or one decode launch) serve both projections
(the reference groups the decode sidecars only, peft_integration.py:270-411).
With ``group_attention`` the same packing serves an attention block's q, k and
v projections (an extension; the reference has no attention grouping).

``peft`` itself is optional: modules are recognised by PEFT's LoRA Linear
attributes when the package is not importable.
"""

from __future__ import annotations

import os
import types
from collections import Counter

import torch

from .fused_linear import MIN_GEMM_ROWS, build_plan

try:  # pragma: no cover - exercised only where peft is installed
    from peft.tuners.lora.layer import Linear as _PeftLoraLinear
except Exception:  # noqa: BLE001
    _PeftLoraLinear = None

_GROUPED_MLP_CHOICE_CACHE: dict = {}


def is_lora_linear(module) -> bool:
    """A PEFT LoRA Linear (or an object exposing the same attributes)."""
    if _PeftLoraLinear is not None and isinstance(module, _PeftLoraLinear):
        return True
    d = module.__dict__
    return all(hasattr(module, a) for a in ("lora_A", "lora_B", "scaling", "base_layer", "active_adapters")) and \
        "_modules" in d and "lora_A" in d["_modules"]


def _inactive_dropout(dropout):
    """Training dropout is an identity after eval(), regardless of saved p."""
    return isinstance(dropout, torch.nn.Identity) or (
        isinstance(dropout, torch.nn.Dropout) and not dropout.training
    )


def _sidecar(module, name):
    """Return (A, B, scale) for one active adapter, or None if unsupported."""
    use_dora = getattr(module, "use_dora", {}) or {}
    if name not in module.lora_A or use_dora.get(name, False):
        return None
    a = module.lora_A[name].weight
    b = module.lora_B[name].weight
    if a.ndim != 2 or b.ndim != 2:
        return None
    return a, b, float(module.scaling[name])


def _supported(module, x, name):
    base_layer = module.base_layer
    sidecar = _sidecar(module, name)
    if sidecar is None:
        return None
    a, b, scale = sidecar
    ok = (
        isinstance(base_layer, torch.nn.Linear)
        and _inactive_dropout(module.lora_dropout[name])
        and x.is_cuda
        and x.dtype in (torch.float16, torch.bfloat16)
        and x.dtype == base_layer.weight.dtype
        and a.dtype == x.dtype
        and b.dtype == x.dtype
    )
    return (a, b, scale) if ok else None


def _build_plan(module, x, rows):
    """Resolve everything that does not change between steps, once (peft_integration.py:41-96)."""
    declined = (module._active_adapter, rows, None)
    active = list(module.active_adapters)
    if len(active) != 1:
        return declined
    name = active[0]
    sidecar = _supported(module, x, name)
    if sidecar is None:
        return declined
    a, b, scale = sidecar
    base_layer = module.base_layer
    probe = x.reshape(-1, x.shape[-1])
    if not probe.is_contiguous():
        probe = probe.contiguous()
    run = build_plan(probe, base_layer.weight, base_layer.bias, a, b, scale)
    module._loraforge_decode_choice = "base" if (a.shape[0] == 0 or scale == 0) else (
        "decode" if rows < MIN_GEMM_ROWS else "gemm")
    out_features = base_layer.out_features

    def call(x):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        return run(x2).reshape(*shape[:-1], out_features)

    return module._active_adapter, rows, call


def _loraforge_linear_forward(self, x: torch.Tensor, *args, **kwargs):
    """Drop-in inference forward for a PEFT LoRA Linear (peft_integration.py:199-232)."""
    if args or kwargs or self.training or getattr(self, "merged", False) or getattr(self, "disable_adapters", False):
        return self._loraforge_original_forward(x, *args, **kwargs)
    rows = x.numel() // x.shape[-1]
    plan = getattr(self, "_loraforge_plan", None)
    if (plan is None or plan[0] != self._active_adapter or plan[1] != rows
            or plan[3] != self.scaling or plan[4] != (x.dtype, x.device)):
        cache = self._loraforge_plans
        key = (tuple(self.active_adapters), rows, tuple(self.scaling.items()), x.dtype, x.device)
        plan = cache.get(key)
        if plan is None:
            adapter, plan_rows, call = _build_plan(self, x, rows)
            adapter = adapter.copy() if isinstance(adapter, list) else adapter
            plan = (adapter, plan_rows, call, dict(self.scaling), (x.dtype, x.device))
            if len(cache) >= 2:
                cache.pop(next(iter(cache)))
            cache[key] = plan
        self._loraforge_plan = plan
    call = plan[2]
    if call is not None:
        return call(x)
    return self._loraforge_original_forward(x)


def _patch_grouped_mlp(mlp_module) -> bool:
    """Serve gate_proj and up_proj with one packed weight (peft_integration.py:270-411).

    The gate call computes both projections and caches up for the following
    up call on the same input; anything unusual falls back to the individual
    forwards.
    """
    gate_proj = mlp_module._modules.get("gate_proj")
    up_proj = mlp_module._modules.get("up_proj")
    if getattr(mlp_module, "_loraforge_grouped_mlp", False):
        return False
    if gate_proj is None or up_proj is None or not (is_lora_linear(gate_proj) and is_lora_linear(up_proj)):
        return False
    name = list(gate_proj.active_adapters)[0] if gate_proj.active_adapters else "default"
    if name not in gate_proj.lora_A or name not in up_proj.lora_A:
        return False
    wg, wu = gate_proj.base_layer.weight, up_proj.base_layer.weight
    a_g, a_u = gate_proj.lora_A[name].weight, up_proj.lora_A[name].weight
    b_g, b_u = gate_proj.lora_B[name].weight, up_proj.lora_B[name].weight
    rg, ru = a_g.shape[0], a_u.shape[0]
    if rg + ru > 128 or wg.shape != wu.shape:
        return False
    dtype = wg.dtype
    if not (
        _inactive_dropout(gate_proj.lora_dropout[name]) and _inactive_dropout(up_proj.lora_dropout[name])
        and all(t.dtype == dtype for t in (wu, a_g, a_u, b_g, b_u)) and dtype in (torch.float16, torch.bfloat16)
        and gate_proj.base_layer.bias is None and up_proj.base_layer.bias is None
    ):
        return False
    n, k = wg.shape
    # Packed once: [W_g; W_u], [A_g; A_u], block-diagonal B with scales folded.
    w_gu = torch.cat([wg, wu], dim=0).detach().contiguous()
    a_gu = torch.cat([a_g, a_u], dim=0).detach().contiguous()
    b_gu = torch.zeros((2 * n, rg + ru), device=wg.device, dtype=dtype)
    b_gu[:n, :rg].copy_(b_g.detach().float() * float(gate_proj.scaling[name]))
    b_gu[n:, rg:].copy_(b_u.detach().float() * float(up_proj.scaling[name]))

    gate_individual = gate_proj.forward
    up_individual = up_proj.forward
    cache = {"key": None, "up": None}
    plans = {}

    def gate_forward(self, x, *args, **kwargs):
        rows = x.numel() // x.shape[-1]
        if (
            args or kwargs or list(self.active_adapters) != [name] or list(up_proj.active_adapters) != [name]
            or getattr(self, "merged", False) or getattr(up_proj, "merged", False)
            or getattr(self, "disable_adapters", False) or getattr(up_proj, "disable_adapters", False)
            or not x.is_cuda or x.dtype != dtype
        ):
            cache["key"] = cache["up"] = None
            return gate_individual(x, *args, **kwargs)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        plan = plans.get(rows)
        if plan is None:
            plan = build_plan(x2, w_gu, None, a_gu, b_gu, 1.0)
            plans[rows] = plan
            mlp_module._loraforge_grouped_choices[rows] = "grouped"
        both = plan(x2)
        gate = both[:, :n].reshape(*shape[:-1], n)
        up = both[:, n:].reshape(*shape[:-1], n)
        cache["key"] = (x.data_ptr(), tuple(shape))
        cache["up"] = up
        return gate

    def up_forward(self, x, *args, **kwargs):
        key = (x.data_ptr(), tuple(x.shape))
        if not args and not kwargs and cache["key"] == key and cache["up"] is not None:
            result = cache["up"]
            cache["key"] = cache["up"] = None
            return result
        cache["key"] = cache["up"] = None
        return up_individual(x, *args, **kwargs)

    gate_proj._loraforge_individual_forward = gate_individual
    up_proj._loraforge_individual_forward = up_individual
    gate_proj.forward = types.MethodType(gate_forward, gate_proj)
    up_proj.forward = types.MethodType(up_forward, up_proj)
    mlp_module._gate_up_packed = (w_gu, a_gu, b_gu)
    mlp_module._loraforge_grouped_choices = {}
    mlp_module._loraforge_grouped_timings_us = {}
    mlp_module._loraforge_grouped_mlp = True
    return True


ATTENTION_GROUP = ("q_proj", "k_proj", "v_proj")


def _patch_grouped_siblings(parent, names, tag: str) -> bool:
    """Serve sibling projections that read the same x with ONE packed linear.

    An extension beyond the reference (which groups only gate/up): for an
    attention block's q, k and v (``names``), ``[W_q; W_k; W_v]`` and
    ``[A_q; A_k; A_v]`` are packed once with a block-diagonal
    ``[B_q*s_q, 0, 0; 0, B_k*s_k, 0; 0, 0, B_v*s_v]`` sidecar and the biases side
    by side, so one plan (one shrink and one GEMM, or one small-M launch) reads x
    once for all of them.  Output widths may differ (grouped-query attention).
    Whichever member is called first with a new x computes every member's
    output and keeps the others' for their own calls; the cache key is x's
    storage, shape and version counter, so an x modified in place in between
    takes the member's individual forward.  Anything unusual (other call
    arguments, several or disabled adapters, merged weights, other dtypes)
    also falls back to the individual forwards, and so do 129..256-row calls
    whose summed rank exceeds 32 (measured slower packed there).  Measured at
    K = N = 4096, r = 16 per projection: 8192 rows 829 -> 824 us, 16 rows
    42.1 -> 39.7 us for the three projections.
    """
    mods = [parent._modules.get(nm) for nm in names]
    if any(m is None or not is_lora_linear(m) for m in mods):
        return False
    if getattr(parent, "_loraforge_grouped_" + tag, False):
        return False
    name = list(mods[0].active_adapters)[0] if mods[0].active_adapters else "default"
    ws, bs, a_s, b_s, ranks = [], [], [], [], []
    for m in mods:
        if name not in m.lora_A or list(m.active_adapters) != [name] or not isinstance(m.base_layer, torch.nn.Linear):
            return False
        if not _inactive_dropout(m.lora_dropout[name]) or (getattr(m, "use_dora", {}) or {}).get(name, False):
            return False
        ws.append(m.base_layer.weight)
        bs.append(m.base_layer.bias)
        a_s.append(m.lora_A[name].weight)
        b_s.append(m.lora_B[name].weight)
        ranks.append(a_s[-1].shape[0])
    dtype = ws[0].dtype
    k = ws[0].shape[1]
    if dtype not in (torch.float16, torch.bfloat16) or sum(ranks) > 128:
        return False
    if any(w.shape[1] != k or w.dtype != dtype for w in ws) or any(t.dtype != dtype for t in a_s + b_s):
        return False
    widths = [w.shape[0] for w in ws]
    n_all, r_all = sum(widths), sum(ranks)
    w_pack = torch.cat(ws, dim=0).detach().contiguous()
    a_pack = torch.cat(a_s, dim=0).detach().contiguous()
    b_pack = torch.zeros((n_all, r_all), device=ws[0].device, dtype=dtype)
    bias_pack = None
    if any(b is not None for b in bs):
        bias_pack = torch.zeros((n_all,), device=ws[0].device, dtype=dtype)
    n0 = r0 = 0
    for m, w, bias, bb, r in zip(mods, ws, bs, b_s, ranks):
        b_pack[n0:n0 + w.shape[0], r0:r0 + r].copy_(bb.detach().float() * float(m.scaling[name]))
        if bias is not None:
            bias_pack[n0:n0 + w.shape[0]].copy_(bias.detach())
        n0 += w.shape[0]
        r0 += r
    individual = [m.forward for m in mods]
    cache = {"key": None, "outs": {}}
    plans = {}

    def member_forward(i):
        def forward(self, x, *args, **kwargs):
            key = (x.data_ptr(), tuple(x.shape), x._version)
            if not args and not kwargs and cache["key"] == key and i in cache["outs"]:
                return cache["outs"].pop(i)
            cache["key"], cache["outs"] = None, {}
            if (
                args or kwargs or not x.is_cuda or x.dtype != dtype
                or any(list(m.active_adapters) != [name] or getattr(m, "merged", False)
                       or getattr(m, "disable_adapters", False) for m in mods)
            ):
                return individual[i](x, *args, **kwargs)
            shape = x.shape
            x2 = x.reshape(-1, shape[-1])
            if not x2.is_contiguous():
                x2 = x2.contiguous()
            rows = x2.shape[0]
            if 128 < rows <= 256 and r_all > 64:
                # the one-launch split-K linear of this row range takes ranks <= 64
                # only: the individual projections measured faster here than the
                # pack with its summed rank
                return individual[i](x, *args, **kwargs)
            plan = plans.get(rows)
            if plan is None:
                plan = build_plan(x2, w_pack, bias_pack, a_pack, b_pack, 1.0)
                plans[rows] = plan
                parent._loraforge_grouped_choices[rows] = "grouped"
            packed = plan(x2)
            outs, c0 = {}, 0
            for j, wd in enumerate(widths):
                outs[j] = packed[:, c0:c0 + wd].reshape(*shape[:-1], wd)
                c0 += wd
            mine = outs.pop(i)
            cache["key"], cache["outs"] = key, outs
            return mine
        return forward

    for i, m in enumerate(mods):
        m._loraforge_individual_forward = individual[i]
        m.forward = types.MethodType(member_forward(i), m)
    setattr(parent, "_" + tag + "_packed", (w_pack, a_pack, b_pack, bias_pack))
    if not hasattr(parent, "_loraforge_grouped_choices"):
        parent._loraforge_grouped_choices = {}
    setattr(parent, "_loraforge_grouped_" + tag, True)
    return True


def enable_loraforge_peft(model, enable_grouping: bool = True, cast_adapter_dtype: bool = True,
                          group_attention: bool | None = None) -> int:
    """Patch supported PEFT LoRA Linear modules for inference (peft_integration.py:414-448).

    ``group_attention`` (default: the ``LORAFORGE_GROUPED_ATTN`` environment
    variable, off) additionally packs each attention block's q, k and v
    projections into one linear that reads x once (``_patch_grouped_siblings``);
    the reference has no such grouping.
    """
    count = 0
    for module in model.modules():
        if is_lora_linear(module) and not hasattr(module, "_loraforge_original_forward"):
            if cast_adapter_dtype and isinstance(module.base_layer, torch.nn.Linear):
                target_dtype = module.base_layer.weight.dtype
                if target_dtype in (torch.float16, torch.bfloat16):
                    for name in module.active_adapters:
                        if name in module.lora_A and name in module.lora_B:
                            module.lora_A[name].to(dtype=target_dtype)
                            module.lora_B[name].to(dtype=target_dtype)
            module._loraforge_original_forward = module.forward
            module._loraforge_plan = None
            module._loraforge_plans = {}
            module.forward = types.MethodType(_loraforge_linear_forward, module)
            count += 1
    grouped = 0
    if enable_grouping and os.environ.get("LORAFORGE_GROUPED_MLP", "").strip().lower() != "individual":
        for module in model.modules():
            if _patch_grouped_mlp(module):
                grouped += 1
    model._loraforge_grouped_mlp_count = grouped
    if group_attention is None:
        group_attention = os.environ.get("LORAFORGE_GROUPED_ATTN", "").strip().lower() in ("1", "true", "yes")
    grouped_attn = 0
    if group_attention:
        for module in model.modules():
            if _patch_grouped_siblings(module, ATTENTION_GROUP, "attention"):
                grouped_attn += 1
    model._loraforge_grouped_attention_count = grouped_attn
    return count


def peft_plan_report(model) -> dict:
    """Summarize selected implementations (peft_integration.py:451-479)."""
    choices = Counter()
    timing_samples = []
    grouped_choices = Counter()
    grouped_timing_samples = []
    for module in model.modules():
        choice = module.__dict__.get("_loraforge_decode_choice")
        if choice is not None:
            choices[choice] += 1
            timing_samples.append({"choice": choice,
                                   "timings_us": module.__dict__.get("_loraforge_decode_timings_us", {})})
        for rows, grouped_choice in module.__dict__.get("_loraforge_grouped_choices", {}).items():
            grouped_choices[grouped_choice] += 1
            grouped_timing_samples.append({"rows": rows, "choice": grouped_choice, "timings_us": {}})
    return {
        "decode_choices": dict(choices),
        "grouped_mlp_modules": getattr(model, "_loraforge_grouped_mlp_count", 0),
        "grouped_attention_modules": getattr(model, "_loraforge_grouped_attention_count", 0),
        "decode_timing_samples": timing_samples,
        "grouped_mlp_choices": dict(grouped_choices),
        "grouped_mlp_timing_samples": grouped_timing_samples,
    }
