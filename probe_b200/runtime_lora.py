"""Runtime (unmerged) LoRA on plain ``nn.Linear`` layers, served by the fused kernels.

Drop-in for ``loraforge_kernels.runtime_lora`` (runtime_lora.py:1-69):
``attach_fused_lora`` replaces the ``nn.Linear`` found at a dotted path with a
:class:`FusedLoRALinear` that keeps the base weight untouched and runs the
adapter inside the base GEMM.  Attaching again at the same path adds the new
adapter to the stack.

Stacking algebra.  A layer carrying adapters (A_i, B_i, alpha_i) computes
``x W^T + sum_i alpha_i (x A_i^T) B_i^T``.  The fused layer holds one scale s
(the first adapter's alpha) and one pair of factors, so the i-th adapter
enters as the rank block ``A_i * (alpha_i / s)`` of the down factor and the
column block ``B_i`` of the up factor: ``s [A_1; (a_2/s) A_2] ... `` times
``[B_1 | B_2]`` reproduces the sum exactly, and the kernels see one adapter of
the summed rank.  The ratio is applied in fp32 and the result rounded once to
the layer's dtype, which is the reference's rounding (runtime_lora.py:49-53).
"""

from __future__ import annotations

import torch
from torch import nn

from .fused_linear import FusedLoRALinear


def resolve_parent(root: nn.Module, dotted_path: str) -> tuple[nn.Module, str]:
    """The module that owns the last component of ``dotted_path``, and that component's name."""
    owner_path, _, leaf = dotted_path.rpartition(".")
    owner = root
    for step in owner_path.split(".") if owner_path else ():
        owner = getattr(owner, step)
    return owner, leaf


def _with_extra_adapter(layer: FusedLoRALinear, down: torch.Tensor, up: torch.Tensor, alpha: float):
    """``layer``'s factors with one more adapter appended as a new rank block."""
    device, dtype = layer.weight.device, layer.weight.dtype
    ratio = float(alpha) / layer.scale
    down_block = (down.detach().to(device=device, dtype=torch.float32) * ratio).to(dtype)
    up_block = up.detach().to(device=device, dtype=dtype)
    return torch.cat((layer.lora_a, down_block), dim=0), torch.cat((layer.lora_b, up_block), dim=1)


def attach_fused_lora(root: nn.Module, dotted_path: str, down: torch.Tensor, up: torch.Tensor,
                      alpha: float = 1.0) -> FusedLoRALinear:
    """Serve the ``nn.Linear`` at ``dotted_path`` with a fused LoRA sidecar (runtime_lora.py:29-61).

    ``down`` is lora_A.weight ``[r, in]``, ``up`` is lora_B.weight ``[out, r]``
    and ``alpha`` the adapter's scale.  A path that already holds a fused layer
    gets the adapter stacked onto it; anything other than an ``nn.Linear`` is
    refused with ``TypeError``.  Returns the fused layer.
    """
    owner, leaf = resolve_parent(root, dotted_path)
    current = getattr(owner, leaf)
    if isinstance(current, FusedLoRALinear):
        current.set_factors(*_with_extra_adapter(current, down, up, alpha))
        return current
    if not isinstance(current, nn.Linear):
        raise TypeError(f"LoRA target {dotted_path} is {type(current).__name__}, not nn.Linear")
    replacement = FusedLoRALinear(current, down, up, scale=alpha)
    setattr(owner, leaf, replacement)
    return replacement


def _fused_layers(root: nn.Module):
    return [m for m in root.modules() if isinstance(m, FusedLoRALinear)]


def fused_lora_module_count(root: nn.Module) -> int:
    """How many fused LoRA layers ``root`` contains."""
    return len(_fused_layers(root))


def total_fused_rank(root: nn.Module) -> int:
    """Sum of the (stacked) ranks of every fused LoRA layer under ``root``."""
    return sum(layer.rank for layer in _fused_layers(root))
