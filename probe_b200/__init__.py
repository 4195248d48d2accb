"""probe_b200 -- B200-native (sm_100a) LoRA-linear kernels.

A drop-in for the ``loraforge_kernels`` package of lishenghui/probe: the same
public names (``__init__.py:1-71`` there), backed by hand-written CUDA for
Blackwell behind the C ABI in ``include/lora_b200.h``.  The PEFT bridge is
resolved lazily, as in the reference.
"""

from .fused_linear import (
    FUSED_MAX_RANK,
    MIN_GEMM_ROWS,
    FusedLoRALinear,
    augment_bias,
    augment_weight,
    build_ext,
    build_plan,
    expand_add,
    fused_gemm,
    fused_lora_linear,
    kconcat_weight,
    packed_rank,
    pad_rank,
    selection_report,
)
from .fused_lora import classed_lora, classed_tiled_lora, fused_lora, grouped_lora, tiled_lora
from .overlapped_linear import DualStreamOverlappedLinear
from .runtime_lora import attach_fused_lora, fused_lora_module_count, total_fused_rank
from .splitk_lora import (
    DEPLOY_RANK_BUCKETS,
    align_to_deploy_rank,
    persistent_expand_add,
    splitk_lora_shrink,
    splitk_persistent_fused_lora,
)

__all__ = [
    "fused_lora",
    "grouped_lora",
    "tiled_lora",
    "classed_lora",
    "classed_tiled_lora",
    "fused_lora_linear",
    "fused_gemm",
    "FusedLoRALinear",
    "expand_add",
    "augment_weight",
    "augment_bias",
    "kconcat_weight",
    "build_ext",
    "build_plan",
    "selection_report",
    "pad_rank",
    "packed_rank",
    "FUSED_MAX_RANK",
    "MIN_GEMM_ROWS",
    "attach_fused_lora",
    "fused_lora_module_count",
    "total_fused_rank",
    "enable_loraforge_peft",
    "peft_plan_report",
    "splitk_lora_shrink",
    "persistent_expand_add",
    "splitk_persistent_fused_lora",
    "align_to_deploy_rank",
    "DEPLOY_RANK_BUCKETS",
    "DualStreamOverlappedLinear",
]


def __getattr__(name):
    """Resolve the PEFT bridge lazily, as the reference does."""
    if name in ("enable_loraforge_peft", "peft_plan_report"):
        from . import peft_integration

        return getattr(peft_integration, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
