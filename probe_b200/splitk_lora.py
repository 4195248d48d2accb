"""Split-K shrink and persistent expand for small-batch decode.

Drop-in for ``loraforge_kernels.splitk_lora`` (splitk_lora.py:10-159).  The
reference writes fp32 partials ``[M, SPLIT_K, R]`` and reduces them with a
second (torch) launch; here the split-K kernel reduces its own partials in a
fixed order (last CTA per tile), so the shrink is one launch and deterministic.
"""

from __future__ import annotations

import torch

from . import kernels
from .fused_linear import next_power_of_2

# Hardware-aligned rank bucket choices for GPU deployment (splitk_lora.py:11).
DEPLOY_RANK_BUCKETS = (8, 16, 24, 32, 48, 64)


def align_to_deploy_rank(r: int) -> int:
    """Smallest deploy bucket >= r, else the next power of two (splitk_lora.py:14-19)."""
    for bucket in DEPLOY_RANK_BUCKETS:
        if r <= bucket:
            return bucket
    return next_power_of_2(r)


def splitk_lora_shrink(x: torch.Tensor, a: torch.Tensor, split_k: int = 8) -> torch.Tensor:
    """``x [M, K] @ a [R, K].T -> z [M, R]`` in x's dtype (splitk_lora.py:104-126)."""
    m, k = x.shape
    r, ka = a.shape
    assert ka == k and x.is_cuda and a.is_cuda
    return kernels.shrink(x, a, 1.0, z_dtype=x.dtype, split_k=split_k)


def persistent_expand_add(z: torch.Tensor, b: torch.Tensor, y: torch.Tensor | None = None,
                          scale: float = 1.0) -> torch.Tensor:
    """``z [M, R] @ b [N, R].T * scale + y [M, N]`` -> fresh out in z's dtype (splitk_lora.py:129-153)."""
    m, r = z.shape
    n, rb = b.shape
    assert rb == r and z.is_cuda and b.is_cuda
    return kernels.expand_add(y, z, b, scale, dtype=z.dtype)


def splitk_persistent_fused_lora(x: torch.Tensor, a: torch.Tensor, b: torch.Tensor, y: torch.Tensor | None = None,
                                 scale: float = 1.0, split_k: int = 8) -> torch.Tensor:
    """Shrink then expand-add (splitk_lora.py:156-159)."""
    z = splitk_lora_shrink(x, a, split_k=split_k)
    return persistent_expand_add(z, b, y=y, scale=scale)
