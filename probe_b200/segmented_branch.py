"""Tensor-core LoRA for contiguous token segments, one adapter per segment.

Drop-in for ``loraforge_kernels.segmented_branch`` (segmented_branch.py:50-60):
``A_flat [sum r, K]`` and a rank-major ``B_flat [sum r, N]`` with each adapter's
scale already folded into B; ``offsets`` / ``ranks`` / ``request_ids`` are device
int64 tensors, so no host synchronisation happens.

The reference requires equal-length segments (``ValueError`` otherwise);
that contract is kept for ``segmented_branch``.  ``segmented_branch_varlen``
takes arbitrary segment boundaries (e.g. Zipf-distributed request lengths):
the device tile list splits every segment into <= 64-token tiles.
``segmented_linear_varlen`` (no reference counterpart) adds the base linear:
the base GEMM and the adapters in one tensor-core GEMM, so the branch costs no
extra pass over the output.
"""

from __future__ import annotations

import torch

from . import kernels


def segmented_branch(x, y, a, b, offsets, ranks, request_ids, tokens_per_request, rmax, split_k=4):
    """out = y + per-request (x @ A_a.T) @ B_a for uniform request segments."""
    if rmax == 0:
        return y
    x = x.contiguous()
    y = y.contiguous()
    total, k = x.shape
    n = y.shape[1]
    requests = request_ids.numel()
    if total != requests * tokens_per_request:
        raise ValueError("Invalid contiguous request segments")
    seg_start = torch.arange(requests + 1, device=x.device, dtype=torch.int64) * tokens_per_request
    return segmented_branch_varlen(x, y, a, b, offsets, ranks, seg_start, request_ids, rmax, split_k=split_k)


def segmented_branch_varlen(x, y, a, b, offsets, ranks, seg_start, seg_adapter, rmax, split_k=0):
    """out = y + (x[s] @ A_a.T) @ B_a for segments ``[seg_start[i], seg_start[i+1])``.

    ``seg_start`` has S+1 entries (0 ... T), ``seg_adapter`` S adapter ids.
    """
    if rmax == 0:
        return y
    x = x.contiguous()
    y = y.contiguous()
    total, k = x.shape
    n = y.shape[1]
    tiles, s = kernels.sgmv_schedule(total, offsets.numel(), seg_start=seg_start, seg_adapter=seg_adapter)
    out = kernels.sgmv_branch(x, y, a, b, offsets, ranks, tiles, s, rmax)
    if out is not None:
        return out
    # ranks above 64 or unaligned rows: shrink then expand
    z = kernels.sgmv_shrink(x, a, offsets, ranks, tiles, s, rmax, z_dtype=torch.float32,
                            split_k=split_k if split_k and split_k > 0 else 0)
    return kernels.sgmv_expand(y, z, b, n, 1, offsets, ranks, tiles, s, n, rmax)


def segmented_linear_varlen(x, weight, bias, a, b, offsets, ranks, seg_start, seg_adapter, rmax):
    """out = x @ weight.T + bias + (x[s] @ A_a.T) @ B_a for segments ``[seg_start[i], seg_start[i+1])``.

    The base linear of the layer and its segmented adapters in one GEMM: each
    256-token output tile runs the base K blocks and then one block per adapter
    piece of the tile (lora_sgmv_linear).  Shapes outside that kernel (rmax > 64,
    K or N not a multiple of 64) run the base GEMM, then the branch.
    """
    x = x.contiguous()
    if rmax == 0:
        return kernels.gemm(x, weight, bias=bias)
    total = x.shape[0]
    tiles, s = kernels.sgmv_schedule(total, offsets.numel(), seg_start=seg_start, seg_adapter=seg_adapter)
    out = kernels.sgmv_linear(x, weight, bias, a, b, offsets, ranks, tiles, s, rmax)
    if out is not None:
        return out
    y = kernels.gemm(x, weight, bias=bias)
    return segmented_branch_varlen(x, y, a, b, offsets, ranks, seg_start, seg_adapter, rmax)
