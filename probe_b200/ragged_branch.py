"""Compact multi-LoRA branch with per-token adapter ids and rank-0 skip.

Drop-in for ``loraforge_kernels.ragged_branch`` (ragged_branch.py:30-40):
``A [sum ranks, K]``, ``B [sum ranks, N]`` with the adapter scale folded into B,
int64 device ``offsets`` / ``ranks`` / ``indices``.  Consecutive tokens with the
same id are grouped into tiles on the device, so a run of one request's tokens
reads its adapter once per 64 tokens.  ``linear`` (no reference counterpart)
fuses the layer's base linear with the branch in one tensor-core GEMM.
"""

from __future__ import annotations

import torch

from . import kernels


def branch(x, y, a, b, offsets, ranks, indices, rmax, skip_zero=True, split_k=8):
    """out = y + (x[t] @ A_{i(t)}.T) @ B_{i(t)} for every token t."""
    if rmax == 0:
        return y
    x = x.contiguous()
    y = y.contiguous()
    t, k = x.shape
    n = y.shape[1]
    tiles, s = kernels.sgmv_schedule(t, offsets.numel(), ids=indices)
    out = kernels.sgmv_branch(x, y, a, b, offsets, ranks, tiles, s, rmax)
    if out is not None:
        return out
    # ranks above 64 or unaligned rows: shrink then expand
    z = kernels.sgmv_shrink(x, a, offsets, ranks, tiles, s, rmax, z_dtype=torch.float32, split_k=split_k)
    return kernels.sgmv_expand(y, z, b, n, 1, offsets, ranks, tiles, s, n, rmax)


def linear(x, weight, bias, a, b, offsets, ranks, indices, rmax):
    """out = x @ weight.T + bias + (x[t] @ A_{i(t)}.T) @ B_{i(t)} for every token t, in one GEMM
    (adapters as a per-256-token-tile K tail; rank-0 and unknown ids add nothing).

    Best for runs of tokens sharing an id (requests): every run inside a
    256-token tile adds one k-block to that tile.  Shapes outside the fused
    kernel run the base GEMM, then ``branch``."""
    x = x.contiguous()
    if rmax == 0:
        return kernels.gemm(x, weight, bias=bias)
    t = x.shape[0]
    tiles, s = kernels.sgmv_schedule(t, offsets.numel(), ids=indices)
    out = kernels.sgmv_linear(x, weight, bias, a, b, offsets, ranks, tiles, s, rmax)
    if out is not None:
        return out
    return branch(x, kernels.gemm(x, weight, bias=bias), a, b, offsets, ranks, indices, rmax)
