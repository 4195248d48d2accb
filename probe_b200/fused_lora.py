"""Decode-style LoRA sidecar ``out = y + scale * (x @ A.T) @ B.T``.

Drop-in for ``loraforge_kernels.fused_lora`` (fused_lora.py:203-311): same
names, arguments and assertions.  Every variant -- row, output-tiled,
execution-class and grouped -- runs the same two B200 kernels: the split-K
shrink (z kept in fp32, as the reference's row kernels keep it in registers)
followed by the tensor-core expand-add.  The reference's distinct Triton
geometries existed to fill a GH200 at small M; the split-K shrink already
spreads K over every SM, so one implementation serves all four entry points.
"""

from __future__ import annotations

import torch

from . import kernels
from .fused_linear import next_power_of_2


def _sidecar(x, a, b, y, scale, rank=None):
    z = kernels.shrink(x, a if rank is None else a[:rank], 1.0, z_dtype=torch.float32)
    return kernels.expand_add(y, z, b if rank is None else b[:, :rank], scale, dtype=x.dtype)


def fused_lora(x: torch.Tensor, a: torch.Tensor, b: torch.Tensor, y=None, scale=1.0):
    """Row kernel semantics (fused_lora.py:203-218): r <= 64, fresh output."""
    m, k = x.shape
    r, ka = a.shape
    n, rb = b.shape
    assert ka == k and rb == r and r <= 64 and x.is_cuda
    return _sidecar(x, a, b, y, scale)


def tiled_lora(x: torch.Tensor, a: torch.Tensor, b: torch.Tensor, y=None, scale=1.0):
    """Output-tiled decode kernel semantics (fused_lora.py:221-238)."""
    m, k = x.shape
    r, ka = a.shape
    n, rb = b.shape
    assert ka == k and rb == r and r <= 64 and x.is_cuda
    return _sidecar(x, a, b, y, scale)


def _validate_execution_class(r: int, execution_rank: int | None) -> int:
    """Execution class: a power of two covering r, at most 64 (fused_lora.py:241-245)."""
    execution_rank = next_power_of_2(r) if execution_rank is None else execution_rank
    assert r <= execution_rank <= 64
    assert execution_rank & (execution_rank - 1) == 0
    return execution_rank


def classed_lora(x, a, b, y=None, scale=1.0, execution_rank: int | None = None):
    """Compact storage mapped to a shared execution class (fused_lora.py:248-268)."""
    m, k = x.shape
    r, ka = a.shape
    n, rb = b.shape
    assert ka == k and rb == r and x.is_cuda
    _validate_execution_class(r, execution_rank)
    return _sidecar(x, a, b, y, scale)


def classed_tiled_lora(x, a, b, y=None, scale=1.0, execution_rank: int | None = None):
    """Output-tiled counterpart of :func:`classed_lora` (fused_lora.py:271-292)."""
    m, k = x.shape
    r, ka = a.shape
    n, rb = b.shape
    assert ka == k and rb == r and x.is_cuda
    _validate_execution_class(r, execution_rank)
    return _sidecar(x, a, b, y, scale)


def grouped_lora(x: torch.Tensor, a: torch.Tensor, b: torch.Tensor, y=None, scale=1.0):
    """P projections sharing one x pass: a [P*R,K], b [P,N,R], y/out [M,P,N] (fused_lora.py:295-311).

    One shrink reads x once for all P projections' ranks; each projection's
    expand then reads its own slice of z.
    """
    m, k = x.shape
    p, n, r = b.shape
    assert a.shape == (p * r, k) and p * r <= 128 and x.is_cuda
    out = torch.empty((m, p, n), device=x.device, dtype=x.dtype)
    z = kernels.shrink(x, a, 1.0, z_dtype=torch.float32)
    for i in range(p):
        yi = None if y is None else y[:, i, :]
        kernels.expand_add(yi, z[:, i * r: (i + 1) * r], b[i], scale, out=out[:, i, :], dtype=x.dtype)
    return out
