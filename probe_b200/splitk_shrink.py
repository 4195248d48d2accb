"""Split-K shrink ``x[M, K] @ A[r, K].T`` (drop-in for ``loraforge_kernels.splitk_shrink``).

The reference offers two reductions of the split-K partials: a partial buffer
plus a second pass (``shrink_partial``) or fp32 atomics into a zeroed buffer
(``shrink_atomic``), splitk_shrink.py:116-141.  The B200 kernel does neither:
the last CTA of each token tile sums the partials in split order, in the same
launch.  Both names call it; the tile-shape arguments are accepted for
compatibility and do not change the result.
"""

from __future__ import annotations

from . import kernels
from .fused_linear import next_power_of_2


def rank_tile(r: int) -> int:
    """Tensor-core tile width for rank r: next power of two, at least 16 (splitk_shrink.py:30-32)."""
    return max(16, next_power_of_2(r))


def shrink_partial(x, a, split_k=4, bm=16, bk=128, num_warps=4):
    """``x @ a.T`` in x's dtype (splitk_shrink.py:116-127)."""
    return kernels.shrink(x, a, 1.0, z_dtype=x.dtype, split_k=split_k)


def shrink_atomic(x, a, split_k=4, bm=16, bk=128, num_warps=4):
    """``x @ a.T`` in x's dtype (splitk_shrink.py:130-141); deterministic here."""
    return kernels.shrink(x, a, 1.0, z_dtype=x.dtype, split_k=split_k)
