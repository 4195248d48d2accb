"""Batched multi-adapter LoRA (BGMV / ragged / rank-bucketed).

Drop-in for ``loraforge_kernels.multilora`` (multilora.py:32-377).  Every entry
point runs the segmented B200 kernels: a device-built tile list groups
consecutive tokens that share an adapter (so an adapter's rows are fetched once
per 64 tokens, not once per token), the shrink is split-K with a deterministic
in-kernel reduction (the reference pre-zeroes an fp32 buffer and uses
atomics), and the expand is a tensor-core tile that reads each adapter's B once
per tile.  Outputs match the reference: fp32 ``z`` padded with zeros beyond
each token's rank, and fresh ``out`` tensors.
"""

from __future__ import annotations

import functools

import torch

from . import kernels
from .fused_linear import next_power_of_2


def rank_tile(r: int) -> int:
    """Next power of two, at least 16 (multilora.py:32-33)."""
    return max(16, next_power_of_2(r))


def auto_split_k(n_tokens: int, target_programs: int = 2048, cap: int = 64) -> int:
    """Split of K that keeps the machine busy for n_tokens (multilora.py:36-48)."""
    if n_tokens <= 0:
        return 1
    return max(1, min(cap, next_power_of_2(max(1, target_programs // n_tokens))))


@functools.lru_cache(maxsize=256)
def _padded_tables(n: int, r: int, device_index: int):
    dev = torch.device("cuda", device_index)
    offsets = torch.arange(n, dtype=torch.int64, device=dev) * r
    ranks = torch.full((n,), r, dtype=torch.int64, device=dev)
    return offsets, ranks


def _dev_index(t: torch.Tensor) -> int:
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def shrink_padded(x, a_stack, idx, split_k=None, bk=128):
    """z[t] = x[t] @ A[idx[t]].T with every adapter padded to r (multilora.py:91-104)."""
    t, k = x.shape
    n, r, _ = a_stack.shape
    offsets, ranks = _padded_tables(n, r, _dev_index(x))
    tiles, s = kernels.sgmv_schedule(t, n, ids=idx)
    return kernels.sgmv_shrink(x, a_stack.reshape(n * r, k), offsets, ranks, tiles, s, r,
                               z_dtype=torch.float32, split_k=0 if split_k is None else split_k)


def shrink_grouped(x, groups, idx, split_k=8, bk=128):
    """One call per distinct rank on the gathered tokens (multilora.py:107-125).

    ``groups`` maps rank -> (a_stack [n_r, rank, K], token positions, local index);
    returns rank -> (z [len(positions), rank] fp32, positions).
    """
    outs = {}
    for rank, (a_stack, positions, local_idx) in groups.items():
        xs = x[positions]
        outs[rank] = (shrink_padded(xs, a_stack, local_idx, split_k=split_k), positions)
    return outs


def shrink_ragged(x, a_flat, offsets, ranks, idx, r_max, split_k=8, bk=128):
    """Rank-aware shrink over a flat [sum r, K] table (multilora.py:171-182)."""
    t, k = x.shape
    tiles, s = kernels.sgmv_schedule(t, offsets.numel(), ids=idx)
    return kernels.sgmv_shrink(x, a_flat, offsets, ranks, tiles, s, r_max, z_dtype=torch.float32,
                               split_k=split_k)


def _bucket_shrink(x, z, rank, a_stack, pos, local, split_k):
    n_r = a_stack.shape[0]
    npos = pos.shape[0]
    offsets, ranks = _padded_tables(n_r, rank, _dev_index(x))
    tiles, s = kernels.sgmv_schedule(npos, n_r, ids=local)
    kernels.sgmv_shrink(x, a_stack.reshape(n_r * rank, x.shape[1]), offsets, ranks, tiles, s, rank,
                        z_width=rank, split_k=split_k or 0, rows=pos, t_total=npos, out=z)


def shrink_bucketed(x, buckets, r_max, split_k=None, bk=128):
    """One call per distinct rank, tokens addressed through ``pos`` (multilora.py:229-250)."""
    t = x.shape[0]
    out = torch.zeros((t, r_max), device=x.device, dtype=torch.float32)
    for rank, (a_stack, pos, local) in buckets.items():
        if pos.shape[0] == 0:
            continue
        _bucket_shrink(x, out, rank, a_stack, pos, local, split_k)
    return out


def shrink_bucketed_parallel(x, buckets, r_max, streams, events, split_k=1, bk=128):
    """Rank buckets on concurrent streams (multilora.py:253-292)."""
    t = x.shape[0]
    out = torch.zeros((t, r_max), device=x.device, dtype=torch.float32)
    main = torch.cuda.current_stream()
    fork = events[0]
    fork.record(main)
    used = []
    for i, (rank, (a_stack, pos, local)) in enumerate(buckets.items()):
        if pos.shape[0] == 0:
            continue
        stream = streams[i % len(streams)]
        stream.wait_event(fork)
        with torch.cuda.stream(stream):
            _bucket_shrink(x, out, rank, a_stack, pos, local, split_k)
        done = events[i + 1]
        done.record(stream)
        used.append(done)
    for done in used:
        main.wait_event(done)
    return out


def expand_padded(y, z, b_stack, idx, scale=1.0, bn=128):
    """out[t] = y[t] + scale * z[t, :r] @ B[idx[t]].T, B stack [n, N, r] (multilora.py:334-347)."""
    t, n = y.shape
    na, _, r = b_stack.shape
    offsets, ranks = _padded_tables(na, r, _dev_index(y))
    tiles, s = kernels.sgmv_schedule(t, na, ids=idx)
    return kernels.sgmv_expand(y, z, b_stack, 1, r, offsets, ranks, tiles, s, n, r, scale=scale)


def expand_bucketed_parallel(y, z, buckets_b, streams, events, scale=1.0, bn=128):
    """Rank buckets of the expand on concurrent streams (multilora.py:350-377)."""
    t, n = y.shape
    out = torch.empty_like(y)
    main = torch.cuda.current_stream()
    fork = events[0]
    fork.record(main)
    used = []
    for i, (rank, (b_stack, pos, local)) in enumerate(buckets_b.items()):
        npos = pos.shape[0]
        if npos == 0:
            continue
        stream = streams[i % len(streams)]
        stream.wait_event(fork)
        with torch.cuda.stream(stream):
            n_r = b_stack.shape[0]
            offsets, ranks = _padded_tables(n_r, rank, _dev_index(y))
            tiles, s = kernels.sgmv_schedule(npos, n_r, ids=local)
            kernels.sgmv_expand(y, z, b_stack, 1, rank, offsets, ranks, tiles, s, n, rank, scale=scale,
                                rows=pos, t_total=npos, out=out)
        done = events[i + 1]
        done.record(stream)
        used.append(done)
    for done in used:
        main.wait_event(done)
    return out
