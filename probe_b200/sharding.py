"""Token / request sharding of the LoRA linear across the GPUs of one node.

The LoRA linear has no cross-token coupling: rows of x are independent, so the
work splits into contiguous token ranges (single adapter) or into groups of
whole request segments (multi-adapter), with W and every adapter replicated on
each GPU.  No data-path collective is needed.  The only exchange is optional:
``gather_rows`` all-gathers the per-rank outputs into one ``[M, N]`` tensor for
a caller that wants them on every rank (NCCL over NVLink on GPUs; any
torch.distributed backend works, which is how the host logic is tested on CPU
with gloo).

One process per GPU; ranks follow torch.distributed's RANK / WORLD_SIZE.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous token range [start, stop) of ``rank``; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_segments(seg_start, world: int) -> list[tuple[int, int]]:
    """Split S segments (boundaries ``seg_start[0..S]``) into ``world`` contiguous
    groups of whole segments with balanced token counts.

    Returns per-rank segment index ranges [s0, s1).  Each group's token range is
    [seg_start[s0], seg_start[s1]).  A rank may receive no segment when there
    are fewer segments than ranks.
    """
    bounds = [int(v) for v in seg_start]
    s = len(bounds) - 1
    total = bounds[-1] - bounds[0]
    out = []
    s0 = 0
    for r in range(world):
        if r == world - 1:
            out.append((s0, s))
            break
        target = bounds[0] + (total * (r + 1)) // world
        s1 = s0
        # advance while the next boundary is closer to the target than the current one
        while s1 < s and abs(bounds[s1 + 1] - target) <= abs(bounds[s1] - target):
            s1 += 1
        out.append((s0, s1))
        s0 = s1
    return out


def local_segments(seg_start: torch.Tensor, seg_adapter: torch.Tensor, world: int, rank: int):
    """This rank's segment table, rebased so its first token is row 0.

    Returns (token_start, token_stop, seg_start_local [S_r+1], seg_adapter_local [S_r]).
    """
    groups = shard_segments(seg_start.tolist(), world)
    s0, s1 = groups[rank]
    t0, t1 = int(seg_start[s0]), int(seg_start[s1])
    return t0, t1, (seg_start[s0:s1 + 1] - t0).contiguous(), seg_adapter[s0:s1].contiguous()


def gather_rows(local: torch.Tensor, total_rows: int, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather row shards (``shard_rows`` layout) into a full ``[total_rows, ...]`` tensor.

    One ``all_gather_into_tensor`` (NCCL over NVLink on GPUs).  When every rank
    holds the same number of rows the ranks' shards land directly in their
    places of the result (``out`` if given); otherwise shorter shards are padded
    by one row for the collective and the result is compacted by one gather of
    rows.
    """
    world = dist.get_world_size(group)
    sizes = [shard_rows(total_rows, world, r) for r in range(world)]
    width = max(b - a for a, b in sizes)
    tail = tuple(local.shape[1:])
    if local.shape[0] != sizes[dist.get_rank(group)][1] - sizes[dist.get_rank(group)][0]:
        raise ValueError(f"gather_rows: this rank holds {local.shape[0]} rows, its shard of {total_rows} is "
                         f"{sizes[dist.get_rank(group)]}")
    if width * world == total_rows:
        if out is None:
            out = local.new_empty((total_rows,) + tail)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    padded = local.new_zeros((width,) + tail)
    padded[: local.shape[0]] = local
    stacked = local.new_empty((width * world,) + tail)
    dist.all_gather_into_tensor(stacked, padded, group=group)
    keep = torch.cat([torch.arange(r * width, r * width + (b - a)) for r, (a, b) in enumerate(sizes)])
    rows = stacked.index_select(0, keep.to(stacked.device))
    if out is not None:
        out.copy_(rows)
        return out
    return rows


class ShardedLoRALinear(torch.nn.Module):
    """Run a (Fused)LoRA linear on this rank's share of the tokens.

    ``forward(x_full)`` slices the local rows of a full batch (when every rank
    holds the batch) and returns the local output; ``gather=True`` also
    all-gathers the full output.  ``forward_local`` takes an already-local
    shard.
    """

    def __init__(self, inner: torch.nn.Module, group=None):
        super().__init__()
        self.inner = inner
        self.group = group

    def forward(self, x: torch.Tensor, gather: bool = False) -> torch.Tensor:
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        rows = x.reshape(-1, x.shape[-1])
        a, b = shard_rows(rows.shape[0], world, rank)
        out = self.inner(rows[a:b])
        if gather and world > 1:
            return gather_rows(out, rows.shape[0], self.group).reshape(*x.shape[:-1], -1)
        return out

    def forward_local(self, x_local: torch.Tensor) -> torch.Tensor:
        return self.inner(x_local)
