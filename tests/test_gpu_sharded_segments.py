"""Segment-sharded multi-adapter batches (GPU, one device standing in for the
ranks): C3's batch split into 2, 4 and 8 groups of whole segments
(``sharding.local_segments``), each group run through the segmented branch and
the fused segmented linear on its own rebased tables, the groups' outputs
concatenated.

Checked: the groups cover the batch exactly once; every group's device tile
schedule equals the oracle's (routing bit-exact per shard); the concatenated
outputs pass the float64 oracle on sampled tokens; and they agree with the
unsharded call to within the summation-order difference of the K-split
partials (a shard's K-slice count follows its own token count).
"""

import pytest
import torch

from oracle import checks
from oracle import lora_oracle as orc
from probe_b200 import _lib, kernels, segmented_branch, workloads
from probe_b200.sharding import local_segments

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _schedule_matches(t, n_adapters, ss, sa):
    """The device tile list of a shard equals the oracle's (starts and adapters)."""
    tiles, _ = kernels.sgmv_schedule(t, n_adapters, seg_start=ss, seg_adapter=sa)
    n, mt = int(tiles[0]), int(tiles[1])
    want_s, want_a = orc.tile_schedule(seg_start=ss.tolist(), seg_adapter=sa.tolist(), n_adapters=n_adapters)
    return tiles[2:3 + n].tolist() == want_s and tiles[3 + mt:3 + mt + n].tolist() == want_a


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_segments_match_oracle_and_unsharded(world):
    c = workloads.c3(device=DEV, dtype=torch.bfloat16)
    tabs = (c.a_flat, c.b_flat, c.offsets, c.ranks)
    y = kernels.gemm(c.x, c.w)
    full_branch = segmented_branch.segmented_branch_varlen(c.x, y, *tabs, c.seg_start, c.seg_adapter, c.r_max)
    full_linear = segmented_branch.segmented_linear_varlen(c.x, c.w, None, *tabs, c.seg_start, c.seg_adapter,
                                                           c.r_max)
    parts_b, parts_l, covered = [], [], 0
    for rank in range(world):
        t0, t1, ss, sa = local_segments(c.seg_start, c.seg_adapter, world, rank)
        assert t0 == covered  # contiguous, whole segments
        covered = t1
        if t1 == t0:
            continue
        xs, ys = c.x[t0:t1], y[t0:t1]
        assert _schedule_matches(t1 - t0, c.offsets.numel(), ss, sa)
        parts_b.append(segmented_branch.segmented_branch_varlen(xs, ys, *tabs, ss, sa, c.r_max))
        parts_l.append(segmented_branch.segmented_linear_varlen(xs, c.w, None, *tabs, ss, sa, c.r_max))
    assert covered == c.x.shape[0]
    got_b, got_l = torch.cat(parts_b), torch.cat(parts_l)
    ids = c.token_ids()
    rep = checks.branch_report(got_b, c.x, y, c.a_flat, c.b_flat, c.offsets, c.ranks, ids, n_random=64)
    assert rep["ok"], rep
    rep = checks.seg_linear_report(got_l, c.x, c.w, None, c.a_flat, c.b_flat, c.offsets, c.ranks, ids, n_random=64)
    assert rep["ok"], rep
    for got, full in ((got_b, full_branch), (got_l, full_linear)):
        diff = (got.float() - full.float()).abs()
        ulp = torch.exp2(torch.floor(torch.log2(full.float().abs().clamp_min(1e-30))) - 7)
        assert bool((diff <= ulp + 1e-3).all()), float(diff.max())  # one bf16 rounding apart at most
    assert _lib.device_error() == 0
