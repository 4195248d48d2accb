"""Unit-scheduled segmented shrink and branch (GPU): (tile, K slice) units over
persistent CTAs in a cost-sorted snake order (schedule order past 1024 tiles),
partials summed in slice order.

Cases reach its edges: one-token tiles (random per-token ids), a last tile cut
by T, K not a multiple of 64, ranks 1..128 (stage layouts for r_max <= 64 and
> 64), rank-0 adapters, many slices, fp32 and bf16 z; results against the
float64 oracle and bit-identical across repeated calls (the reduction order
is fixed).
"""

import math

import numpy as np
import pytest
import torch

from oracle import lora_oracle as orc
from probe_b200 import _lib, kernels
from tests.helpers import np64, randn

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tables(ranks, k, seed):
    g = torch.Generator().manual_seed(seed)
    rk = torch.tensor(ranks, dtype=torch.int64)
    offs = torch.zeros_like(rk)
    offs[1:] = torch.cumsum(rk, 0)[:-1]
    a = (torch.randn(max(int(rk.sum()), 1), k, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    return a.to(DEV), offs.to(DEV), rk.to(DEV)


def _run(x, a, offs, rk, ids, r_max, split_k, z_dtype=torch.float32, scale=0.7):
    t = x.shape[0]
    tiles, s = kernels.sgmv_schedule(t, offs.numel(), ids=torch.as_tensor(ids, device=DEV))
    return kernels.sgmv_shrink(x, a, offs, rk, tiles, s, r_max, scale=scale, z_dtype=z_dtype, split_k=split_k)


@pytest.mark.parametrize("t,k,ranks,mode,split_k", [
    (1000, 4096, [4, 8, 16, 32, 64], "random", 8),       # one-token tiles everywhere
    (777, 520, [64, 13, 0, 33], "runs", 3),              # K % 64 != 0, rank 0, last tile cut by T
    (300, 1024, [128, 96, 1, 127], "runs", 16),          # r_max > 64: wider stages
    (64, 2048, [16], "runs", 2),                         # one tile
    (3000, 512, [4, 8, 16, 32, 64], "random", 0),        # > 1024 tiles: units in schedule order, no sort
    (4096, 4096, [4, 8, 16, 32, 64] * 12 + [8] * 4, "zipf", 0),  # C3-like, default split
])
def test_unit_shrink_matches_oracle(t, k, ranks, mode, split_k):
    rng = np.random.default_rng(t + k)
    n_ad = len(ranks)
    if mode == "random":
        ids = rng.integers(0, n_ad, size=t)
    elif mode == "runs":
        ids = np.repeat(rng.integers(0, n_ad, size=t // 5 + 1), 5)[:t]
    else:
        lens = np.maximum(1, (t * (np.arange(1, 129) ** -1.1) / (np.arange(1, 129) ** -1.1).sum()).astype(int))
        lens[0] += t - lens.sum()
        ids = np.repeat(rng.integers(0, n_ad, size=128), lens)
    a, offs, rk = _tables(ranks, k, seed=t)
    x = randn((t, k), 1.0, seed=k)
    r_max = max(ranks)
    z = _run(x, a, offs, rk, ids, r_max, split_k)
    want = 0.7 * orc.shrink_ragged(np64(x), np64(a), offs.cpu().numpy(), rk.cpu().numpy(), ids, r_max)
    err = np.abs(np64(z) - want).max()
    assert err < 2e-4 * max(1.0, np.abs(want).max()), err
    again = _run(x, a, offs, rk, ids, r_max, split_k)
    assert torch.equal(z, again)  # fixed reduction order
    zb = _run(x, a, offs, rk, ids, r_max, split_k, z_dtype=torch.bfloat16)
    assert np.abs(np64(zb) - want).max() <= 1e-2 * max(1.0, np.abs(want).max())
    assert _lib.device_error() == 0


def test_unit_shrink_out_of_range_ids_are_zero_and_reported():
    t, k = 200, 512
    a, offs, rk = _tables([16, 32], k, seed=5)
    ids = np.zeros(t, dtype=np.int64)
    ids[50:70] = 7  # no such adapter
    ids[120:] = 1
    x = randn((t, k), 1.0, seed=6)
    z = _run(x, a, offs, rk, ids, 32, 4)
    assert torch.count_nonzero(z[50:70]) == 0
    want = 0.7 * orc.shrink_ragged(np64(x), np64(a), offs.cpu().numpy(), rk.cpu().numpy(),
                                   np.where(ids == 7, 0, ids), 32)
    keep = np.ones(t, dtype=bool)
    keep[50:70] = False
    assert np.abs(np64(z)[keep] - want[keep]).max() < 2e-4
    assert _lib.device_error() == 110  # out-of-range adapter id recorded (and cleared by the read)
    assert _lib.device_error() == 0


def _branch_case(t, k, n, ranks, ids, seed, with_y=True):
    g = torch.Generator().manual_seed(seed)
    rk = torch.tensor(ranks, dtype=torch.int64)
    offs = torch.zeros_like(rk)
    offs[1:] = torch.cumsum(rk, 0)[:-1]
    tot = max(int(rk.sum()), 1)
    a = (torch.randn(tot, k, generator=g) / math.sqrt(k)).to(torch.bfloat16).to(DEV)
    b = (torch.randn(tot, n, generator=g) * 0.3).to(torch.bfloat16).to(DEV)
    x = randn((t, k), 1.0, seed=seed + 1)
    y = randn((t, n), 1.0, seed=seed + 2) if with_y else None
    return x, y, a, b, offs.to(DEV), rk.to(DEV)


@pytest.mark.parametrize("t,k,n,ranks,mode,with_y", [
    (4096, 4096, 4096, [4, 8, 16, 32, 64] * 12 + [8] * 4, "zipf", True),  # C3-like
    (1000, 1024, 320, [4, 8, 16, 32, 64], "random", True),                # one-token tiles, N % 256 != 0
    (777, 576, 512, [64, 13, 0, 33], "runs", True),                      # rank 0, last tile cut by T
    (300, 256, 1024, [16, 48], "runs", False),                           # y = None
    (3000, 512, 256, [4, 8, 16, 32, 64], "random", True),                # > 1024 tiles: schedule order, no sort
])
def test_unit_branch_matches_oracle(t, k, n, ranks, mode, with_y):
    from oracle import checks

    rng = np.random.default_rng(t + n)
    n_ad = len(ranks)
    if mode == "random":
        ids = rng.integers(0, n_ad, size=t)
    elif mode == "runs":
        ids = np.repeat(rng.integers(0, n_ad, size=t // 5 + 1), 5)[:t]
    else:
        lens = np.maximum(1, (t * (np.arange(1, 129) ** -1.1) / (np.arange(1, 129) ** -1.1).sum()).astype(int))
        lens[0] += t - lens.sum()
        ids = np.repeat(rng.integers(0, n_ad, size=128), lens)
    x, y, a, b, offs, rk = _branch_case(t, k, n, ranks, ids, seed=t)
    tiles, s = kernels.sgmv_schedule(t, offs.numel(), ids=torch.as_tensor(ids, device=DEV))
    out = kernels.sgmv_branch(x, y, a, b, offs, rk, tiles, s, max(ranks))
    assert out is not None
    yy = y if y is not None else torch.zeros((t, n), device=DEV, dtype=torch.bfloat16)
    rep = checks.branch_report(out, x, yy, a, b, offs, rk, ids, n_random=64)
    assert rep["ok"], rep
    again = kernels.sgmv_branch(x, y, a, b, offs, rk, tiles, s, max(ranks))
    assert torch.equal(out, again)
    assert _lib.device_error() == 0


def test_unit_branch_fp16():
    """fp16 operands through the one-call branch (the identity pass that adds y
    and the hi/lo z pair in half precision), with and without y."""
    from oracle import checks

    t, k, n = 700, 512, 768
    ranks = [16, 64, 8, 33]
    ids = np.repeat(np.random.default_rng(3).integers(0, len(ranks), size=t // 50 + 1), 50)[:t]
    x, y, a, b, offs, rk = _branch_case(t, k, n, ranks, ids, seed=31)
    x, y, a, b = x.half(), y.half(), a.half(), b.half()
    tiles, s = kernels.sgmv_schedule(t, offs.numel(), ids=torch.as_tensor(ids, device=DEV))
    for yy in (y, None):
        out = kernels.sgmv_branch(x, yy, a, b, offs, rk, tiles, s, max(ranks))
        assert out is not None and out.dtype == torch.float16
        ref_y = yy if yy is not None else torch.zeros((t, n), device=DEV, dtype=torch.float16)
        rep = checks.branch_report(out, x, ref_y, a, b, offs, rk, ids, dtype="f16", n_random=64)
        assert rep["ok"], rep
    assert _lib.device_error() == 0


def test_unit_branch_declines_outside_its_domain():
    """Ranks above 64, N or K not a multiple of 64: the one-call branch declines and
    the public branch surfaces take shrink + expand instead (same results)."""
    from probe_b200 import ragged_branch

    for k, n, ranks in ((256, 256, [96, 16]), (256, 264, [16, 32]), (520, 256, [16, 32])):
        ids = np.repeat([0, 1], 64)
        x, y, a, b, offs, rk = _branch_case(128, k, n, ranks, ids, seed=9)
        idt = torch.as_tensor(ids, device=DEV)
        tiles, s = kernels.sgmv_schedule(128, 2, ids=idt)
        assert kernels.sgmv_branch(x, y, a, b, offs, rk, tiles, s, max(ranks)) is None
        out = ragged_branch.branch(x, y, a, b, offs, rk, idt, max(ranks))
        want = orc.ragged_branch(np64(x), np64(y), np64(a), np64(b), offs.cpu().numpy(), rk.cpu().numpy(), ids)
        from tests.helpers import assert_parity
        assert_parity(out, want)
