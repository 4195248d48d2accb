"""Dense-block SGMV kernels (GPU): shrink and expand over 64-token blocks.

Each case is checked against the float64 oracle (oracle/lora_oracle.py).  The
shapes are chosen to reach every branch of the block kernels: several tiles
per block whose ranks add up to more than one pass of adapter rows, token
counts and K / N that are not multiples of the block or tile, r_max up to 128,
rank-0 and out-of-range tiles, row indirection, y = None, fp32 and 16-bit z,
and the per-tile fallback taken by layouts the block path rejects.
"""

import math

import numpy as np
import pytest
import torch

from oracle import lora_oracle as orc
from probe_b200 import _lib, kernels
from tests.helpers import assert_parity, np64, randn

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tables(ranks, k, n, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    ranks_t = torch.tensor(ranks, dtype=torch.int64)
    offs = torch.zeros_like(ranks_t)
    offs[1:] = torch.cumsum(ranks_t, 0)[:-1]
    tot = int(ranks_t.sum())
    a = (torch.randn(tot, k, generator=g) / math.sqrt(k)).to(dtype)
    b = (torch.randn(tot, n, generator=g) * 0.2).to(dtype)
    return a.to(DEV), b.to(DEV), offs.to(DEV), ranks_t.to(DEV)


def _want_z(x, a, offs, ranks, ids, width, scale=1.0):
    z = orc.shrink_ragged(np64(x), np64(a), offs.cpu().numpy(), ranks.cpu().numpy(), ids, width)
    return scale * z


def _want_out(y, z, b, offs, ranks, ids, scale=1.0):
    """y + scale * z[t, :r] . B_a for every token (z as given, fp32)."""
    yv = np.zeros((z.shape[0], b.shape[1])) if y is None else np64(y)
    out = yv.copy()
    bv = np64(b)
    o, r = offs.cpu().numpy(), ranks.cpu().numpy()
    for t, ad in enumerate(ids):
        if ad < 0 or ad >= len(r) or r[ad] == 0:
            continue
        rr = min(int(r[ad]), z.shape[1])
        out[t] += scale * (z[t, :rr] @ bv[o[ad]:o[ad] + rr])
    return out


@pytest.mark.parametrize("split_k", [1, 3, 0])
def test_multi_pass_blocks(split_k):
    """Runs of 3 tokens cycling over six rank-64 adapters: every block holds
    ~21 tiles whose adapter rows need several passes of 128 rows."""
    k, n, t = 520, 264, 300
    ranks = [64, 64, 48, 64, 64, 40, 0, 17]
    a, b, offs, rk = _tables(ranks, k, n, seed=1)
    ids = np.array([(i // 3) % 6 for i in range(t)])
    ids[100:110] = 6  # rank 0
    ids[200:205] = 7  # rank 17
    idt = torch.as_tensor(ids, device=DEV)
    x = randn((t, k), 1.0, seed=2)
    y = randn((t, n), 1.0, seed=3)
    tiles, s = kernels.sgmv_schedule(t, len(ranks), ids=idt)
    z = kernels.sgmv_shrink(x, a, offs, rk, tiles, s, 64, scale=0.5, z_dtype=torch.float32, split_k=split_k)
    want_z = _want_z(x, a, offs, rk, ids, 64, scale=0.5)
    assert np.abs(np64(z) - want_z).max() < 2e-4
    out = kernels.sgmv_expand(y, z, b, n, 1, offs, rk, tiles, s, n, 64, scale=0.75)
    assert_parity(out, _want_out(y, np64(z), b, offs, rk, ids, scale=0.75))
    assert _lib.device_error() == 0


def test_split_results_agree_and_repeat():
    k, n, t = 1024, 256, 640
    ranks = [16, 32, 8, 64]
    a, b, offs, rk = _tables(ranks, k, n, seed=4)
    ids = np.repeat(np.array([0, 3, 1, 2, 3, 0, 2]), [50, 100, 7, 200, 90, 150, 43])
    idt = torch.as_tensor(ids, device=DEV)
    x = randn((t, k), 1.0, seed=5)
    tiles, s = kernels.sgmv_schedule(t, 4, ids=idt)
    zs = [kernels.sgmv_shrink(x, a, offs, rk, tiles, s, 64, split_k=sk) for sk in (1, 2, 5, 16)]
    want = _want_z(x, a, offs, rk, ids, 64)
    for z in zs:
        assert np.abs(np64(z) - want).max() < 2e-4
    again = kernels.sgmv_shrink(x, a, offs, rk, tiles, s, 64, split_k=5)
    assert torch.equal(again, zs[2])  # deterministic split-K reduction


def test_rank_128_and_row_indirection():
    k, n, t = 256, 392, 200
    ranks = [128, 96, 5]
    a, b, offs, rk = _tables(ranks, k, n, seed=6)
    gen = torch.Generator().manual_seed(7)
    ids = torch.randint(0, 3, (t,), generator=gen).numpy()
    order = np.argsort(ids, kind="stable")  # adapter-sorted logical order
    rows = torch.as_tensor(order, device=DEV)
    sorted_ids = torch.as_tensor(ids[order], device=DEV)
    x = randn((t, k), 1.0, seed=8)
    y = randn((t, n), 1.0, seed=9)
    tiles, s = kernels.sgmv_schedule(t, 3, ids=sorted_ids)
    z = kernels.sgmv_shrink(x, a, offs, rk, tiles, s, 128, z_dtype=torch.float32, rows=rows)
    want_z = _want_z(x, a, offs, rk, ids, 128)
    assert np.abs(np64(z) - want_z).max() < 2e-4
    out = kernels.sgmv_expand(y, z, b, n, 1, offs, rk, tiles, s, n, 128, rows=rows)
    assert_parity(out, _want_out(y, np64(z), b, offs, rk, ids))


@pytest.mark.parametrize("zdt", [torch.float32, torch.bfloat16])
def test_expand_without_y_and_16bit_z(zdt):
    k, n, t = 128, 136, 130
    ranks = [8, 24, 16]
    a, b, offs, rk = _tables(ranks, k, n, seed=10)
    seg_start = torch.tensor([0, 40, 41, 100, 130], device=DEV)
    seg_ad = torch.tensor([2, 0, 1, 2], device=DEV)
    ids = orc.segments_to_ids(seg_start.cpu().numpy(), seg_ad.cpu().numpy())
    x = randn((t, k), 1.0, seed=11)
    tiles, s = kernels.sgmv_schedule(t, 3, seg_start=seg_start, seg_adapter=seg_ad)
    z = kernels.sgmv_shrink(x, a, offs, rk, tiles, s, 24, z_dtype=zdt)
    out = kernels.sgmv_expand(None, z, b, n, 1, offs, rk, tiles, s, n, 24, dtype=torch.bfloat16)
    assert_parity(out, _want_out(None, np64(z), b, offs, rk, ids))


def test_fallback_layouts_match_block_path():
    """N not a multiple of 8 and a PEFT-layout B take the per-tile kernels."""
    k, t = 64, 150
    ranks = [16, 8]
    for n in (100, 101):
        a, b, offs, rk = _tables(ranks, k, n, seed=12)
        ids = np.array([i % 2 for i in range(t)])
        idt = torch.as_tensor(ids, device=DEV)
        x = randn((t, k), 1.0, seed=13)
        y = randn((t, n), 1.0, seed=14)
        tiles, s = kernels.sgmv_schedule(t, 2, ids=idt)
        z = kernels.sgmv_shrink(x, a, offs, rk, tiles, s, 16)
        out = kernels.sgmv_expand(y, z, b, n, 1, offs, rk, tiles, s, n, 16)
        assert_parity(out, _want_out(y, np64(z), b, offs, rk, ids))


@pytest.mark.parametrize("t,k,ranks", [(300, 520, [128, 96, 5]), (129, 4096, [64, 16, 4, 32, 8]),
                                       (4096, 1024, [4, 8, 16, 32, 64] * 4)])
def test_tensor_core_shrink_matches_oracle(t, k, ranks):
    """The tcgen05 segmented shrink (128-token blocks, adapter rows gathered by
    TMA, passes when a block's adapters exceed 256 rows, cluster split-K)."""
    n = 64
    a, b, offs, rk = _tables(ranks, k, n, seed=t)
    gen = torch.Generator().manual_seed(t + 1)
    lens = torch.randint(1, 90, (t,), generator=gen)
    seg = [0]
    while seg[-1] < t:
        seg.append(min(t, seg[-1] + int(lens[len(seg)])))
    seg_start = torch.tensor(seg, device=DEV)
    seg_ad = torch.randint(0, len(ranks), (len(seg) - 1,), generator=gen).to(DEV)
    ids = orc.segments_to_ids(seg_start.cpu().numpy(), seg_ad.cpu().numpy())
    x = randn((t, k), 1.0, seed=t + 2)
    tiles, s = kernels.sgmv_schedule(t, len(ranks), seg_start=seg_start, seg_adapter=seg_ad)
    r_max = max(ranks)
    for zdt in (torch.float32, torch.bfloat16):
        z = kernels.sgmv_shrink(x, a, offs, rk, tiles, s, r_max, scale=0.5, z_dtype=zdt)
        want = _want_z(x, a, offs, rk, ids, r_max, scale=0.5)
        tol = 2e-4 if zdt == torch.float32 else 1e-2
        assert np.abs(np64(z) - want).max() < tol * max(1.0, np.abs(want).max())
        assert torch.equal(z, kernels.sgmv_shrink(x, a, offs, rk, tiles, s, r_max, scale=0.5, z_dtype=zdt))
    assert _lib.device_error() == 0


@pytest.mark.parametrize("ranks", [[64] * 12, [128, 96, 64, 128, 32, 128, 80, 128]])
def test_tensor_core_shrink_wide_blocks(ranks):
    """8-token segments cycling over many wide adapters: a 128-token block needs
    more than 256 adapter rows (two MMAs per pass) and more than one pass."""
    t, k, n = 384, 1024, 64
    a, b, offs, rk = _tables(ranks, k, n, seed=len(ranks))
    seg = list(range(0, t, 8)) + [t]
    seg_start = torch.tensor(seg, device=DEV)
    seg_ad = torch.tensor([i % len(ranks) for i in range(len(seg) - 1)], device=DEV)
    ids = orc.segments_to_ids(seg_start.cpu().numpy(), seg_ad.cpu().numpy())
    x = randn((t, k), 1.0, seed=17)
    tiles, s = kernels.sgmv_schedule(t, len(ranks), seg_start=seg_start, seg_adapter=seg_ad)
    r_max = max(ranks)
    z = kernels.sgmv_shrink(x, a, offs, rk, tiles, s, r_max, scale=0.25, z_dtype=torch.float32)
    want = _want_z(x, a, offs, rk, ids, r_max, scale=0.25)
    assert np.abs(np64(z) - want).max() < 2e-4 * max(1.0, np.abs(want).max())
    assert torch.equal(z, kernels.sgmv_shrink(x, a, offs, rk, tiles, s, r_max, scale=0.25, z_dtype=torch.float32))
    assert _lib.device_error() == 0
