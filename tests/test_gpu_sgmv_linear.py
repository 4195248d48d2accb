"""Fused base + multi-adapter linear (GPU): lora_sgmv_linear, the adapters of
every 256-token output tile as a K tail of the base CTA-pair GEMM.

Cases reach its edges: both tile widths (256 x 256 and 256 x 512), C3's
Zipf segments over 64 adapters (with a bias),
per-token random ids (many pieces per tile), rank-0 adapters, ranks above 32
(two slots per piece) and at most 16 (one K step), T not a multiple of 256 and
below one tile, N not a multiple of 256, unknown adapter ids (base only,
error recorded).  Results against the float64 oracle (the exact base plus
``ragged_branch``) on sampled tokens, against a plain PyTorch fp32 computation
of the same op over the whole output, and bit-identical on repeat.
"""

import math

import numpy as np
import pytest
import torch

from oracle import checks
from probe_b200 import _lib, kernels, ragged_branch, segmented_branch, workloads
from tests.helpers import randn

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tables(ranks, k, n, seed):
    g = torch.Generator().manual_seed(seed)
    rk = torch.tensor(ranks, dtype=torch.int64)
    offs = torch.zeros_like(rk)
    offs[1:] = torch.cumsum(rk, 0)[:-1]
    tot = max(int(rk.sum()), 1)
    a = (torch.randn(tot, k, generator=g) / math.sqrt(k)).to(torch.bfloat16).to(DEV)
    b = (torch.randn(tot, n, generator=g) * 0.3).to(torch.bfloat16).to(DEV)
    return a, b, offs.to(DEV), rk.to(DEV)


def _ids(mode, t, n_ad, rng):
    if mode == "random":
        return rng.integers(0, n_ad, size=t)
    if mode == "runs":
        return np.repeat(rng.integers(0, n_ad, size=t // 37 + 1), 37)[:t]
    lens = np.maximum(1, (t * (np.arange(1, 33) ** -1.1) / (np.arange(1, 33) ** -1.1).sum()).astype(int))
    lens[0] += t - lens.sum()
    return np.repeat(rng.integers(0, n_ad, size=32), lens)


def _fp32_close(got, x, w, bias, a, b, offs, rk, ids):
    """Whole output against a plain PyTorch fp32 computation of the same op (z in
    fp32; the kernel carries it as a bf16 hi/lo pair, ~16 mantissa bits)."""
    ref = x.float() @ w.float().T
    if bias is not None:
        ref += bias.float()
    ids_t = torch.as_tensor(ids, device=x.device)
    offs_c, rk_c = offs.cpu().tolist(), rk.cpu().tolist()
    for ad in torch.unique(ids_t).tolist():
        if ad < 0 or ad >= len(rk_c) or rk_c[ad] == 0:
            continue
        rows = (ids_t == ad).nonzero().flatten()
        o, r = offs_c[ad], rk_c[ad]
        z = x[rows].float() @ a[o:o + r].float().T
        ref[rows] += z @ b[o:o + r].float()
    diff = (got.float() - ref).abs()
    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - 7)
    ok = bool((diff <= ulp + 2e-3).all())  # the final bf16 rounding plus the hi/lo residue
    return ok, float(diff.max())


@pytest.mark.parametrize("t,k,n,ranks,mode,with_bias", [
    (1000, 1024, 320, [4, 8, 16, 32, 64], "random", True),   # every token its own piece; N % 256 != 0
    (777, 576, 512, [64, 13, 0, 33], "runs", False),         # rank 0, ranks > 32, last tile cut by T
    (300, 256, 1024, [16, 48], "zipf", True),                 # two tiles, one of 44 tokens
    (200, 512, 256, [8, 16], "runs", False),                  # less than one tile
    (2048, 2048, 2048, [4, 8, 16, 32, 64] * 4, "zipf", True),
    (1500, 3072, 4608, [4, 8, 16, 32, 64] * 4, "runs", True),  # 256 x 512 tiles, last tile cut by T
    (600, 3072, 4096, [64, 8, 0, 40], "random", False),          # 256 x 512 tiles, many pieces
    (50, 64, 64, [16, 8], "runs", True),                          # one k-block, one 64-column chunk
    (3000, 128, 192, [32, 64, 4], "zipf", False),                 # short K, N = 3 chunks
])
def test_sgmv_linear_matches_oracle(t, k, n, ranks, mode, with_bias):
    rng = np.random.default_rng(t + n)
    ids = _ids(mode, t, len(ranks), rng)
    a, b, offs, rk = _tables(ranks, k, n, seed=t)
    x = randn((t, k), 1.0, seed=k)
    w = randn((n, k), 1 / math.sqrt(k), seed=n)
    bias = randn((n,), 1.0, seed=3) if with_bias else None
    idt = torch.as_tensor(ids, device=DEV)
    r_max = max(ranks)
    got = ragged_branch.linear(x, w, bias, a, b, offs, rk, idt, r_max)
    tiles, s = kernels.sgmv_schedule(t, len(ranks), ids=idt)
    assert kernels.sgmv_linear(x, w, bias, a, b, offs, rk, tiles, s, r_max) is not None  # the fused kernel ran
    rep = checks.seg_linear_report(got, x, w, bias, a, b, offs, rk, ids, n_random=64)
    assert rep["ok"], rep
    ok, worst = _fp32_close(got, x, w, bias, a, b, offs, rk, ids)
    assert ok, worst
    again = ragged_branch.linear(x, w, bias, a, b, offs, rk, idt, r_max)
    assert torch.equal(got, again)
    assert _lib.device_error() == 0


def test_sgmv_linear_c3_config():
    """C3's batch (4096 tokens, 128 Zipf segments, 64 adapters, K = N = 4096) with
    its base weight: the segmented surface, oracle rows, the unfused path over the
    whole output, and per-token ids giving the same bits as the segment table."""
    c = workloads.c3(device=DEV, dtype=torch.bfloat16)
    got = segmented_branch.segmented_linear_varlen(c.x, c.w, None, c.a_flat, c.b_flat, c.offsets, c.ranks,
                                                   c.seg_start, c.seg_adapter, c.r_max)
    ids = c.token_ids()
    rep = checks.seg_linear_report(got, c.x, c.w, None, c.a_flat, c.b_flat, c.offsets, c.ranks, ids, n_random=96)
    assert rep["ok"], rep
    idt = torch.as_tensor(ids, device=DEV)
    ok, worst = _fp32_close(got, c.x, c.w, None, c.a_flat, c.b_flat, c.offsets, c.ranks, ids)
    assert ok, worst
    by_ids = ragged_branch.linear(c.x, c.w, None, c.a_flat, c.b_flat, c.offsets, c.ranks, idt, c.r_max)
    assert torch.equal(got, by_ids)
    assert _lib.device_error() == 0


def test_sgmv_linear_unknown_ids_add_nothing():
    t, k, n = 512, 256, 256
    a, b, offs, rk = _tables([16, 32], k, n, seed=5)
    ids = np.zeros(t, dtype=np.int64)
    ids[100:140] = 9  # no such adapter
    ids[300:] = 1
    x = randn((t, k), 1.0, seed=6)
    w = randn((n, k), 1 / math.sqrt(k), seed=7)
    idt = torch.as_tensor(ids, device=DEV)
    got = ragged_branch.linear(x, w, None, a, b, offs, rk, idt, 32)
    base = kernels.gemm(x, w)
    assert torch.equal(got[100:140], base[100:140])  # same GEMM, no tail for those tokens
    assert _lib.device_error() == 110
    assert _lib.device_error() == 0
    keep = np.ones(t, dtype=bool)
    keep[100:140] = False
    rep = checks.seg_linear_report(got[torch.as_tensor(np.flatnonzero(keep), device=DEV)],
                                   x[torch.as_tensor(np.flatnonzero(keep), device=DEV)], w, None, a, b, offs, rk,
                                   ids[keep])
    assert rep["ok"], rep


def test_sgmv_linear_declines_outside_its_domain():
    """Ranks above 64, N or K not a multiple of 64: the fused kernel declines and the
    surfaces run base GEMM + branch (same results as that path)."""
    for k, n, ranks in ((256, 256, [96, 16]), (256, 264, [16, 32]), (520, 256, [16, 32])):
        ids = np.repeat([0, 1], 64)
        a, b, offs, rk = _tables(ranks, k, n, seed=9)
        x = randn((128, k), 1.0, seed=10)
        w = randn((n, k), 1 / math.sqrt(k), seed=11)
        idt = torch.as_tensor(ids, device=DEV)
        tiles, s = kernels.sgmv_schedule(128, 2, ids=idt)
        assert kernels.sgmv_linear(x, w, None, a, b, offs, rk, tiles, s, max(ranks)) is None
        got = ragged_branch.linear(x, w, None, a, b, offs, rk, idt, max(ranks))
        rep = checks.seg_linear_report(got, x, w, None, a, b, offs, rk, ids)
        assert rep["ok"], rep


def test_sgmv_linear_fp16():
    t, k, n = 700, 512, 768
    ids = np.repeat(np.random.default_rng(3).integers(0, 3, size=t // 50 + 1), 50)[:t]
    a, b, offs, rk = _tables([16, 64, 8], k, n, seed=12)
    a, b = a.half(), b.half()
    x = randn((t, k), 1.0, dtype=torch.float16, seed=13)
    w = randn((n, k), 1 / math.sqrt(k), dtype=torch.float16, seed=14)
    bias = randn((n,), 1.0, dtype=torch.float16, seed=15)
    got = ragged_branch.linear(x, w, bias, a, b, offs, rk, torch.as_tensor(ids, device=DEV), 64)
    assert got.dtype == torch.float16
    rep = checks.seg_linear_report(got, x, w, bias, a, b, offs, rk, ids, dtype="f16")
    assert rep["ok"], rep
    ok, worst = _fp32_close(got, x, w, bias, a, b, offs, rk, ids)
    assert ok, worst


def test_sgmv_linear_declines_batches_beyond_its_workspace_cap():
    """Per-token ids over 9000 tokens: the slot region's worst case (every token
    its own piece) is above the cap, so the fused kernel declines and the surface
    runs base GEMM + branch."""
    t, k, n = 9000, 256, 256
    a, b, offs, rk = _tables([16, 8], k, n, seed=21)
    ids = np.random.default_rng(22).integers(0, 2, size=t)
    x = randn((t, k), 1.0, seed=23)
    w = randn((n, k), 1 / math.sqrt(k), seed=24)
    idt = torch.as_tensor(ids, device=DEV)
    assert _lib.load().lora_sgmv_linear_workspace_size(t, 0, k, 16) == 0
    tiles, s = kernels.sgmv_schedule(t, 2, ids=idt)
    assert kernels.sgmv_linear(x, w, None, a, b, offs, rk, tiles, s, 16) is None
    got = ragged_branch.linear(x, w, None, a, b, offs, rk, idt, 16)
    rep = checks.seg_linear_report(got, x, w, None, a, b, offs, rk, ids)
    assert rep["ok"], rep
