"""Reference call surfaces on the GPU, against golden vectors and the oracle.

Mirrors the reference's own tests (test_fused_linear.py, test_decode_linear.py,
test_peft_integration.py) plus the multi-adapter branch paths, which the
reference leaves untested.
"""

import math

import numpy as np
import pytest
import torch
from torch import nn

from oracle import lora_oracle as orc
from probe_b200 import (
    DualStreamOverlappedLinear,
    FusedLoRALinear,
    attach_fused_lora,
    build_ext,
    classed_lora,
    classed_tiled_lora,
    expand_add,
    fused_gemm,
    fused_lora,
    fused_lora_linear,
    fused_lora_module_count,
    grouped_lora,
    kconcat_weight,
    persistent_expand_add,
    splitk_lora_shrink,
    splitk_persistent_fused_lora,
    tiled_lora,
    total_fused_rank,
)
from probe_b200 import _lib, fused_linear, kernels, multilora, ragged_branch, segmented_branch, splitk_shrink
from probe_b200 import workloads
from probe_b200.decode_linear import decode_lora_linear
from tests.golden_io import from_bits, load
from tests.helpers import assert_parity, np64, randn

pytestmark = pytest.mark.gpu
DEV = "cuda"


def t(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).to(DEV)


# ------------------------------------------------------------- golden vectors
def test_golden_linear_cases():
    d = load("linear_cases.npz")
    for i in range(int(d["n_cases"])):
        bias = t(from_bits(d[f"c{i}_bias"])) if d[f"c{i}_bias"].size else None
        out = fused_lora_linear(t(from_bits(d[f"c{i}_x"])), t(from_bits(d[f"c{i}_w"])), bias,
                                t(from_bits(d[f"c{i}_a"])), t(from_bits(d[f"c{i}_b"])), float(d[f"c{i}_scale"]))
        assert_parity(out, d[f"c{i}_out"])
    x = t(from_bits(d["nd_x"]))
    out = fused_lora_linear(x, t(from_bits(d["nd_w"])), None, t(from_bits(d["nd_a"])), t(from_bits(d["nd_b"])), 0.8)
    assert out.shape == (2, 5, 64)
    assert_parity(out, d["nd_out"])


def test_golden_c1_full_config():
    d = load("c1_checksums.npz")
    p = workloads.c1(device="cpu", dtype=torch.float32)
    out = fused_lora_linear(p.x.to(DEV, torch.bfloat16), p.w.to(DEV, torch.bfloat16), None,
                            p.a.to(DEV, torch.bfloat16), p.b.to(DEV, torch.bfloat16), p.scale)
    o = np64(out)
    assert_parity(out[torch.as_tensor(d["rows"], device=DEV)], d["bf16in_rows"])
    # size-independent properties over the whole output.  Each bf16 output carries
    # a rounding error of std ~ ulp/sqrt(12) (~0.0045 at |y| ~ 2); a row sum of
    # 4096 of them random-walks to ~0.29, so 2.0 is a ~6 sigma bound.
    assert np.abs(o.sum(1) - d["bf16in_row_sums"]).max() < 2.0
    assert abs(np.linalg.norm(o) - float(d["bf16in_fro"])) / float(d["bf16in_fro"]) < 2e-3


def test_golden_stacked_adapters():
    d = load("stack_case.npz")
    base = nn.Linear(64, 48, bias=True, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        base.weight.copy_(t(from_bits(d["w"])))
        base.bias.copy_(t(from_bits(d["bias"])))
    holder = nn.Module()
    holder.proj = base
    for i in range(3):
        attach_fused_lora(holder, "proj", t(from_bits(d[f"down{i}"])), t(from_bits(d[f"up{i}"])),
                          float(d[f"alpha{i}"]))
    assert holder.proj.rank == int(d["rank"])
    assert fused_lora_module_count(holder) == 1 and total_fused_rank(holder) == 28
    out = holder.proj(t(from_bits(d["x"])))
    assert_parity(out, d["out"])


def test_golden_branches():
    d = load("branch_cases.npz")
    a, b = t(from_bits(d["a_flat"])), t(from_bits(d["b_flat"]))
    offs, ranks = torch.as_tensor(d["offsets"], device=DEV), torch.as_tensor(d["ranks"], device=DEV)
    ids = torch.as_tensor(d["ids"], device=DEV)
    rmax = int(d["ranks"].max())
    out = ragged_branch.branch(t(from_bits(d["x"])), t(from_bits(d["y"])), a, b, offs, ranks, ids, rmax)
    assert_parity(out, d["ragged_out"])
    out = ragged_branch.branch(t(from_bits(d["x"])), t(from_bits(d["y"])), a, b, offs, ranks, ids, rmax,
                               skip_zero=False)
    assert_parity(out, d["ragged_noskip_out"])
    req = torch.as_tensor(d["req"], device=DEV)
    out = segmented_branch.segmented_branch(t(from_bits(d["xs"])), t(from_bits(d["ys"])), a, b, offs, ranks, req,
                                            12, rmax)
    assert_parity(out, d["seg_out"])
    with pytest.raises(ValueError):
        segmented_branch.segmented_branch(t(from_bits(d["xs"])), t(from_bits(d["ys"])), a, b, offs, ranks, req,
                                          11, rmax)
    assert _lib.device_error() == 0


# --------------------------------------------------- test_fused_linear mirror
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("m,k,n", [(512, 320, 320), (1024, 1536, 8960), (256, 640, 1280)])
@pytest.mark.parametrize("r", [1, 7, 16, 17, 40, 64, 130])
def test_variants_match(dtype, m, k, n, r):
    """Every variant reproduces the naive formulation (test_fused_linear.py:49-78)."""
    torch.manual_seed(r + m)
    x = torch.randn(m, k, device=DEV, dtype=dtype) / k**0.5
    w = torch.randn(n, k, device=DEV, dtype=dtype) / k**0.5
    bias = torch.randn(n, device=DEV, dtype=dtype)
    a = torch.randn(r, k, device=DEV, dtype=dtype) / k**0.5
    b = torch.randn(n, r, device=DEV, dtype=dtype) / r**0.5
    scale = 0.75
    want = orc.naive_linear(np64(x), np64(w), np64(bias), np64(a), np64(b), scale)
    assert_parity(fused_gemm(x, w, bias, a, b, scale), want, dtype)
    assert_parity(fused_linear._KConcat(w, bias, a, b, scale)(x), want, dtype)
    if r <= 128:
        assert_parity(fused_linear._hybrid(x, w, bias, a, b, scale), want, dtype)
    w_aug = fused_linear.augment_weight(w, a)
    b_aug = fused_linear.augment_bias(bias, r)
    assert w_aug.shape[0] == n + fused_linear.packed_rank(r)
    assert_parity(fused_linear._concat(x, w_aug, b_aug, b, scale, n), want, dtype)
    w_kc = kconcat_weight(w, b)
    assert w_kc.shape == (n, k + fused_linear.packed_rank(r))
    if r <= 128:
        assert_parity(fused_linear._kconcat(x, w_kc, bias, a, scale, fused_linear.packed_rank(r)), want, dtype)
    assert_parity(fused_lora_linear(x, w, bias, a, b, scale), want, dtype)


def test_fused_gemm_without_sidecar():
    for dtype in (torch.float16, torch.bfloat16):
        m, k, n = 1024, 640, 1280
        x = torch.randn(m, k, device=DEV, dtype=dtype) / k**0.5
        w = torch.randn(n, k, device=DEV, dtype=dtype) / k**0.5
        bias = torch.randn(n, device=DEV, dtype=dtype)
        assert_parity(fused_gemm(x, w, bias, None, None, 1.0), orc.naive_linear(np64(x), np64(w), np64(bias), None,
                                                                                  None, 0), dtype)


def test_build_ext():
    for dtype in (torch.float16, torch.bfloat16):
        for k, r in ((640, 24), (1536, 128), (320, 7)):
            m = 512
            x = torch.randn(m, k, device=DEV, dtype=dtype) / k**0.5
            a = torch.randn(r, k, device=DEV, dtype=dtype) / k**0.5
            pad = fused_linear.packed_rank(r)
            ext = build_ext(x, a, 0.5, pad)
            assert torch.equal(ext[:, :k], x)
            assert_parity(ext[:, k:k + r], 0.5 * (np64(x) @ np64(a).T), dtype)
            if pad > r:
                assert torch.count_nonzero(ext[:, k + r:]) == 0


def test_expand_add_leaves_input():
    m, n, r = 512, 1280, 24
    y = torch.randn(m, n, device=DEV, dtype=torch.float16)
    z = torch.randn(m, r, device=DEV, dtype=torch.float16)
    b = torch.randn(n, r, device=DEV, dtype=torch.float16) / r**0.5
    y0 = y.clone()
    assert_parity(expand_add(y, z, b, 0.5), orc.expand_add(np64(y), np64(z), np64(b), 0.5), torch.float16)
    assert torch.equal(y, y0)


def test_module_and_swap():
    """FusedLoRALinear, attach and stacking (test_fused_linear.py:127-168)."""
    dtype = torch.float16
    k, n, r, m = 640, 1280, 24, 2048
    base = nn.Linear(k, n, bias=True).cuda().to(dtype)
    a = torch.randn(r, k, device=DEV, dtype=dtype) / k**0.5
    b = torch.randn(n, r, device=DEV, dtype=dtype) / r**0.5
    x = torch.randn(4, m // 4, k, device=DEV, dtype=dtype) / k**0.5
    alpha = 0.8
    x2 = np64(x.reshape(-1, k))
    want = orc.naive_linear(x2, np64(base.weight), np64(base.bias), np64(a), np64(b), alpha).reshape(4, m // 4, n)
    module = FusedLoRALinear(base, a, b, scale=alpha)
    assert_parity(module(x), want, dtype)
    assert module.rank == r and module.weight.shape == (n, k)
    holder = nn.Module()
    holder.inner = nn.Module()
    holder.inner.proj = nn.Linear(k, n, bias=False).cuda().to(dtype)
    w0 = np64(holder.inner.proj.weight)
    attach_fused_lora(holder, "inner.proj", a, b, alpha)
    assert isinstance(holder.inner.proj, FusedLoRALinear)
    want1 = orc.naive_linear(x2, w0, None, np64(a), np64(b), alpha)
    assert_parity(holder.inner.proj(x).reshape(-1, n), want1, dtype)
    r2, alpha2 = 40, 0.35
    a2 = torch.randn(r2, k, device=DEV, dtype=dtype) / k**0.5
    b2 = torch.randn(n, r2, device=DEV, dtype=dtype) / r2**0.5
    attach_fused_lora(holder, "inner.proj", a2, b2, alpha2)
    assert holder.inner.proj.rank == r + r2
    want2 = want1 + alpha2 * (x2 @ np64(a2).T) @ np64(b2).T
    assert_parity(holder.inner.proj(x).reshape(-1, n), want2, dtype)
    holder.inner.proj.set_factors(a, b, scale=alpha)
    assert holder.inner.proj.rank == r
    assert_parity(holder.inner.proj(x).reshape(-1, n), want1, dtype)
    with pytest.raises(ValueError):
        FusedLoRALinear(base, a[:, :10], b, 1.0)
    with pytest.raises(TypeError):
        attach_fused_lora(holder, "inner", a, b)


# -------------------------------------------------- test_decode_linear mirror
def test_decode_linear_cases():
    """Noncontiguous inputs, odd shapes, r in {0..64}, scale {0, -0.7} (test_decode_linear.py:14-44)."""
    torch.manual_seed(93)
    for dtype in (torch.float16, torch.bfloat16):
        for m, k, n in ((1, 257, 131), (4, 1536, 512), (8, 769, 259)):
            x = torch.randn(m, k * 2, device=DEV, dtype=dtype)[:, ::2]
            w = torch.randn(n, k * 2, device=DEV, dtype=dtype)[:, ::2] / k**0.5
            for r in (0, 1, 3, 8, 13, 16, 33, 64):
                a = torch.randn(k, r, device=DEV, dtype=dtype).t() / k**0.5
                b = torch.randn(r, n, device=DEV, dtype=dtype).t() / max(r, 1)**0.5
                for scale, bias in ((0.0, None), (-0.7, torch.randn(n * 2, device=DEV, dtype=dtype)[::2])):
                    ref = orc.naive_linear(np64(x), np64(w), None if bias is None else np64(bias), np64(a), np64(b),
                                           scale)
                    got = decode_lora_linear(x, w, bias, a, b, scale)
                    err = float(np.linalg.norm(np64(got) - ref) / np.linalg.norm(ref))
                    assert err < (0.002 if dtype == torch.float16 else 0.012), (m, k, n, r, err)
                    if r == 0 or scale == 0:
                        base = fused_linear._base_linear(x.contiguous(), w.contiguous(), bias)
                        assert torch.equal(got, base)
    with pytest.raises(ValueError):
        decode_lora_linear(x, w, None, a[:, :5], b, 1.0)
    with pytest.raises(ValueError):
        decode_lora_linear(x.float(), w, None, a, b, 1.0)


def test_cuda_graph_replay():
    """Plans are graph-capturable: replay equals eager (test_decode_linear.py:48-55)."""
    for rows in (4, 256):
        base = nn.Linear(256, 512).cuda().bfloat16().eval()
        a = torch.randn(3, 256, device=DEV, dtype=torch.bfloat16) / 16
        b = torch.randn(512, 3, device=DEV, dtype=torch.bfloat16) / 3**0.5
        module = FusedLoRALinear(base, a, b, 0.2)
        x = torch.randn(rows, 256, device=DEV, dtype=torch.bfloat16)
        module(x)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            output = module(x)
        x.mul_(0.5)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(output, module(x))
        module.set_factors(a[:0], b[:, :0])
        assert torch.equal(module(x), fused_linear._base_linear(x, base.weight, base.bias))


# ------------------------------------------------------- decode-style sidecar
@pytest.mark.parametrize("m,k,n,r", [(1, 4096, 11008, 16), (4, 640, 1280, 24), (8, 257, 131, 7), (64, 1536, 512, 64)])
def test_fused_lora_family(m, k, n, r):
    x = randn((m, k), 1.0, seed=1)
    a = randn((r, k), 1 / math.sqrt(k), seed=2)
    b = randn((n, r), 1 / math.sqrt(r), seed=3)
    y = randn((m, n), 1.0, seed=4)
    want = orc.expand_add(np64(y), orc.shrink(np64(x), np64(a)), np64(b), 0.6)
    for fn in (fused_lora, tiled_lora, classed_lora, classed_tiled_lora):
        assert_parity(fn(x, a, b, y, 0.6), want)
    assert_parity(fused_lora(x, a, b, None, 0.6), want - np64(y))
    assert_parity(classed_lora(x, a, b, y, 0.6, execution_rank=64), want)
    with pytest.raises(AssertionError):
        classed_lora(x, a, b, y, 0.6, execution_rank=48)
    z = splitk_lora_shrink(x, a)
    assert z.dtype == x.dtype
    assert_parity(z, orc.shrink(np64(x), np64(a)))
    assert_parity(splitk_shrink.shrink_partial(x, a), orc.shrink(np64(x), np64(a)))
    assert_parity(splitk_shrink.shrink_atomic(x, a), orc.shrink(np64(x), np64(a)))
    assert_parity(persistent_expand_add(z, b, y, 0.6), orc.expand_add(np64(y), np64(z), np64(b), 0.6))
    assert_parity(splitk_persistent_fused_lora(x, a, b, y, 0.6), want)


def test_grouped_lora():
    m, k, n, r, p = 8, 512, 384, 16, 3
    x = randn((m, k), 1.0, seed=5)
    a = randn((p * r, k), 1 / math.sqrt(k), seed=6)
    b = randn((p, n, r), 1 / math.sqrt(r), seed=7)
    y = randn((m, p, n), 1.0, seed=8)
    out = grouped_lora(x, a, b, y, 0.9)
    assert out.shape == (m, p, n)
    z = orc.shrink(np64(x), np64(a))
    want = np.stack([np64(y)[:, i] + 0.9 * z[:, i * r:(i + 1) * r] @ np64(b)[i].T for i in range(p)], 1)
    assert_parity(out, want)


def test_dual_stream_overlapped():
    torch.manual_seed(0)
    mod = DualStreamOverlappedLinear(512, 768, 16, bias=True, dtype=torch.bfloat16)
    for rows in (8, 300):
        x = torch.randn(rows, 512, device=DEV, dtype=torch.bfloat16)
        out = mod(x, scale=0.5)
        want = orc.naive_linear(np64(x), np64(mod.weight), np64(mod.bias), np64(mod.lora_A), np64(mod.lora_B), 0.5)
        assert_parity(out, want)


# ------------------------------------------------------------ multi-adapter
def _tables(ranks, k, n, seed=0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    ranks_t = torch.tensor(ranks, dtype=torch.int64)
    offs = torch.zeros_like(ranks_t)
    offs[1:] = torch.cumsum(ranks_t, 0)[:-1]
    tot = int(ranks_t.sum())
    a = (torch.randn(tot, k, generator=g) / math.sqrt(k)).to(dtype)
    b = (torch.randn(tot, n, generator=g) * 0.2).to(dtype)
    return a.to(DEV), b.to(DEV), offs.to(DEV), ranks_t.to(DEV)


def test_schedule_matches_oracle():
    ids = torch.tensor([0] * 70 + [1] * 3 + [0] * 2 + [9] + [2] * 130, dtype=torch.int64, device=DEV)
    tiles, s = kernels.sgmv_schedule(ids.numel(), 4, ids=ids)
    n = int(tiles[0])
    mt = int(tiles[1])
    starts = tiles[2:3 + n].tolist()
    adapters = tiles[3 + mt:3 + mt + n].tolist()
    want_s, want_a = orc.tile_schedule(ids=ids.tolist(), n_adapters=4)
    assert starts == want_s and adapters == want_a
    assert _lib.device_error() == 110  # the out-of-range id 9 was recorded
    seg_start = torch.tensor([0, 5, 5, 9, 200], device=DEV)
    seg_ad = torch.tensor([2, 7, 2, 1], device=DEV)
    tiles, s = kernels.sgmv_schedule(200, 8, seg_start=seg_start, seg_adapter=seg_ad)
    n, mt = int(tiles[0]), int(tiles[1])
    want_s, want_a = orc.tile_schedule(seg_start=[0, 5, 5, 9, 200], seg_adapter=[2, 7, 2, 1], n_adapters=8)
    assert tiles[2:3 + n].tolist() == want_s and tiles[3 + mt:3 + mt + n].tolist() == want_a
    assert _lib.device_error() == 0


def _schedule(tiles):
    n, mt = int(tiles[0]), int(tiles[1])
    return tiles[2:3 + n].tolist(), tiles[3 + mt:3 + mt + n].tolist(), tiles[3 + 2 * mt:].tolist()


@pytest.mark.parametrize("seed", range(6))
def test_schedule_segments_match_oracle(seed):
    """Segment tables that cover the batch in order (tiled segment by segment on
    the device): empty segments, neighbours with the same adapter, out-of-range
    adapters, long segments, T not a multiple of 64.  Tile starts, adapters and
    the first tile of every 64-token block match the oracle."""
    rng = np.random.default_rng(seed)
    t = int(rng.integers(1, 3000))
    n_seg = int(rng.integers(1, 300))
    seg_start = np.concatenate([[0], np.sort(rng.integers(0, t + 1, size=n_seg - 1)), [t]])
    n_ad = 6
    seg_ad = rng.integers(-1, n_ad + 1, size=n_seg)  # -1 and n_ad are out of range
    seg_ad[rng.random(n_seg) < 0.3] = 2              # runs of neighbours sharing an adapter
    tiles, _ = kernels.sgmv_schedule(t, n_ad, seg_start=torch.as_tensor(seg_start, device=DEV),
                                     seg_adapter=torch.as_tensor(seg_ad, device=DEV))
    starts, adapters, first = _schedule(tiles)
    want_s, want_a = orc.tile_schedule(seg_start=seg_start.tolist(), seg_adapter=seg_ad.tolist(), n_adapters=n_ad)
    assert starts == want_s and adapters == want_a
    blocks = (t + 63) // 64
    assert first[:blocks + 1] == [want_s.index(64 * b) for b in range(blocks)] + [len(want_a)]
    bad = any((seg_ad[i] < 0 or seg_ad[i] >= n_ad) and seg_start[i + 1] > seg_start[i] for i in range(n_seg))
    assert _lib.device_error() == (110 if bad else 0)


def test_schedule_segments_with_gaps():
    """A table that leaves tokens uncovered takes the token-by-token walk: those
    tokens get no adapter (-1) and the error is recorded."""
    seg_start = [5, 70, 200]
    seg_ad = [1, 3]
    t = 250
    tiles, _ = kernels.sgmv_schedule(t, 4, seg_start=torch.tensor(seg_start, device=DEV),
                                     seg_adapter=torch.tensor(seg_ad, device=DEV))
    starts, adapters, _ = _schedule(tiles)
    ids = [-1] * 5 + [1] * 65 + [3] * 130 + [-1] * 50
    want_s, want_a = orc.tile_schedule(ids=ids, n_adapters=4)
    assert starts == want_s and adapters == want_a
    assert _lib.device_error() == 110


def test_routing_bit_exact():
    """Exactly representable probe: out - y == adapter id + 1 for every token."""
    n_ad, k, n = 12, 64, 48
    ranks = [4, 8, 1, 16, 2, 8, 4, 32, 16, 8, 4, 64]
    offs = np.concatenate([[0], np.cumsum(ranks)[:-1]])
    a = torch.zeros(sum(ranks), k, dtype=torch.bfloat16)
    b = torch.zeros(sum(ranks), n, dtype=torch.bfloat16)
    for ad in range(n_ad):
        a[offs[ad], 3] = 1.0
        b[offs[ad], :] = ad + 1
    gen = torch.Generator().manual_seed(1)
    ids = torch.randint(0, n_ad, (500,), generator=gen)
    ids[100:180] = 7  # a long run
    x = torch.zeros(500, k, dtype=torch.bfloat16)
    x[:, 3] = 1.0
    y = torch.zeros(500, n, dtype=torch.bfloat16, device=DEV)
    args = (x.to(DEV), y, a.to(DEV), b.to(DEV), torch.as_tensor(offs, device=DEV),
            torch.tensor(ranks, device=DEV), ids.to(DEV), 64)
    out = ragged_branch.branch(*args)
    want = (ids + 1).to(torch.bfloat16)[:, None].expand(500, n).to(DEV)
    assert torch.equal(out, want)
    seg_start = torch.tensor([0, 3, 3, 50, 64, 65, 300, 500], device=DEV)
    seg_ad = torch.tensor([5, 0, 11, 2, 7, 3, 9], device=DEV)
    out = segmented_branch.segmented_branch_varlen(x.to(DEV), y, a.to(DEV), b.to(DEV), torch.as_tensor(offs, device=DEV),
                                                   torch.tensor(ranks, device=DEV), seg_start, seg_ad, 64)
    ids2 = orc.segments_to_ids(seg_start.cpu().numpy(), seg_ad.cpu().numpy())
    assert torch.equal(out, torch.as_tensor(ids2 + 1).to(torch.bfloat16)[:, None].expand(500, n).to(DEV))


def test_segmented_c3_config():
    """C3: 4096 tokens, 128 Zipf segments, 64 adapters, K = N = 4096 (sampled-row parity)."""
    c = workloads.c3(device="cpu", dtype=torch.bfloat16)
    x, w = c.x.to(DEV), c.w.to(DEV)
    y = fused_linear._base_linear(x, w, None)
    out = segmented_branch.segmented_branch_varlen(x, y, c.a_flat.to(DEV), c.b_flat.to(DEV), c.offsets.to(DEV),
                                                   c.ranks.to(DEV), c.seg_start.to(DEV), c.seg_adapter.to(DEV),
                                                   c.r_max, split_k=8)
    assert int(c.seg_start[-1]) == 4096 and c.seg_adapter.numel() == 128
    ids = c.token_ids().numpy()
    rows = np.unique(np.concatenate([np.arange(0, 4096, 37), np.asarray(c.seg_start[:-1])]))
    xr = np64(c.x[rows])
    want = np64(y)[rows] + orc.ragged_branch(xr, np.zeros((len(rows), 4096)), np64(c.a_flat), np64(c.b_flat),
                                             c.offsets.numpy(), c.ranks.numpy(), ids[rows])
    assert_parity(out[torch.as_tensor(rows, device=DEV)], want)
    # ragged (per-token ids) path gives bit-identical results to the segment path
    out2 = ragged_branch.branch(x, y, c.a_flat.to(DEV), c.b_flat.to(DEV), c.offsets.to(DEV), c.ranks.to(DEV),
                                torch.as_tensor(ids, device=DEV), c.r_max, split_k=8)
    assert torch.equal(out, out2)


def test_multilora_entry_points():
    k, n, t = 256, 192, 300
    ranks = [8, 16, 4, 32, 8]
    a_flat, b_flat, offs, rk = _tables(ranks, k, n, seed=3)
    gen = torch.Generator().manual_seed(2)
    ids = torch.randint(0, len(ranks), (t,), generator=gen).to(DEV)
    x = randn((t, k), 1.0, seed=9)
    y = randn((t, n), 1.0, seed=10)
    z = multilora.shrink_ragged(x, a_flat, offs, rk, ids, 32)
    want_z = orc.shrink_ragged(np64(x), np64(a_flat), offs.cpu().numpy(), rk.cpu().numpy(), ids.cpu().numpy(), 32)
    assert z.dtype == torch.float32
    assert np.abs(np64(z) - want_z).max() < 1e-4
    # padded stacks [n, r, K] / [n, N, r]
    r = 16
    a_st = randn((5, r, k), 1 / 16, seed=11)
    b_st = randn((5, n, r), 0.25, seed=12)
    zp = multilora.shrink_padded(x, a_st, ids)
    want_zp = orc.shrink_padded(np64(x), np64(a_st), ids.cpu().numpy())
    assert np.abs(np64(zp) - want_zp).max() < 1e-4
    out = multilora.expand_padded(y, zp, b_st, ids, scale=0.7)
    assert_parity(out, orc.expand_padded(np64(y), np64(zp), np64(b_st), ids.cpu().numpy(), 0.7))
    # rank buckets addressed by position
    buckets, buckets_b = {}, {}
    perm = torch.randperm(t, generator=gen).to(DEV)
    splits = {4: perm[:90], 16: perm[90:200], 32: perm[200:]}
    for rr, pos in splits.items():
        n_r = 3
        local = torch.randint(0, n_r, (pos.numel(),), generator=gen).to(DEV)
        buckets[rr] = (randn((n_r, rr, k), 1 / 16, seed=rr), pos, local)
        buckets_b[rr] = (randn((n_r, n, rr), 0.2, seed=rr + 1), pos, local)
    zb = multilora.shrink_bucketed(x, buckets, 32)
    streams = [torch.cuda.Stream() for _ in range(3)]
    events = [torch.cuda.Event() for _ in range(4)]
    zbp = multilora.shrink_bucketed_parallel(x, buckets, 32, streams, events)
    torch.cuda.synchronize()
    want_zb = np.zeros((t, 32))
    for rr, (a_s, pos, local) in buckets.items():
        p_np, l_np = pos.cpu().numpy(), local.cpu().numpy()
        want_zb[p_np, :rr] = orc.shrink_padded(np64(x)[p_np], np64(a_s), l_np)
    assert np.abs(np64(zb) - want_zb).max() < 1e-4
    assert torch.equal(zb, zbp)
    outb = multilora.expand_bucketed_parallel(y, zb, buckets_b, streams, events, scale=0.5)
    torch.cuda.synchronize()
    want_o = np.zeros((t, n))
    zq = np64(zb)
    for rr, (b_s, pos, local) in buckets_b.items():
        p_np, l_np = pos.cpu().numpy(), local.cpu().numpy()
        want_o[p_np] = orc.expand_padded(np64(y)[p_np], zq[p_np, :rr], np64(b_s), l_np, 0.5)
    assert_parity(outb, want_o)
    grouped = multilora.shrink_grouped(x, {rr: bk for rr, bk in buckets.items()}, ids)
    for rr, (zg, pos) in grouped.items():
        a_s, p2, local = buckets[rr]
        want_g = orc.shrink_padded(np64(x)[pos.cpu().numpy()], np64(a_s), local.cpu().numpy())
        assert np.abs(np64(zg) - want_g).max() < 1e-4


# ------------------------------------------------------------ PEFT bridge
class _FakeLoraLinear(nn.Module):
    """The attributes of peft.tuners.lora.layer.Linear that the bridge reads."""

    def __init__(self, base, r, alpha, dtype):
        super().__init__()
        self.base_layer = base
        self.lora_A = nn.ModuleDict({"default": nn.Linear(base.in_features, r, bias=False).to(DEV, dtype)})
        self.lora_B = nn.ModuleDict({"default": nn.Linear(r, base.out_features, bias=False).to(DEV, dtype)})
        with torch.no_grad():
            self.lora_B["default"].weight.normal_(0, 0.2)
        self.lora_dropout = nn.ModuleDict({"default": nn.Identity()})
        self.scaling = {"default": alpha / r}
        self.use_dora = {"default": False}
        self._active_adapter = "default"
        self.merged = False
        self.disable_adapters = False

    @property
    def active_adapters(self):
        return [self._active_adapter]

    def forward(self, x):
        y = self.base_layer(x)
        return y + self.lora_B["default"](self.lora_A["default"](x)) * self.scaling["default"]


class _ToyMLP(nn.Module):
    def __init__(self, dtype, width=256, hidden=512):
        super().__init__()
        self.gate_proj = _FakeLoraLinear(nn.Linear(width, hidden, bias=False).to(DEV, dtype), 16, 16, dtype)
        self.up_proj = _FakeLoraLinear(nn.Linear(width, hidden, bias=False).to(DEV, dtype), 16, 16, dtype)
        self.down_proj = _FakeLoraLinear(nn.Linear(hidden, width, bias=False).to(DEV, dtype), 16, 16, dtype)

    def forward(self, x):
        return self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))


class _ToyAttention(nn.Module):
    """q, k, v read the same x; k and v narrower (grouped-query attention), q and v with biases."""

    def __init__(self, dtype, width=256, kv=128):
        super().__init__()
        self.q_proj = _FakeLoraLinear(nn.Linear(width, width, bias=True).to(DEV, dtype), 16, 16, dtype)
        self.k_proj = _FakeLoraLinear(nn.Linear(width, kv, bias=False).to(DEV, dtype), 8, 16, dtype)
        self.v_proj = _FakeLoraLinear(nn.Linear(width, kv, bias=True).to(DEV, dtype), 16, 32, dtype)

    def forward(self, x):
        return self.q_proj(x), self.k_proj(x), self.v_proj(x)


def test_peft_grouped_attention():
    """q/k/v packed into one linear (opt-in): same outputs as the individual
    forwards, any call order, and an x modified in place between the calls
    takes the individual path instead of the cached outputs."""
    import copy

    from probe_b200 import enable_loraforge_peft, peft_plan_report

    torch.manual_seed(11)
    dtype = torch.bfloat16
    model = _ToyAttention(dtype).eval()
    reference = copy.deepcopy(model)
    enable_loraforge_peft(model, group_attention=True)
    assert model._loraforge_grouped_attention_count == 1
    with torch.no_grad():
        for rows in (1, 8, 200, 300):  # 200 rows, summed rank 40: the split-K linear at rank 64
            x = torch.randn(rows, 256, device=DEV, dtype=dtype)
            for got, want in zip(model(x), reference(x)):
                rel = float((got.float() - want.float()).abs().max() / want.float().abs().max())
                assert rel < 4e-2, (rows, rel)
        x = torch.randn(2, 5, 256, device=DEV, dtype=dtype)
        v = model.v_proj(x)  # another member first
        q = model.q_proj(x)
        assert v.shape == (2, 5, 128) and q.shape == (2, 5, 256)
        assert float((q.float() - reference.q_proj(x).float()).abs().max()) < 0.1
        x.add_(1.0)  # in place: the cached k must not be used
        k = model.k_proj(x)
        want = reference.k_proj(x)
        assert float((k.float() - want.float()).abs().max() / want.float().abs().max()) < 4e-2
    assert peft_plan_report(model)["grouped_attention_modules"] == 1


def test_peft_bridge():
    from probe_b200 import enable_loraforge_peft, peft_plan_report

    torch.manual_seed(7)
    dtype = torch.bfloat16
    model = _ToyMLP(dtype).eval()
    import copy

    reference = copy.deepcopy(model)
    patched = enable_loraforge_peft(model, enable_grouping=True)
    assert patched == 3
    assert model._loraforge_grouped_mlp_count == 1
    with torch.no_grad():
        for rows in (1, 8, 128, 300):
            x = torch.randn(rows, 256, device=DEV, dtype=dtype)
            want = reference(x).float()
            got = model(x).float()
            rel = float((got - want).abs().max() / want.abs().max().clamp_min(1e-6))
            assert rel < 4e-2, (rows, rel)
    report = peft_plan_report(model)
    assert report["grouped_mlp_modules"] == 1
    # a zero scaling falls back to the base linear exactly
    model.down_proj.scaling["default"] = 0.0
    with torch.no_grad():
        h = torch.randn(4, 512, device=DEV, dtype=dtype)
        assert torch.equal(model.down_proj(h), fused_linear._base_linear(h, model.down_proj.base_layer.weight, None))
