"""Parity of each CUDA entry point against the CPU oracle (GPU only).

Every call goes through the C ABI (probe_b200.kernels -> liblora_b200.so).
"""

import math

import numpy as np
import pytest
import torch

from oracle import lora_oracle as orc
from probe_b200 import _lib, kernels
from probe_b200.kernels import pad_cols, round_up
from tests.helpers import assert_parity, np64, randn

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float16]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 1024), (300, 320, 320), (1000, 1536, 768),
                                   (129, 200, 136), (64, 4096, 512)])
@pytest.mark.parametrize("r", [0, 7, 16, 130])
def test_gemm_kconcat(dtype, m, n, k, r):
    x = randn((m, k), 1.0, dtype, seed=1)
    w = randn((n, k), 1 / math.sqrt(k), dtype, seed=2)
    bias = randn((n,), 1.0, dtype, seed=3)
    if r:
        a = randn((r, k), 1 / math.sqrt(k), dtype, seed=4)
        b = randn((n, r), 1 / math.sqrt(r), dtype, seed=5)
        width = round_up(r, 64)
        # z = scale * x a^T rounded to dtype, zero tail (what the shrink produces)
        z64 = orc.shrink(np64(x), np64(a), 0.75)
        z = torch.zeros((m, width), dtype=dtype, device="cuda")
        z[:, :r] = torch.from_numpy(z64).to(dtype).cuda()
        out = kernels.gemm(x, w, z, pad_cols(b, width), rank=r, bias=bias)
        want = np64(x) @ np64(w).T + np64(z)[:, :r] @ np64(b).T + np64(bias)
    else:
        out = kernels.gemm(x, w, bias=bias)
        want = orc.naive_linear(np64(x), np64(w), np64(bias), None, None, 0.0)
    torch.cuda.synchronize()
    assert_parity(out, want, dtype)


@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (384, 640, 1280)])
def test_gemm_alpha_no_bias(m, n, k):
    x = randn((m, k), 1.0, seed=11)
    w = randn((n, k), 1 / math.sqrt(k), seed=12)
    out = kernels.gemm(x, w, alpha=0.5)
    assert_parity(out, 0.5 * (np64(x) @ np64(w).T))


def test_gemm_rejects_unaligned_k():
    x = randn((128, 100), 1.0)
    w = randn((64, 100), 0.1)
    with pytest.raises(ValueError):
        kernels.gemm(x, w)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m", [1, 4, 16, 33, 64, 200, 1000])
@pytest.mark.parametrize("k,r", [(4096, 16), (257, 7), (1536, 64), (640, 1), (768, 40), (512, 128)])
@pytest.mark.parametrize("split_k", [0, 1, 3])
def test_shrink(dtype, m, k, r, split_k):
    x = randn((m, k), 1.0, dtype, seed=m + r)
    a = randn((r, k), 1 / math.sqrt(k), dtype, seed=k)
    width = round_up(r, 64)
    z = kernels.shrink(x, a, 1.5, z_dtype=torch.float32, z_width=width, split_k=split_k)
    want = np.zeros((m, width))
    want[:, :r] = orc.shrink(np64(x), np64(a), 1.5)
    g = np64(z)
    assert np.array_equal(g[:, r:], np.zeros_like(g[:, r:]))
    # fp32 accumulation over K: relative error ~ sqrt(K) * 2^-24 (4e-6 at K = 4096)
    _, fro = orc.parity(g, want)
    assert fro < 2e-5, fro
    zq = kernels.shrink(x, a, 1.5, z_dtype=dtype, split_k=split_k)
    assert_parity(zq, want[:, :r], dtype)
    # hi/lo pair: hi is the rounded z, hi + lo carries ~16 mantissa bits
    zs = kernels.shrink(x, a, 1.5, z_dtype=dtype, z_width=width, z_split=True, split_k=split_k)
    assert zs.shape == (m, 2 * width)
    assert torch.equal(zs[:, :r], zq)
    pair = np64(zs[:, :width]) + np64(zs[:, width:])
    _, fro = orc.parity(pair, want)
    assert fro < 2e-5, fro


def test_shrink_deterministic():
    x = randn((64, 4096), 1.0, seed=5)
    a = randn((16, 4096), 1 / 64, seed=6)
    z1 = kernels.shrink(x, a, 1.0, split_k=16)
    z2 = kernels.shrink(x, a, 1.0, split_k=16)
    assert torch.equal(z1, z2)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n,r", [(1, 11008, 16), (4, 512, 13), (64, 1280, 24), (200, 4096, 64),
                                   (37, 259, 3), (128, 1000, 128), (16, 384, 224)])
@pytest.mark.parametrize("layout", ["peft", "rank_major"])
def test_expand_add(dtype, m, n, r, layout):
    y = randn((m, n), 1.0, dtype, seed=7)
    z = randn((m, r), 1.0, torch.float32, seed=8)
    b = randn((n, r), 1 / math.sqrt(r), dtype, seed=9)
    bias = randn((n,), 1.0, dtype, seed=10)
    bb = b if layout == "peft" else b.t().contiguous()
    y0 = y.clone()
    out = kernels.expand_add(y, z, bb, 0.5, bias=bias, b_layout=layout)
    assert torch.equal(y, y0)
    # an fp32 z is carried as a hi/lo pair up to rank 128 (rounded above that)
    zq = np64(z) if r <= 128 else orc.round_dtype(np64(z).astype(np.float32),
                                                   "bf16" if dtype == torch.bfloat16 else "f16")
    want = orc.expand_add(np64(y), zq, np64(b), 0.5, np64(bias))
    assert_parity(out, want, dtype)
    out2 = kernels.expand_add(None, z, bb, 0.5, b_layout=layout, dtype=dtype)
    assert_parity(out2, orc.expand_add(None, zq, np64(b), 0.5), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,k,n", [(1, 257, 131), (4, 1536, 512), (8, 769, 259), (16, 4096, 11008),
                                   (64, 4096, 1024), (33, 512, 300)])
@pytest.mark.parametrize("r", [0, 1, 13, 16, 64])
def test_decode_linear(dtype, m, k, n, r):
    x = randn((m, k), 1.0, dtype, seed=m)
    w = randn((n, k), 1 / math.sqrt(k), dtype, seed=n)
    bias = randn((n,), 1.0, dtype, seed=3)
    a = randn((r, k), 1 / math.sqrt(k), dtype, seed=4) if r else None
    b = randn((n, r), 1 / math.sqrt(max(r, 1)), dtype, seed=5) if r else None
    z = kernels.shrink(x, a, 1.0, z_dtype=torch.float32) if r else None
    out = kernels.decode_linear(x, w, z, b, bias, -0.7)
    want = orc.naive_linear(np64(x), np64(w), np64(bias), np64(a) if r else None, np64(b) if r else None, -0.7)
    assert_parity(out, want, dtype)
    # with z rounded to the input dtype first, the reference's decode semantics
    if r:
        zr = kernels.shrink(x, a, 1.0, z_dtype=dtype)
        tag = "bf16" if dtype == torch.bfloat16 else "f16"
        want_r = orc.decode_linear(np64(x), np64(w), np64(bias), np64(a), np64(b), -0.7, tag)
        assert_parity(kernels.decode_linear(x, w, zr, b, bias, -0.7), want_r, dtype)


@pytest.mark.parametrize("m,k,n,r,split", [(65, 512, 384, 16, 0), (128, 4096, 4096, 16, 0), (200, 1024, 1000, 40, 3),
                                           (256, 4096, 4096, 16, 2), (17, 2048, 11008, 128, 8),
                                           (3, 320, 200, 72, 1), (256, 128, 130, 8, 0), (256, 256, 512, 0, 0),
                                           (4, 256, 512, 0, 0), (100, 512, 640, 0, 5), (256, 256, 512, 3, 0)])
def test_decode_linear_tensor_core_path(m, k, n, r, split):
    """Token counts up to 256, ranks 0 and across one and two 64-wide tail chunks,
    and clusters of 1..8 K slices (the tensor-core path of lora_decode_linear).
    Rank 0 with 128-token tiles and a 2-deep pipeline is the layout where the
    fp32 partial tile is larger than the operand buffers it reuses."""
    dtype = torch.bfloat16
    x = randn((m, k), 1.0, dtype, seed=m + 1)
    w = randn((n, k), 1 / math.sqrt(k), dtype, seed=n + 1)
    bias = randn((n,), 1.0, dtype, seed=7)
    a = randn((r, k), 1 / math.sqrt(k), dtype, seed=8) if r else None
    b = randn((n, r), 1 / math.sqrt(max(r, 1)), dtype, seed=9) if r else None
    z = kernels.shrink(x, a, 1.0, z_dtype=torch.float32) if r else None
    out = kernels.decode_linear(x, w, z, b, bias, 1.3, split_k=split)
    want = orc.naive_linear(np64(x), np64(w), np64(bias), np64(a) if r else None, np64(b) if r else None, 1.3)
    assert_parity(out, want, dtype)
    again = kernels.decode_linear(x, w, z, b, bias, 1.3, split_k=split)
    assert torch.equal(out, again)  # cluster reduction in rank order: deterministic
    assert _lib.device_error() == 0


@pytest.mark.parametrize("m,k,n,r", [(1, 4096, 11008, 16), (4, 320, 1000, 7), (16, 4096, 4096, 64), (17, 1536, 512, 65),
                                     (64, 4096, 11008, 16), (65, 512, 384, 128), (128, 4096, 4096, 16),
                                     (200, 1024, 1000, 40), (256, 4096, 4096, 16), (3, 64, 96, 1), (33, 256, 130, 0)])
def test_linear_small_fused_shrink(m, k, n, r):
    """One kernel: W streamed once, x . A^T accumulated beside it and reduced over
    the cluster, the expand as the last slice's tail (lora_linear_small)."""
    dtype = torch.bfloat16
    x = randn((m, k), 1.0, dtype, seed=m + 3)
    w = randn((n, k), 1 / math.sqrt(k), dtype, seed=n + 3)
    bias = randn((n,), 1.0, dtype, seed=11)
    a = randn((r, k), 1 / math.sqrt(k), dtype, seed=12) if r else None
    b = randn((n, r), 1 / math.sqrt(max(r, 1)), dtype, seed=13) if r else None
    out = kernels.linear_small(x, w, a, b, bias, 0.9)
    assert out is not None
    want = orc.naive_linear(np64(x), np64(w), np64(bias), np64(a) if r else None, np64(b) if r else None, 0.9)
    assert_parity(out, want, dtype)
    assert torch.equal(out, kernels.linear_small(x, w, a, b, bias, 0.9))
    assert _lib.device_error() == 0


@pytest.mark.parametrize("r", [65, 67, 33])
def test_linear_small_odd_rank_pitch_repeated(r):
    """lora_B with an odd row pitch is staged element by element, which runs the
    last CTA's warps out of step; ranks above 64 need two rank chunks and the
    K split a cluster of several CTAs.  Repeated with other kernels in between
    and the output pre-filled with NaN, so no result can come from memory a
    previous launch left behind."""
    m, k, n = 17, 1536, 512
    dtype = torch.bfloat16
    x = randn((m, k), 1.0, dtype, seed=41)
    w = randn((n, k), 1 / math.sqrt(k), dtype, seed=42)
    a = randn((r, k), 1 / math.sqrt(k), dtype, seed=43)
    b = randn((n, r), 1 / math.sqrt(r), dtype, seed=44)
    assert b.stride(0) == r
    want = orc.naive_linear(np64(x), np64(w), None, np64(a), np64(b), 0.9)
    for _ in range(6):
        torch.empty(1 << 27, dtype=torch.uint8, device="cuda").fill_(0xAB)
        out = torch.full((m, n), float("nan"), device="cuda", dtype=dtype)
        kernels.linear_small(x, w, a, b, None, 0.9, out=out)
        assert_parity(out, want, dtype)
    assert _lib.device_error() == 0


def test_linear_small_declines_unaligned():
    x = randn((4, 257), 1.0, seed=1)
    w = randn((64, 257), 0.05, seed=2)
    assert kernels.linear_small(x, w, None, None, None, 0.0) is None


def test_decode_zero_rank_is_base():
    x = randn((4, 1536), 1.0, seed=1)
    w = randn((512, 1536), 1 / 40, seed=2)
    base = kernels.decode_linear(x, w, None, None, None, 0.0)
    a = randn((8, 1536), 1 / 40, seed=3)
    b = torch.zeros((512, 8), dtype=torch.bfloat16, device="cuda")
    z = kernels.shrink(x, a, 1.0, z_dtype=torch.bfloat16)
    with_zero_b = kernels.decode_linear(x, w, z, b, None, 1.0)
    assert torch.equal(base, with_zero_b)


def test_gemm_hi_lo_epilogue():
    m, n, k = 300, 224, 512
    x = randn((m, k), 1.0, seed=21)
    w = randn((n, k), 1 / math.sqrt(k), seed=22)
    z = torch.empty((m, 2 * n), dtype=torch.bfloat16, device="cuda")
    kernels.gemm(x, w, alpha=0.7, out=z[:, :n], lo_offset=n)
    want = 0.7 * (np64(x) @ np64(w).T)
    assert_parity(z[:, :n], want)
    _, fro = orc.parity(np64(z[:, :n]) + np64(z[:, n:]), want)
    assert fro < 2e-5, fro


def test_pair_gemm_narrow_wide_output():
    """A 224-wide output with the hi/lo epilogue on CTA-pair tiles (the rank
    shrink of a stacked r = 224 adapter at large M): one 256-wide tile per pair,
    columns 224..255 and rows past M clipped."""
    m, n, k = 19000, 224, 256
    x = randn((m, k), 1.0, seed=31)
    w = randn((n, k), 1 / math.sqrt(k), seed=32)
    z = torch.empty((m, 2 * n), dtype=torch.bfloat16, device="cuda")
    kernels.gemm(x, w, alpha=0.5, out=z[:, :n], lo_offset=n)
    rows = np.r_[0:64, 9000:9100, m - 70:m]
    want = 0.5 * (np64(x)[rows] @ np64(w).T)
    got = np64(z[:, :n])[rows] + np64(z[:, n:])[rows]
    _, fro = orc.parity(got, want)
    assert fro < 2e-5, fro
    assert_parity(z[:, :n][torch.as_tensor(rows, device="cuda")], want)
    assert _lib.device_error() == 0


def test_workspace_reuse_across_shapes():
    """Split-K tickets stay valid when one workspace serves calls of different shapes."""
    torch.manual_seed(3)
    cases = [(64, 256, 192, 16), (33, 128, 96, 7), (8, 4096, 11008, 16), (1, 640, 64, 3), (64, 256, 192, 16)]
    for rep in range(2):
        for m, k, n, r in cases:
            x = randn((m, k), 1.0, seed=m + rep)
            w = randn((n, k), 1 / math.sqrt(k), seed=n)
            a = randn((r, k), 1 / math.sqrt(k), seed=r)
            b = randn((n, r), 1 / math.sqrt(r), seed=r + 1)
            z = kernels.shrink(x, a, 1.0, z_dtype=torch.float32, split_k=4)
            out = kernels.decode_linear(x, w, z, b, None, 0.5, split_k=3)
            assert_parity(out, orc.naive_linear(np64(x), np64(w), None, np64(a), np64(b), 0.5))
    assert _lib.device_error() == 0


def test_device_error_word_clear():
    assert _lib.device_error() == 0
