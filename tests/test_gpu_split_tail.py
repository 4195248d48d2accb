"""CTA-pair GEMM with a split tail (GPU): the tiles of the last partial wave
cut along K across the idle pairs, partials summed in a fixed order.

Shapes are picked so the tail is split (lora_gemm_workspace_size > 0, which
needs K >= 8192): the 8- and 4-way shards of the C5 FFN-down projection
(with the rank-224 hi/lo K-slice), a narrow output whose few tiles are all
split, both tile widths (256 and 512 columns), bias and alpha, and the hi/lo
output form of the large-rank shrink.  Each is checked against the float64 oracle, against the
same call without a workspace (no split), and for bit-identical repeats.
"""

import math

import numpy as np
import pytest
import torch

from oracle import lora_oracle as orc
from probe_b200 import _lib, kernels
from tests.helpers import assert_parity, np64, randn

pytestmark = pytest.mark.gpu


def _gemm_no_split(x, w, z=None, bw=None, rank=0, bias=None, alpha=1.0, lo_offset=0, out_cols=None):
    m, n = x.shape[0], w.shape[0]
    out = torch.empty((m, out_cols or n), device=x.device, dtype=x.dtype)
    _lib.call("lora_gemm", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(z) if rank else None,
              z.stride(0) if rank else 0, _lib.ptr(bw) if rank else None, bw.stride(0) if rank else 0,
              _lib.ptr(bias), _lib.ptr(out), out.stride(0), m, n, x.shape[1], rank, float(alpha), lo_offset,
              _lib.dtype_code(x.dtype), _lib.stream_handle(x.device))
    return out


SHAPES = [  # (M, K, N, R): long K (the tail splits only from K = 8192), for 74 resident pairs
    (4095, 13824, 5120, 448),  # C5 FFN-down shard at 8 GPUs (hi/lo tail of rank 224): 3 pieces
    (8190, 13824, 5120, 448),  # the same at 4 GPUs: 256x512 tiles, 3 pieces
    (2000, 8192, 8192, 0),     # 256x256 tiles, 2 pieces
    (1300, 16384, 4096, 0),    # 3 pieces
    (5000, 8192, 4096, 32),
    (4095, 13824, 224, 0),     # a narrow output on few tiles: every tile split (the rank-224 shrink)
]


def test_c5_shard_splits_its_tail():
    lib = _lib.load()
    assert lib.lora_gemm_workspace_size(4095, 5120, 13824, 448) > 0  # FFN down: long K
    assert lib.lora_gemm_workspace_size(4095, 5120, 5120, 448) == 0   # q: K too short to pay


@pytest.mark.parametrize("m,k,n,r", SHAPES)
def test_split_tail_gemm(m, k, n, r):
    lib = _lib.load()
    if lib.lora_gemm_workspace_size(m, n, k, r) == 0:
        pytest.skip("this device's pair capacity leaves no tail to split for this shape")
    x = randn((m, k), 1.0, seed=m)
    w = randn((n, k), 1 / math.sqrt(k), seed=n)
    z = randn((m, r), 0.5, seed=3) if r else None
    bw = randn((n, r), 0.2, seed=4) if r else None
    bias = randn((n,), 1.0, seed=5)
    got = kernels.gemm(x, w, z, bw, rank=r, bias=bias, alpha=0.75)
    again = kernels.gemm(x, w, z, bw, rank=r, bias=bias, alpha=0.75)
    torch.cuda.synchronize()
    assert torch.equal(got, again)  # fixed reduction order
    plain = _gemm_no_split(x, w, z, bw, rank=r, bias=bias, alpha=0.75)
    rows = torch.tensor(sorted({0, 1, m // 3, m // 2, m - 257, m - 256, m - 2, m - 1}), device="cuda")
    xs = np64(x.index_select(0, rows))
    want = 0.75 * (xs @ np64(w).T + (np64(z.index_select(0, rows)) @ np64(bw).T if r else 0.0)) + np64(bias)
    assert_parity(got.index_select(0, rows), want)
    # split and unsplit results differ only by fp32 summation order
    diff = (got.float() - plain.float()).abs()
    assert float(diff.max()) <= 2 * float(orc.half_ulp(np.array([float(plain.float().abs().max())]), "bf16")[0])
    assert _lib.device_error() == 0


@pytest.mark.parametrize("m,k,n", [(2000, 8192, 8192), (4095, 13824, 224)])
def test_split_tail_hilo_output(m, k, n):
    """The hi/lo output form ([round(v) | v - round(v)], the rank-224 shrink's)
    through the split tail's reduction."""
    if _lib.load().lora_gemm_workspace_size(m, n, k, 0) == 0:
        pytest.skip("no split tail for this shape on this device")
    x = randn((m, k), 1.0, seed=7)
    w = randn((n, k), 1 / math.sqrt(k), seed=8)
    z = torch.empty((m, 2 * n), device="cuda", dtype=torch.bfloat16)
    kernels.gemm(x, w, alpha=1.0, out=z[:, :n], lo_offset=n)
    hi, lo = np64(z[:, :n]), np64(z[:, n:])
    rows = [0, 100, 1024, m - 1]
    want = np64(x)[rows] @ np64(w).T
    assert np.abs((hi + lo)[rows] - want).max() < 1e-3 * max(1.0, np.abs(want).max())
