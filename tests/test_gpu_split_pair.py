"""Split-K CTA-pair GEMM (GPU): few 256x256 output tiles, K split over a cluster.

Reached through lora_linear_small for 128 < M <= 256 with rank <= 64 (the
shrink accumulated beside the base tile, the partial tiles exchanged through
the caller's workspace).  Each case is checked against the float64 oracle
(oracle/lora_oracle.py); the slice count is forced both ways through
LORA_B200_SPLIT_PAIR so that the 2-, 3- and 4-slice reductions and the
single-slice form (no exchange; chosen on its own for wide outputs) all run.  Shapes
cover partial token tiles (M not a multiple of 256), output widths that are
not multiples of 256 or of 8, ranks 1, 16, 17, 32, 48 and 64 (the wider
shrink accumulator), bias and no bias, fp16.
"""

import math

import pytest
import torch

from oracle import lora_oracle as orc
from probe_b200 import _lib, kernels
from tests.helpers import assert_parity, np64, randn

pytestmark = pytest.mark.gpu


def _case(m, n, k, r, dtype, seed):
    x = randn((m, k), 1.0, dtype, seed=seed)
    w = randn((n, k), 1 / math.sqrt(k), dtype, seed=seed + 1)
    bias = randn((n,), 1.0, dtype, seed=seed + 2)
    a = randn((r, k), 1 / math.sqrt(k), dtype, seed=seed + 3) if r else None
    b = randn((n, r), 1 / math.sqrt(max(r, 1)), dtype, seed=seed + 4) if r else None
    return x, w, bias, a, b


@pytest.mark.parametrize("slices", ["1", "2", "3", "4", ""])
@pytest.mark.parametrize("m,n,k,r", [(256, 4096, 4096, 16), (129, 1000, 2048, 1), (200, 1002, 1024, 17),
                                     (256, 512, 4096, 32), (160, 4096, 1536, 0), (256, 4096, 4096, 64),
                                     (231, 1000, 2048, 48), (129, 4096, 1024, 33), (256, 12288, 1024, 48)])
def test_linear_split_fused_shrink(monkeypatch, slices, m, n, k, r):
    monkeypatch.setenv("LORA_B200_SPLIT_PAIR", slices)
    dtype = torch.bfloat16
    x, w, bias, a, b = _case(m, n, k, r, dtype, seed=m + n)
    out = kernels.linear_small(x, w, a, b, bias, 1.7)
    assert out is not None
    want = orc.naive_linear(np64(x), np64(w), np64(bias), np64(a) if r else None, np64(b) if r else None, 1.7)
    assert_parity(out, want, dtype)
    assert torch.equal(out, kernels.linear_small(x, w, a, b, bias, 1.7))  # deterministic reduction
    assert _lib.device_error() == 0


def test_linear_split_single_slice_waves():
    """An output of 112 tiles of 256 x 256: more CTA pairs than SMs, so the
    single-slice form runs in two waves."""
    m, n, k, r = 256, 28672, 1024, 16
    dtype = torch.bfloat16
    x, w, bias, a, b = _case(m, n, k, r, dtype, seed=21)
    out = kernels.linear_small(x, w, a, b, bias, 0.75)
    assert out is not None
    want = orc.naive_linear(np64(x), np64(w), np64(bias), np64(a), np64(b), 0.75)
    assert_parity(out, want, dtype)
    assert _lib.device_error() == 0


def test_linear_split_rank64_fp16_strided():
    """fp16 at rank 64 (two 64-wide K atoms in the expand), lora_B with a row
    pitch wider than its rank, no bias."""
    m, n, k, r = 256, 1536, 4096, 64
    dtype = torch.float16
    x, w, _, a, _ = _case(m, n, k, r, dtype, seed=9)
    b = randn((n, 72), 1 / math.sqrt(r), dtype, seed=10)[:, :r]
    res = kernels.linear_small(x, w, a, b, None, 0.25)
    assert res is not None
    want = orc.naive_linear(np64(x), np64(w), None, np64(a), np64(b), 0.25)
    assert_parity(res, want, dtype)
    assert _lib.device_error() == 0


def test_linear_split_fp16_no_bias_strided_b():
    """fp16, no bias, lora_B with a row pitch wider than its rank."""
    m, n, k, r = 250, 768, 2048, 20
    dtype = torch.float16
    x, w, _, a, _ = _case(m, n, k, r, dtype, seed=5)
    b_full = randn((n, 40), 1 / math.sqrt(r), dtype, seed=6)
    b = b_full[:, :r]
    out = torch.full((m, n), float("nan"), device="cuda", dtype=dtype)
    res = kernels.linear_small(x, w, a, b, None, 0.5, out=out)
    assert res is not None
    want = orc.naive_linear(np64(x), np64(w), None, np64(a), np64(b), 0.5)
    assert_parity(res, want, dtype)
    assert _lib.device_error() == 0


def test_split_small_workspace_takes_skinny_kernel():
    """A NULL or short workspace makes lora_linear_small run the skinny kernel
    instead: same results within tolerance."""
    import ctypes

    m, n, k, r = 256, 1024, 2048, 16
    dtype = torch.bfloat16
    x, w, bias, a, b = _case(m, n, k, r, dtype, seed=9)
    lib = _lib.load()
    need = lib.lora_linear_small_workspace_size(m, n, r)
    assert need > 0
    want = orc.naive_linear(np64(x), np64(w), np64(bias), np64(a), np64(b), 1.25)
    for ws_bytes in (0, need - 16):
        ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
        out = torch.empty((m, n), device="cuda", dtype=dtype)
        rc = lib.lora_linear_small(_lib.ptr(x), k, _lib.ptr(w), k, _lib.ptr(a), k, _lib.ptr(b), r, _lib.ptr(bias),
                                   _lib.ptr(out), n, m, n, k, r, ctypes.c_float(1.25), _lib.LORA_BF16,
                                   _lib.ptr(ws) if ws_bytes else None, ws_bytes, _lib.stream_handle(x.device))
        assert rc == 0
        assert_parity(out, want, dtype)
    assert _lib.device_error() == 0


def test_split_repeated_with_other_kernels_between():
    """The partial exchange reuses one workspace and lora_B is staged in shared
    memory the pipeline also uses: repeated runs with unrelated launches in
    between and a NaN-filled output agree bit for bit."""
    m, n, k, r = 256, 2304, 3072, 16
    dtype = torch.bfloat16
    x, w, bias, a, b = _case(m, n, k, r, dtype, seed=77)
    first = kernels.linear_small(x, w, a, b, bias, 1.0)
    for i in range(3):
        junk = torch.randn(4096, 4096, device="cuda").to(dtype)
        kernels.gemm(junk, junk)
        out = torch.full_like(first, float("nan"))
        kernels.linear_small(x, w, a, b, bias, 1.0, out=out)
        assert torch.equal(out, first)
    want = orc.naive_linear(np64(x), np64(w), np64(bias), np64(a), np64(b), 1.0)
    assert_parity(first, want, dtype)
    assert _lib.device_error() == 0
