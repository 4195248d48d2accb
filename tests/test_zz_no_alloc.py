"""The shrink entry point that allocates nothing (GPU only).

lora_shrink_static_scratch serves callers that cannot call cudaMalloc --
serving loops that cannot pay cudaMalloc's device synchronisation, host
frameworks that own all device memory.  Its scratch is an array the library holds on the device.  This test
calls it through the C ABI and checks it against the workspace-taking
lora_shrink on two calls in a row with different shapes, so a second call that
found the first call's leftovers in the shared array would be caught.
"""

import ctypes
import math

import pytest
import torch

from probe_b200 import _lib, kernels
from tests.helpers import assert_parity, np64, randn

pytestmark = pytest.mark.gpu


def _static_shrink(x, a, scale, z_dtype, z_width, z_split, split_k):
    lib = _lib.load()
    m, k = x.shape
    r = a.shape[0]
    z = torch.empty((m, z_width * (2 if z_split else 1)), device=x.device, dtype=z_dtype)
    rc = lib.lora_shrink_static_scratch(
        ctypes.c_void_p(x.data_ptr()), x.stride(0), ctypes.c_void_p(a.data_ptr()), a.stride(0),
        ctypes.c_void_p(z.data_ptr()), z.stride(0), _lib.dtype_code(z_dtype), z_width, 1 if z_split else 0,
        m, k, r, scale, _lib.dtype_code(x.dtype), split_k,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.LORA_OK, lib.lora_b200_status_string(rc)
    return z


@pytest.mark.parametrize("split_k", [0, 4])
def test_static_scratch_shrink_matches_workspace_shrink(split_k):
    cases = [  # (M, K, R, z dtype, hi/lo split)
        (64, 4096, 16, torch.float32, False),
        (200, 1536, 64, torch.bfloat16, True),
    ]
    for m, k, r, zdt, split in cases:  # two calls in a row, different shapes
        x = randn((m, k), 1.0, seed=m)
        a = randn((r, k), 1 / math.sqrt(k), seed=r)
        width = ((r + 15) // 16) * 16
        got = _static_shrink(x, a, 0.75, zdt, width, split, split_k)
        want = kernels.shrink(x, a, 0.75, z_dtype=zdt, z_width=width, z_split=split, split_k=split_k)
        torch.cuda.synchronize()
        assert got.shape == want.shape
        # against the existing entry point and against the float64 product
        assert_parity(got[:, :r], np64(want[:, :r]), torch.bfloat16)
        assert_parity(got[:, :r], 0.75 * (np64(x) @ np64(a).T), torch.bfloat16)
        assert torch.count_nonzero(got[:, r:width]) == 0


def test_static_scratch_rejects_oversize_split():
    lib = _lib.load()
    assert lib.lora_shrink_static_scratch_capacity() == (8 << 20) - (16 << 10)
    m, k, r = 4096, 4096, 128  # 64 splits x 4096 x 128 x 4 B = 128 MiB, far beyond the array
    x = randn((m, k), 1.0, seed=1)
    a = randn((r, k), 1 / 64, seed=2)
    z = torch.empty((m, r), device="cuda", dtype=torch.float32)
    rc = lib.lora_shrink_static_scratch(
        ctypes.c_void_p(x.data_ptr()), k, ctypes.c_void_p(a.data_ptr()), k, ctypes.c_void_p(z.data_ptr()), r,
        _lib.LORA_F32, r, 0, m, k, r, 1.0, _lib.LORA_BF16, 64,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.LORA_ERR_WORKSPACE


def test_static_scratch_allocates_nothing():
    """After a first call has loaded the library's device code on this GPU,
    further calls change neither torch's allocator nor the device's free memory."""
    m, k, r = 128, 4096, 32
    x = randn((m, k), 1.0, seed=3)
    a = randn((r, k), 1 / 64, seed=4)
    _static_shrink(x, a, 1.0, torch.float32, r, False, 4)  # loads the module and the array
    lib = _lib.load()
    z = torch.empty((m, r), device=x.device, dtype=torch.float32)
    torch.cuda.synchronize()
    allocated, reserved = torch.cuda.memory_allocated(), torch.cuda.memory_reserved()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        rc = lib.lora_shrink_static_scratch(
            ctypes.c_void_p(x.data_ptr()), k, ctypes.c_void_p(a.data_ptr()), k, ctypes.c_void_p(z.data_ptr()), r,
            _lib.LORA_F32, r, 0, m, k, r, 1.0, _lib.LORA_BF16, 4,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == _lib.LORA_OK
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == allocated
    assert torch.cuda.memory_reserved() == reserved
    assert torch.cuda.mem_get_info()[0] == free_before
    assert_parity(z, np64(x) @ np64(a).T, torch.bfloat16)
