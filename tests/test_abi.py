"""The C ABI library loads and exports every symbol include/lora_b200.h declares (CPU only)."""

import ctypes
import re
from pathlib import Path

import pytest

from probe_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "lora_b200.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^LORA_API\s+[\w\s\*]+?\b(lora_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "lora_gemm" in names and "lora_sgmv_expand" in names
    assert len(names) >= 16


def test_library_exports_every_declared_symbol(lib):
    for name in declared():
        assert hasattr(lib, name), name
    assert set(declared()) == set(_lib.SIGNATURES), "ctypes signatures and header disagree"


def test_abi_version_and_status_strings(lib):
    assert lib.lora_b200_abi_version() == 1
    assert lib.lora_b200_status_string(0) == b"ok"
    assert lib.lora_b200_status_string(5) == b"index out of range"


def test_workspace_sizes_are_host_only(lib):
    assert lib.lora_shrink_workspace_size(64, 16, 1) == 256
    assert lib.lora_shrink_workspace_size(64, 16, 4) >= 4 * 64 * 16 * 4
    assert lib.lora_decode_workspace_size(8, 11008, 3) >= 3 * 8 * 11008 * 4
    # split-K pair kernel: only above 128 tokens and for ranks <= 64
    assert lib.lora_linear_small_workspace_size(256, 4096, 16) >= 16 * 2 * 4 * 3 * 128 * 64 * 4
    assert lib.lora_linear_small_workspace_size(128, 4096, 16) == 0
    assert lib.lora_linear_small_workspace_size(256, 4096, 40) == lib.lora_linear_small_workspace_size(256, 4096, 16)
    assert lib.lora_linear_small_workspace_size(256, 4096, 65) == 0
    assert lib.lora_sgmv_tiles_size(4096, 128) >= 4 * (2 + 2 * (64 + 128 + 1))


def test_argument_errors_without_gpu(lib):
    # NULL pointers and bad dtypes are rejected before any device work
    assert lib.lora_gemm(None, 0, None, 0, None, 0, None, 0, None, None, 0, 1, 1, 8, 0, 1.0, 0, 1,
                         None) == _lib.LORA_ERR_ARG
    p = ctypes.c_void_p(16)
    assert lib.lora_shrink(p, 8, p, 8, p, 8, 7, 8, 0, 1, 8, 4, 1.0, 1, 1, None, 0, None) == _lib.LORA_ERR_DTYPE
    # a split (hi/lo) z must be 16-bit
    assert lib.lora_shrink(p, 8, p, 8, p, 16, _lib.LORA_F32, 8, 1, 1, 8, 4, 1.0, 1, 1, None, 0,
                           None) == _lib.LORA_ERR_ARG
    assert lib.lora_expand_add(p, 8, p, 8, 2, p, 8, 5, None, p, 8, 1, 8, 4, 1.0, 1, None) == _lib.LORA_ERR_ARG
    assert lib.lora_decode_linear(p, 8, p, 8, None, 0, 1, None, 0, None, p, 8, 257, 8, 8, 0, 1.0, 1, 0, None, 0,
                                  None) == _lib.LORA_ERR_SHAPE


def test_cpu_tensors_raise():
    import torch

    from probe_b200 import fused_lora_linear

    x = torch.randn(4, 8, dtype=torch.bfloat16)
    w = torch.randn(8, 8, dtype=torch.bfloat16)
    a = torch.randn(2, 8, dtype=torch.bfloat16)
    b = torch.randn(8, 2, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_lora_linear(x, w, None, a, b, 1.0)
