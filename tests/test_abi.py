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


def _host_calls():
    """Each drop-in surface called with host tensors; the reference raises the
    same way (assertions on x.is_cuda in fused_lora.py / splitk_lora.py,
    ValueError in decode_linear.py:89-99)."""
    import importlib

    import torch

    fl = importlib.import_module("probe_b200.fused_lora")
    from probe_b200 import decode_linear, fused_linear, multilora, ragged_branch, segmented_branch, splitk_lora, \
        splitk_shrink

    x = torch.randn(4, 64, dtype=torch.bfloat16)
    w = torch.randn(32, 64, dtype=torch.bfloat16)
    a = torch.randn(2, 64, dtype=torch.bfloat16)
    b = torch.randn(32, 2, dtype=torch.bfloat16)
    y = torch.randn(4, 32, dtype=torch.bfloat16)
    z = torch.randn(4, 2, dtype=torch.bfloat16)
    offs, ranks, ids = torch.tensor([0]), torch.tensor([2]), torch.zeros(4, dtype=torch.long)
    bf = b.T.contiguous()
    return {
        "fused_lora": lambda: fl.fused_lora(x, a, b, y, 1.0),
        "tiled_lora": lambda: fl.tiled_lora(x, a, b, y, 1.0),
        "splitk_lora_shrink": lambda: splitk_lora.splitk_lora_shrink(x, a),
        "persistent_expand_add": lambda: splitk_lora.persistent_expand_add(z, b, y, 1.0),
        "shrink_partial": lambda: splitk_shrink.shrink_partial(x, a),
        "shrink_ragged": lambda: multilora.shrink_ragged(x, a, offs, ranks, ids, 2),
        "segmented_branch_varlen": lambda: segmented_branch.segmented_branch_varlen(
            x, y, a, bf, offs, ranks, torch.tensor([0, 4]), torch.tensor([0]), 2),
        "ragged_branch": lambda: ragged_branch.branch(x, y, a, bf, offs, ranks, ids, 2),
        "decode_lora_linear": lambda: decode_linear.decode_lora_linear(x, w, None, a, b, 1.0),
        "expand_add": lambda: fused_linear.expand_add(y, z, b, 1.0),
        "fused_gemm": lambda: fused_linear.fused_gemm(x, w, None, a, b, 1.0),
    }


@pytest.mark.parametrize("name", sorted(_host_calls()))
def test_every_drop_in_refuses_host_tensors(name):
    """No CPU fallback anywhere on the product path: host tensors raise."""
    with pytest.raises((RuntimeError, AssertionError, ValueError)):
        _host_calls()[name]()
