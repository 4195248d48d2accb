"""ctypes binding of ``liblora_b200.so`` (the C ABI declared in include/lora_b200.h).

Every GPU computation in this package goes through the functions below; there
is no Triton, cuBLAS or CPU fallback.  If the shared library is missing or the
tensors are not on an sm_100 CUDA device, the call raises.

Helpers here translate torch tensors into (pointer, leading dimension, dtype
code) triples, pick the caller's current CUDA stream, and hold the per-stream
workspaces whose split-K ticket counters must start at zero.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

from . import _build

LORA_OK = 0
LORA_ERR_SHAPE = 1
LORA_ERR_ALIGN = 2
LORA_ERR_DTYPE = 3
LORA_ERR_DEVICE = 4
LORA_ERR_INDEX = 5
LORA_ERR_CUDA = 6
LORA_ERR_TIMEOUT = 7
LORA_ERR_WORKSPACE = 8
LORA_ERR_UNSUPPORTED = 9
LORA_ERR_ARG = 10

LORA_F16 = 0
LORA_BF16 = 1
LORA_F32 = 2

LORA_B_PEFT = 0
LORA_B_RANK_MAJOR = 1

# Every symbol declared in include/lora_b200.h: name -> (restype, argtypes).
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t
SIGNATURES = {
    "lora_b200_abi_version": (_I, []),
    "lora_b200_status_string": (ctypes.c_char_p, [_I]),
    "lora_b200_device_error": (_I, [_I, ctypes.POINTER(_I)]),
    "lora_gemm": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _I64, _I,
                       _P]),
    "lora_gemm_workspace_size": (_SZ, [_I64, _I64, _I64, _I64]),
    "lora_gemm_ex": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _I64,
                          _I, _P, _SZ, _P]),
    "lora_shrink_workspace_size": (_SZ, [_I64, _I64, _I]),
    "lora_shrink_pick_split_k": (_I, [_I64, _I64, _I64]),
    "lora_shrink": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _I64, _I, _I64, _I64, _I64, _F, _I, _I, _P, _SZ, _P]),
    "lora_shrink_static_scratch_capacity": (_SZ, []),
    "lora_shrink_static_scratch": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _I64, _I, _I64, _I64, _I64, _F, _I, _I,
                                        _P]),
    "lora_expand_add": (_I, [_P, _I64, _P, _I64, _I, _P, _I64, _I, _P, _P, _I64, _I64, _I64, _I64, _F, _I, _P]),
    "lora_decode_workspace_size": (_SZ, [_I64, _I64, _I]),
    "lora_decode_pick_split_k": (_I, [_I64, _I64, _I64]),
    "lora_decode_linear": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                _F, _I, _I, _P, _SZ, _P]),
    "lora_linear_small_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "lora_linear_small": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _F,
                               _I, _P, _SZ, _P]),
    "lora_sgmv_tiles_size": (_SZ, [_I64, _I64]),
    "lora_sgmv_schedule": (_I, [_P, _P, _P, _I64, _I64, _I64, _P, _SZ, _P]),
    "lora_sgmv_shrink_workspace_size": (_SZ, [_I64, _I64, _I64, _I]),
    "lora_sgmv_pick_split_k": (_I, [_I64, _I64, _I64]),
    "lora_sgmv_shrink": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _P, _P, _P, _I64, _I, _I64, _I64, _I64, _I64, _I64,
                              _F, _I, _I, _P, _SZ, _P]),
    "lora_sgmv_shrink_ex": (_I, [_P, _I64, _P, _I64, _I64, _P, _P, _I64, _P, _P, _P, _I64, _I, _I64, _I64, _I64,
                                 _I64, _I64, _F, _I, _I, _P, _SZ, _P]),
    "lora_sgmv_expand": (_I, [_P, _I64, _P, _I64, _I, _P, _I64, _I64, _P, _P, _I64, _P, _P, _P, _I64, _I64, _I64,
                              _I64, _I64, _F, _I, _P]),
    "lora_sgmv_branch_workspace_size": (_SZ, [_I64, _I64, _I64, _I64]),
    "lora_sgmv_branch": (_I, [_P, _I64, _P, _I64, _P, _I64, _I64, _P, _I64, _I64, _P, _P, _I64, _P, _P, _I64, _I64,
                              _I64, _I64, _I64, _I64, _F, _I, _P, _SZ, _P]),
    "lora_sgmv_linear_workspace_size": (_SZ, [_I64, _I64, _I64, _I64]),
    "lora_sgmv_linear": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _I64, _P, _I64, _I64, _P, _P, _I64, _P, _P, _I64, _I64,
                              _I64, _I64, _I64, _I64, _F, _I, _P, _SZ, _P]),
}


class LoraError(RuntimeError):
    """A lora_b200 entry point returned a non-zero status."""

    def __init__(self, status: int, func: str, detail: str = ""):
        self.status = status
        name = _STATUS_NAMES.get(status, f"status {status}")
        super().__init__(f"{func}: {name}{': ' + detail if detail else ''}")


class LoraValueError(LoraError, ValueError):
    """Shape, alignment, index or argument rejected by the C ABI."""


_STATUS_NAMES = {
    LORA_ERR_SHAPE: "shape",
    LORA_ERR_ALIGN: "alignment",
    LORA_ERR_DTYPE: "dtype",
    LORA_ERR_DEVICE: "device (needs an sm_100 GPU)",
    LORA_ERR_INDEX: "index out of range",
    LORA_ERR_CUDA: "CUDA error",
    LORA_ERR_TIMEOUT: "device wait timed out",
    LORA_ERR_WORKSPACE: "workspace",
    LORA_ERR_UNSUPPORTED: "unsupported",
    LORA_ERR_ARG: "invalid argument",
}

_lib = None
_lib_lock = threading.Lock()


def library_path() -> Path:
    return _build.LIB_PATH


def load(build_if_missing: bool = False):
    """Load the shared library (raises if it is missing and not built here)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            if not build_if_missing:
                raise RuntimeError(
                    f"{path} is missing: build the CUDA extension with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` (or probe_b200._build.build())"
                )
            _build.build()
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int, func: str, detail: str = "") -> None:
    if status == LORA_OK:
        return
    if status in (LORA_ERR_SHAPE, LORA_ERR_ALIGN, LORA_ERR_ARG, LORA_ERR_INDEX, LORA_ERR_DTYPE):
        raise LoraValueError(status, func, detail)
    raise LoraError(status, func, detail)


def call(func: str, *args, detail: str = "") -> None:
    lib = load()
    check(getattr(lib, func)(*args), func, detail)


# --------------------------------------------------------------------- tensors
def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return LORA_BF16
    if dtype == torch.float16:
        return LORA_F16
    if dtype == torch.float32:
        return LORA_F32
    raise TypeError(f"unsupported dtype {dtype}: the LoRA kernels take bfloat16 or float16")


def require_cuda(*tensors: torch.Tensor, where: str = "lora_b200") -> None:
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                f"{where}: tensors must be on a CUDA (sm_100) device; this build has no CPU path")


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def row_major(t: torch.Tensor) -> torch.Tensor:
    """A 2-D view with unit inner stride (copies only when needed)."""
    if t.dim() != 2:
        raise ValueError(f"expected a 2-D tensor, got shape {tuple(t.shape)}")
    if t.stride(1) != 1 or t.stride(0) < t.shape[1] or t.stride(0) == 0:
        t = t.contiguous()
    return t


def ld(t: torch.Tensor) -> int:
    return t.stride(0) if t.shape[0] > 1 else max(t.stride(0), t.shape[1])


def stream_handle(device: torch.device | None = None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


# ------------------------------------------------------------------ workspaces
class _Workspace:
    """Zero-initialised byte buffers, one per (device, stream, slot).

    The split-K kernels leave their ticket counters at zero when they finish,
    so a buffer stays valid for every later call on the same stream.  Calls on
    one stream are ordered, so they never share a buffer concurrently.  A
    buffer only grows (by allocating a new zeroed one); warm the shapes you
    will capture before capturing a CUDA graph.
    """

    def __init__(self):
        self._bufs: dict[tuple, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, nbytes: int, device: torch.device, slot: str) -> torch.Tensor:
        stream = torch.cuda.current_stream(device).cuda_stream
        key = (device.index, stream, slot)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(int(nbytes), 1 << 12)
                if buf is not None:
                    size = max(size, buf.numel() * 2)
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf


WORKSPACE = _Workspace()


def device_error(device: int | None = None) -> int:
    """Read and clear the device-side error word (synchronises the device)."""
    lib = load()
    dev = torch.cuda.current_device() if device is None else device
    code = ctypes.c_int(0)
    check(lib.lora_b200_device_error(dev, ctypes.byref(code)), "lora_b200_device_error")
    return code.value
