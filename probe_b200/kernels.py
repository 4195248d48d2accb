"""Torch-facing wrappers of the C ABI, one per entry point of include/lora_b200.h.

These take CUDA tensors, validate them, pick the caller's current stream and
call ``liblora_b200.so``.  The reference-compatible modules (fused_linear,
splitk_lora, multilora, ...) are written on top of these.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import LORA_B_PEFT, LORA_B_RANK_MAJOR, LORA_F32

GEMM_TAIL_ALIGN = 64  # K-slice width of the tcgen05 mainloop


def round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


def _dt(t: torch.Tensor) -> int:
    return _lib.dtype_code(t.dtype)


def _check_half(t: torch.Tensor, where: str) -> None:
    if t.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"{where}: expected float16/bfloat16, got {t.dtype}")


def pad_cols(t: torch.Tensor, width: int) -> torch.Tensor:
    """Copy of a 2-D tensor zero-padded (or kept) to ``width`` columns, row-major."""
    rows, cols = t.shape
    if cols == width and t.is_contiguous():
        return t
    out = torch.zeros((rows, width), device=t.device, dtype=t.dtype)
    out[:, :cols] = t
    return out


# ----------------------------------------------------------------------- GEMM
def gemm(x: torch.Tensor, w: torch.Tensor, z: torch.Tensor | None = None, bw: torch.Tensor | None = None,
         rank: int = 0, bias: torch.Tensor | None = None, alpha: float = 1.0,
         out: torch.Tensor | None = None, lo_offset: int = 0) -> torch.Tensor:
    """``out = alpha * (x @ w.T + z[:, :rank] @ bw[:, :rank].T) + bias`` on tcgen05.

    ``rank`` is the width of the K-slice tail (columns of z / bw beyond it are
    not read); rank == 0 is a plain linear.  ``lo_offset > 0`` writes the
    result as a hi/lo pair, the residual at column + lo_offset of ``out``.
    """
    _lib.require_cuda(x, w, where="gemm")
    _check_half(x, "gemm")
    if w.dtype != x.dtype or (bias is not None and bias.dtype != x.dtype):
        raise TypeError("gemm: x, w and bias must share one dtype")
    x = _lib.row_major(x)
    w = _lib.row_major(w)
    m, k = x.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"gemm: x {tuple(x.shape)} and w {tuple(w.shape)} disagree on K")
    if bias is not None:
        bias = bias.contiguous()
        if bias.shape != (n,):
            raise ValueError("gemm: bias must have out_features elements")
    if out is None:
        out = torch.empty((m, n), device=x.device, dtype=x.dtype)
    elif out.shape != (m, n) or out.stride(1) != 1 or out.dtype != x.dtype:
        raise ValueError("gemm: out must be a row-major [M, N] tensor of the input dtype")
    if lo_offset and out.stride(0) < n + lo_offset:
        raise ValueError("gemm: lo_offset needs out rows of at least N + lo_offset elements")
    if rank > 0:
        if z is None or bw is None or z.dtype != x.dtype or bw.dtype != x.dtype:
            raise ValueError("gemm: z and bw are required (input dtype) when rank > 0")
        z = _lib.row_major(z)
        bw = _lib.row_major(bw)
        if z.shape[0] != m or bw.shape[0] != n or z.shape[1] < rank or bw.shape[1] < rank:
            raise ValueError("gemm: z / bw must be [M|N, >= rank]")
    ws_bytes = _lib.load().lora_gemm_workspace_size(m, n, k, int(rank))
    ws = _lib.WORKSPACE.get(ws_bytes, x.device, "gemm") if ws_bytes else None
    _lib.call("lora_gemm_ex", _lib.ptr(x), _lib.ld(x), _lib.ptr(w), _lib.ld(w),
              _lib.ptr(z) if rank > 0 else None, _lib.ld(z) if rank > 0 else 0,
              _lib.ptr(bw) if rank > 0 else None, _lib.ld(bw) if rank > 0 else 0,
              _lib.ptr(bias), _lib.ptr(out), out.stride(0), m, n, k, int(rank), float(alpha), int(lo_offset), _dt(x),
              _lib.ptr(ws), ws.numel() if ws is not None else 0, _lib.stream_handle(x.device))
    return out


# --------------------------------------------------------------------- shrink
def shrink(x: torch.Tensor, a: torch.Tensor, scale: float = 1.0, z_dtype: torch.dtype | None = torch.float32,
           z_width: int | None = None, split_k: int = 0, out: torch.Tensor | None = None,
           z_split: bool = False) -> torch.Tensor:
    """Split-K ``z = scale * x @ a.T`` -> ``[M, z_width]`` (zeros beyond rank).

    ``z_split`` (input dtype only) appends the rounding residual, giving
    ``[round(z) | z - round(z)]`` of width ``2 * z_width``.
    """
    _lib.require_cuda(x, a, where="shrink")
    _check_half(x, "shrink")
    if a.dtype != x.dtype:
        raise TypeError("shrink: x and a must share one dtype")
    x = _lib.row_major(x)
    a = _lib.row_major(a)
    m, k = x.shape
    r = a.shape[0]
    if a.shape[1] != k:
        raise ValueError(f"shrink: x {tuple(x.shape)} and a {tuple(a.shape)} disagree on K")
    if r > 128:
        raise ValueError("shrink: rank above 128 goes through the tensor-core GEMM (gemm)")
    z_dtype = x.dtype if z_dtype is None else z_dtype
    width = r if z_width is None else int(z_width)
    if z_split and z_dtype == torch.float32:
        raise ValueError("shrink: z_split needs a 16-bit z")
    if out is None:
        out = torch.empty((m, width * (2 if z_split else 1)), device=x.device, dtype=z_dtype)
    if split_k <= 0:
        split_k = _lib.load().lora_shrink_pick_split_k(m, k, r)
    ws_bytes = _lib.load().lora_shrink_workspace_size(m, r, split_k)
    ws = _lib.WORKSPACE.get(ws_bytes, x.device, "shrink")
    _lib.call("lora_shrink", _lib.ptr(x), _lib.ld(x), _lib.ptr(a), _lib.ld(a), _lib.ptr(out), out.stride(0),
              _lib.dtype_code(out.dtype), width, 1 if z_split else 0, m, k, r, float(scale), _dt(x), int(split_k),
              _lib.ptr(ws), ws.numel(), _lib.stream_handle(x.device))
    return out


# --------------------------------------------------------------------- expand
def expand_add(y: torch.Tensor | None, z: torch.Tensor, b: torch.Tensor, scale: float = 1.0,
               bias: torch.Tensor | None = None, b_layout: str = "peft", rank: int | None = None,
               out: torch.Tensor | None = None, n: int | None = None, dtype: torch.dtype | None = None
               ) -> torch.Tensor:
    """``out = y + scale * z[:, :rank] @ B.T + bias`` (fresh output, never aliases y).

    ``b_layout`` is ``"peft"`` for lora_B.weight ``[N, R]`` or ``"rank_major"``
    for a ``[R, N]`` table.
    """
    _lib.require_cuda(z, b, y, where="expand_add")
    dtype = y.dtype if y is not None else (dtype or b.dtype)
    z = _lib.row_major(z)
    b = _lib.row_major(b)
    m = z.shape[0]
    if b_layout == "peft":
        nb, rb = b.shape
        lay = LORA_B_PEFT
    elif b_layout == "rank_major":
        rb, nb = b.shape
        lay = LORA_B_RANK_MAJOR
    else:
        raise ValueError(f"unknown b_layout {b_layout!r}")
    n = nb if n is None else n
    r = rb if rank is None else int(rank)
    if y is not None:
        y = _lib.row_major(y)
        if y.shape != (m, n):
            raise ValueError(f"expand_add: y {tuple(y.shape)} does not match [{m}, {n}]")
    if z.dtype not in (torch.float32, dtype) or b.dtype != dtype:
        raise TypeError("expand_add: z must be float32 or the activation dtype; b the activation dtype")
    if out is None:
        out = torch.empty((m, n), device=z.device, dtype=dtype)
    if bias is not None:
        bias = bias.contiguous()
    _lib.call("lora_expand_add", _lib.ptr(y), _lib.ld(y) if y is not None else 0, _lib.ptr(z), _lib.ld(z),
              _lib.dtype_code(z.dtype), _lib.ptr(b), _lib.ld(b), lay, _lib.ptr(bias), _lib.ptr(out), out.stride(0),
              m, n, r, float(scale), _lib.dtype_code(dtype), _lib.stream_handle(z.device))
    return out


# --------------------------------------------------------------------- decode
def decode_linear(x: torch.Tensor, w: torch.Tensor, z: torch.Tensor | None, b: torch.Tensor | None,
                  bias: torch.Tensor | None, scale: float, split_k: int = 0,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Small-M full linear ``x @ w.T + scale * z @ b.T + bias`` streaming W once."""
    _lib.require_cuda(x, w, where="decode_linear")
    _check_half(x, "decode_linear")
    x = _lib.row_major(x)
    w = _lib.row_major(w)
    m, k = x.shape
    n = w.shape[0]
    r = 0 if z is None else b.shape[1]
    if m > 256:
        raise ValueError("decode_linear: at most 256 rows")
    if out is None:
        out = torch.empty((m, n), device=x.device, dtype=x.dtype)
    if r > 0:
        z = _lib.row_major(z)
        b = _lib.row_major(b)
    if bias is not None:
        bias = bias.contiguous()
    lib = _lib.load()
    # the workspace covers the register path's split; split_k = 0 lets each path plan its own
    ws_split = split_k if split_k > 0 else lib.lora_decode_pick_split_k(m, n, k)
    ws_bytes = lib.lora_decode_workspace_size(m, n, ws_split)
    ws = _lib.WORKSPACE.get(ws_bytes, x.device, "decode")
    _lib.call("lora_decode_linear", _lib.ptr(x), _lib.ld(x), _lib.ptr(w), _lib.ld(w),
              _lib.ptr(z) if r > 0 else None, _lib.ld(z) if r > 0 else 0,
              _lib.dtype_code(z.dtype) if r > 0 else _dt(x), _lib.ptr(b) if r > 0 else None,
              _lib.ld(b) if r > 0 else 0, _lib.ptr(bias), _lib.ptr(out), out.stride(0), m, n, k, r, float(scale),
              _dt(x), int(split_k), _lib.ptr(ws), ws.numel(), _lib.stream_handle(x.device))
    return out


def linear_small(x: torch.Tensor, w: torch.Tensor, a: torch.Tensor | None, b: torch.Tensor | None,
                 bias: torch.Tensor | None, scale: float, out: torch.Tensor | None = None) -> torch.Tensor | None:
    """``x @ w.T + scale * (x @ a.T) @ b.T + bias`` for M <= 256 in ONE kernel (the
    shrink fused into the W stream).  Returns None when the shape or alignment is
    outside that kernel (then use shrink + decode_linear)."""
    _lib.require_cuda(x, w, where="linear_small")
    _check_half(x, "linear_small")
    x = _lib.row_major(x)
    w = _lib.row_major(w)
    m, k = x.shape
    n = w.shape[0]
    r = 0 if a is None or scale == 0 else a.shape[0]
    if m > 256 or r > 128:
        return None
    if r > 0:
        a = _lib.row_major(a)
        b = _lib.row_major(b)
    if bias is not None:
        bias = bias.contiguous()
    if out is None:
        out = torch.empty((m, n), device=x.device, dtype=x.dtype)
    lib = _lib.load()
    ws_bytes = lib.lora_linear_small_workspace_size(m, n, r)
    ws = _lib.WORKSPACE.get(ws_bytes, x.device, "small") if ws_bytes else None
    rc = lib.lora_linear_small(_lib.ptr(x), _lib.ld(x), _lib.ptr(w), _lib.ld(w), _lib.ptr(a) if r else None,
                               _lib.ld(a) if r else 0, _lib.ptr(b) if r else None, _lib.ld(b) if r else 0,
                               _lib.ptr(bias), _lib.ptr(out), out.stride(0), m, n, k, r, float(scale), _dt(x),
                               _lib.ptr(ws), ws_bytes, _lib.stream_handle(x.device))
    if rc == _lib.LORA_ERR_UNSUPPORTED:
        return None
    _lib.check(rc, "lora_linear_small")
    return out


# ----------------------------------------------------------------------- SGMV
def _i64(t: torch.Tensor, device) -> torch.Tensor:
    t = torch.as_tensor(t, device=device)
    if t.dtype != torch.int64:
        t = t.to(torch.int64)
    return t.contiguous()


def sgmv_schedule(t_total: int, n_adapters: int, ids: torch.Tensor | None = None,
                  seg_start: torch.Tensor | None = None, seg_adapter: torch.Tensor | None = None,
                  device=None) -> tuple[torch.Tensor, int]:
    """Build the device tile list; returns (tiles int32 tensor, S) with S = 0 for ids."""
    _lib.require_cuda(ids, seg_start, seg_adapter, where="sgmv_schedule")
    lib = _lib.load()
    if ids is not None:
        device = ids.device if device is None else device
        ids = _i64(ids, device)
        s = 0
    else:
        device = seg_start.device if device is None else device
        seg_start = _i64(seg_start, device)
        seg_adapter = _i64(seg_adapter, device)
        s = seg_adapter.numel()
    nbytes = lib.lora_sgmv_tiles_size(t_total, s)
    tiles = torch.empty((nbytes + 3) // 4, dtype=torch.int32, device=device)
    _lib.call("lora_sgmv_schedule", _lib.ptr(ids), _lib.ptr(seg_start), _lib.ptr(seg_adapter), t_total, s,
              n_adapters, _lib.ptr(tiles), tiles.numel() * 4, _lib.stream_handle(device))
    return tiles, s


def sgmv_shrink(x: torch.Tensor, a_flat: torch.Tensor, offsets: torch.Tensor, ranks: torch.Tensor,
                tiles: torch.Tensor, s: int, r_max: int, scale: float = 1.0, z_dtype=torch.float32,
                z_width: int | None = None, split_k: int = 0, rows: torch.Tensor | None = None,
                t_total: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    _lib.require_cuda(x, a_flat, where="sgmv_shrink")
    _check_half(x, "sgmv_shrink")
    x = _lib.row_major(x)
    a_flat = _lib.row_major(a_flat)
    t = x.shape[0] if t_total is None else t_total
    k = x.shape[1]
    width = r_max if z_width is None else int(z_width)
    if out is None:
        out = torch.zeros((x.shape[0], width), device=x.device, dtype=z_dtype) if rows is not None else \
            torch.empty((x.shape[0], width), device=x.device, dtype=z_dtype)
    lib = _lib.load()
    if split_k <= 0:
        split_k = lib.lora_sgmv_pick_split_k(t, k, r_max)
    ws = _lib.WORKSPACE.get(lib.lora_sgmv_shrink_workspace_size(t, s, width, split_k), x.device, "sgmv")
    offsets = _i64(offsets, x.device)
    ranks = _i64(ranks, x.device)
    if rows is not None:
        rows = _i64(rows, x.device)
    _lib.call("lora_sgmv_shrink_ex", _lib.ptr(x), _lib.ld(x), _lib.ptr(a_flat), _lib.ld(a_flat), a_flat.shape[0],
              _lib.ptr(offsets), _lib.ptr(ranks), offsets.numel(), _lib.ptr(tiles), _lib.ptr(rows), _lib.ptr(out),
              out.stride(0),
              _lib.dtype_code(out.dtype), width, t, s, k, int(r_max), float(scale), _dt(x), int(split_k),
              _lib.ptr(ws), ws.numel(), _lib.stream_handle(x.device))
    return out


def sgmv_expand(y: torch.Tensor | None, z: torch.Tensor, b: torch.Tensor, b_sj: int, b_sn: int,
                offsets: torch.Tensor, ranks: torch.Tensor, tiles: torch.Tensor, s: int, n: int, r_max: int,
                scale: float = 1.0, rows: torch.Tensor | None = None, t_total: int | None = None,
                out: torch.Tensor | None = None, dtype: torch.dtype | None = None) -> torch.Tensor:
    _lib.require_cuda(z, b, y, where="sgmv_expand")
    dtype = y.dtype if y is not None else (dtype or b.dtype)
    z = _lib.row_major(z)
    t = z.shape[0] if t_total is None else t_total
    if y is not None:
        y = _lib.row_major(y)
    if out is None:
        out = torch.empty((z.shape[0], n), device=z.device, dtype=dtype)
    offsets = _i64(offsets, z.device)
    ranks = _i64(ranks, z.device)
    if rows is not None:
        rows = _i64(rows, z.device)
    _lib.call("lora_sgmv_expand", _lib.ptr(y), _lib.ld(y) if y is not None else 0, _lib.ptr(z), _lib.ld(z),
              _lib.dtype_code(z.dtype), _lib.ptr(b.contiguous()), int(b_sj), int(b_sn), _lib.ptr(offsets),
              _lib.ptr(ranks), offsets.numel(), _lib.ptr(tiles), _lib.ptr(rows), _lib.ptr(out), out.stride(0), t, s, n,
              int(r_max), float(scale), _lib.dtype_code(dtype), _lib.stream_handle(z.device))
    return out


def sgmv_branch(x: torch.Tensor, y: torch.Tensor | None, a_flat: torch.Tensor, b_flat: torch.Tensor,
                offsets: torch.Tensor, ranks: torch.Tensor, tiles: torch.Tensor, s: int, r_max: int,
                scale: float = 1.0, out: torch.Tensor | None = None) -> torch.Tensor | None:
    """``out = y + (scale * x @ A_a.T) @ B_a`` per tile in one ABI call (tensor-core shrink,
    ordered reduction, tensor-core expand).  Returns None when the shape is outside
    that path (r_max > 64, unaligned rows): then use sgmv_shrink + sgmv_expand."""
    _lib.require_cuda(x, a_flat, b_flat, y, where="sgmv_branch")
    _check_half(x, "sgmv_branch")
    x = _lib.row_major(x)
    a_flat = _lib.row_major(a_flat)
    b_flat = _lib.row_major(b_flat)
    t, k = x.shape
    n = b_flat.shape[1]
    if y is not None:
        y = _lib.row_major(y)
    if out is None:
        out = torch.empty((t, n), device=x.device, dtype=x.dtype)
    lib = _lib.load()
    ws_bytes = lib.lora_sgmv_branch_workspace_size(t, s, k, int(r_max))
    ws = _lib.WORKSPACE.get(ws_bytes, x.device, "branch")
    offsets = _i64(offsets, x.device)
    ranks = _i64(ranks, x.device)
    rc = lib.lora_sgmv_branch(_lib.ptr(x), _lib.ld(x), _lib.ptr(y), _lib.ld(y) if y is not None else 0,
                              _lib.ptr(a_flat), _lib.ld(a_flat), a_flat.shape[0], _lib.ptr(b_flat), _lib.ld(b_flat),
                              b_flat.shape[0], _lib.ptr(offsets), _lib.ptr(ranks), offsets.numel(), _lib.ptr(tiles),
                              _lib.ptr(out), out.stride(0), t, s, k, n, int(r_max), float(scale), _dt(x),
                              _lib.ptr(ws), ws.numel(), _lib.stream_handle(x.device))
    if rc == _lib.LORA_ERR_UNSUPPORTED:
        return None
    _lib.check(rc, "lora_sgmv_branch")
    return out


def sgmv_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, a_flat: torch.Tensor,
                b_flat: torch.Tensor, offsets: torch.Tensor, ranks: torch.Tensor, tiles: torch.Tensor, s: int,
                r_max: int, scale: float = 1.0, out: torch.Tensor | None = None) -> torch.Tensor | None:
    """``out = x @ weight.T + bias + (scale * x @ A_a.T) @ B_a`` per tile in ONE GEMM: the
    adapters ride as a per-256-token-tile K tail of the base GEMM (lora_sgmv_linear).
    Returns None when the shape is outside that path (r_max > 64, K or N not a
    multiple of 64, unaligned rows): then use gemm + sgmv_branch."""
    _lib.require_cuda(x, weight, a_flat, b_flat, bias, where="sgmv_linear")
    _check_half(x, "sgmv_linear")
    if weight.dtype != x.dtype or a_flat.dtype != x.dtype or b_flat.dtype != x.dtype or (
            bias is not None and bias.dtype != x.dtype):
        raise TypeError("sgmv_linear: x, weight, bias and the adapter tables must share one dtype")
    x = _lib.row_major(x)
    weight = _lib.row_major(weight)
    a_flat = _lib.row_major(a_flat)
    b_flat = _lib.row_major(b_flat)
    t, k = x.shape
    n = weight.shape[0]
    if weight.shape[1] != k or a_flat.shape[1] != k or b_flat.shape[1] != n:
        raise ValueError("sgmv_linear: x, weight, a_flat and b_flat disagree on K / N")
    if bias is not None:
        bias = bias.contiguous()
        if bias.shape != (n,):
            raise ValueError("sgmv_linear: bias must have out_features elements")
    if out is None:
        out = torch.empty((t, n), device=x.device, dtype=x.dtype)
    lib = _lib.load()
    ws_bytes = lib.lora_sgmv_linear_workspace_size(t, s, k, int(r_max))
    if ws_bytes == 0:  # beyond the fused kernel's workspace cap (per-token ids over many tokens)
        return None
    ws = _lib.WORKSPACE.get(ws_bytes, x.device, "sgmv_linear")
    offsets = _i64(offsets, x.device)
    ranks = _i64(ranks, x.device)
    rc = lib.lora_sgmv_linear(_lib.ptr(x), _lib.ld(x), _lib.ptr(weight), _lib.ld(weight), _lib.ptr(bias),
                              _lib.ptr(a_flat), _lib.ld(a_flat), a_flat.shape[0], _lib.ptr(b_flat), _lib.ld(b_flat),
                              b_flat.shape[0], _lib.ptr(offsets), _lib.ptr(ranks), offsets.numel(), _lib.ptr(tiles),
                              _lib.ptr(out), out.stride(0), t, s, k, n, int(r_max), float(scale), _dt(x),
                              _lib.ptr(ws), ws.numel(), _lib.stream_handle(x.device))
    if rc == _lib.LORA_ERR_UNSUPPORTED:
        return None
    _lib.check(rc, "lora_sgmv_linear")
    return out
