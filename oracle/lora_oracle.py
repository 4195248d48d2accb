"""CPU oracle for the LoRA-linear hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy (float64 unless stated), the arithmetic of the
reference implementation (lishenghui/probe, ``loraforge_kernels/``) for every
function on the hot path.  It is the checker for the CUDA kernels: only the
tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may use
it, and never as the thing measured or shipped.

Parity pinning: the restatement is checked against golden vectors produced by
running the reference itself in this container (its CPU path
``fused_lora_linear`` -> ``_torch_naive`` and its Triton kernels for the
segmented / ragged branch under the Triton interpreter, in fp32), committed
under ``tests/golden/`` with the script that generated them
(``tests/golden/make_golden.py``), plus the reference's own known-answer
tables for ``pad_rank`` / ``packed_rank`` (test_fused_linear.py:171-185).
"""

from __future__ import annotations

import numpy as np

# --------------------------------------------------------------- integer helpers


def next_power_of_2(n: int) -> int:
    """triton.next_power_of_2 semantics for n >= 0 (1 for n <= 1)."""
    n = int(n)
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def pad_rank(r: int) -> int:
    """max(16, next_pow2(r)) -- fused_linear.py:77-79."""
    return max(16, next_power_of_2(r))


def packed_rank(r: int) -> int:
    """r rounded up to a multiple of 16 -- fused_linear.py:331-333."""
    return ((r + 15) // 16) * 16


def align_to_deploy_rank(r: int) -> int:
    """First bucket of (8,16,24,32,48,64) >= r, else next_pow2 -- splitk_lora.py:11-19."""
    for bucket in (8, 16, 24, 32, 48, 64):
        if r <= bucket:
            return bucket
    return next_power_of_2(r)


def rank_tile(r: int) -> int:
    """max(16, next_pow2(r)) -- splitk_shrink.py:30-32, multilora.py:32-33."""
    return max(16, next_power_of_2(r))


def auto_split_k(n_tokens: int, target_programs: int = 2048, cap: int = 64) -> int:
    """multilora.py:36-48."""
    if n_tokens <= 0:
        return 1
    return max(1, min(cap, next_power_of_2(max(1, target_programs // n_tokens))))


# ---------------------------------------------------------------- rounding


def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round to the nearest bfloat16 (ties to even); returns float32 values."""
    f = np.ascontiguousarray(a, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    u = (u + 0x7FFF + lsb) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32)
    # NaN stays NaN
    return np.where(np.isnan(f), f, out)


def half_ulp(a: np.ndarray, dtype: str) -> np.ndarray:
    """Half a unit in the last place of the output dtype at |a| (the rounding error
    every correctly rounded output may carry)."""
    mant = {"bf16": 8, "f16": 11, "f32": 24}[dtype]
    a = np.abs(np.asarray(a, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, np.finfo(np.float64).tiny)))
    if dtype == "f16":
        e = np.maximum(e, -14.0)  # subnormal spacing
    return np.ldexp(1.0, (e - mant).astype(np.int64))


def round_dtype(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(a)
    if dtype == "f16":
        return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)
    return np.asarray(a, dtype=np.float32)


# --------------------------------------------------------- single adapter


def _f64(*arrs):
    return [None if a is None else np.asarray(a, dtype=np.float64) for a in arrs]


def naive_linear(x, w, bias, a, b, scale):
    """``F.linear(x, W, bias) + scale * (x @ A.T) @ B.T`` -- fused_linear.py:376-378.

    x [M,K], W [N,K], bias [N] or None, A [r,K], B [N,r]; float64.
    """
    x, w, bias, a, b = _f64(x, w, bias, a, b)
    y = x @ w.T
    if bias is not None:
        y = y + bias
    if a is not None and a.shape[0] > 0 and scale != 0:
        y = y + scale * ((x @ a.T) @ b.T)
    return y


def naive_linear_torch(x, w, bias, a, b, scale):
    """The reference's CPU path itself (``_torch_naive``, fused_linear.py:376-378) in torch.

    Used only to time the CPU baseline: F.linear + two mm, in the input dtype.
    """
    import torch

    y = torch.nn.functional.linear(x, w, bias)
    return y + scale * torch.mm(torch.mm(x, a.t()), b.t())


def shrink(x, a, scale=1.0):
    """``scale * x @ A.T`` -- splitk_lora.py:104-126 (before the dtype cast)."""
    x, a = _f64(x, a)
    return scale * (x @ a.T)


def expand_add(y, z, b, scale, bias=None):
    """``y + scale * z @ B.T (+ bias)`` -- fused_linear.py:176-200, splitk_lora.py:129-153."""
    y, z, b, bias = _f64(y, z, b, bias)
    out = scale * (z @ b.T)
    if y is not None:
        out = out + y
    if bias is not None:
        out = out + bias
    return out


def decode_linear(x, w, bias, a, b, scale, dtype="bf16"):
    """decode_linear.py:13-50: fp32 accumulation, z rounded to the input dtype before the expand."""
    x, w, bias, a, b = _f64(x, w, bias, a, b)
    out = x @ w.T
    if a is not None and a.shape[0] > 0 and scale != 0:
        z = round_dtype(x @ a.T, dtype).astype(np.float64)
        out = out + scale * (z @ b.T)
    if bias is not None:
        out = out + bias
    return out


def kconcat(x, w, bias, a, b, scale, dtype="bf16"):
    """fused_linear.py:652-677: ``[x | s*z] @ [W | B].T`` with s*z rounded to the input dtype."""
    x, w, bias, a, b = _f64(x, w, bias, a, b)
    z = round_dtype(scale * (x @ a.T), dtype).astype(np.float64)
    out = x @ w.T + z @ b.T
    if bias is not None:
        out = out + bias
    return out


def grouped_lora(x, a, b, y=None, scale=1.0):
    """fused_lora.py:159-200,295-311: a [P*R,K], b [P,N,R], y/out [M,P,N]."""
    x, a, b, y = _f64(x, a, b, y)
    p, n, r = b.shape
    z = x @ a.T
    out = np.zeros((x.shape[0], p, n))
    for i in range(p):
        out[:, i, :] = scale * (z[:, i * r:(i + 1) * r] @ b[i].T)
    if y is not None:
        out = out + y
    return out


def stack_adapters(adapters, base_scale=None, dtype=None):
    """attach_fused_lora stacking (runtime_lora.py:45-54).

    adapters: list of (down [r_i,K], up [N,r_i], alpha_i); the first one fixes
    the layer scale.  Returns (A_stack, B_stack, scale) with
    A_stack = [A_1; (a_2/a_1) A_2; ...], B_stack = [B_1 | B_2 | ...].
    With ``dtype`` ("bf16" / "f16") each folded block is rounded to that dtype
    after an fp32 multiply, as the reference does (``(alpha / target.scale) *
    down.float()`` then ``.to(dtype)``, runtime_lora.py:49-53).
    """
    down0, up0, alpha0 = adapters[0]
    scale = alpha0 if base_scale is None else base_scale
    a_blocks = [np.asarray(down0, dtype=np.float64)]
    b_blocks = [np.asarray(up0, dtype=np.float64)]
    for down, up, alpha in adapters[1:]:
        if dtype is None:
            a_blocks.append((alpha / scale) * np.asarray(down, dtype=np.float64))
        else:
            folded = np.float32(alpha / scale) * np.asarray(down, dtype=np.float32)
            a_blocks.append(round_dtype(folded, dtype).astype(np.float64))
        b_blocks.append(np.asarray(up, dtype=np.float64))
    return np.concatenate(a_blocks, axis=0), np.concatenate(b_blocks, axis=1), scale


def row_sums(x, w, bias, a, b, scale):
    """Row sums of ``naive_linear``'s output without forming it.

    By linearity, ``sum_n out[i, n] = x[i] . (sum_n W[n] + scale * A^T (sum_n B[n]))
    + sum(bias)``: one matrix-vector product over x, so the check covers every
    row of an output too large to compute in float64 here."""
    x, w, bias, a, b = _f64(x, w, bias, a, b)
    v = w.sum(axis=0)
    if a is not None and a.shape[0] > 0 and scale != 0:
        v = v + scale * (a.T @ b.sum(axis=0))
    out = x @ v
    if bias is not None:
        out = out + bias.sum()
    return out


def token_sketch(weights, x, w, bias, a, b, scale):
    """``weights^T . out`` for ``out = naive_linear(x, ...)`` without forming out.

    ``weights`` is one value per token; by linearity the result is
    ``u W^T + scale (u A^T) B^T + sum(weights) bias`` with ``u = weights^T x``,
    a length-N vector that mixes every row of the output into every column."""
    weights, x, w, bias, a, b = _f64(weights, x, w, bias, a, b)
    u = weights @ x
    out = w @ u
    if a is not None and a.shape[0] > 0 and scale != 0:
        out = out + scale * (b @ (a @ u))
    if bias is not None:
        out = out + weights.sum() * bias
    return out


# ------------------------------------------------------------ multi adapter


def ragged_branch(x, y, a_flat, b_flat, offsets, ranks, idx):
    """ragged_branch.py:6-40: out[t] = y[t] + (x[t] @ A[off:off+r].T) @ B[off:off+r] (scale in B)."""
    x, y, a_flat, b_flat = _f64(x, y, a_flat, b_flat)
    out = y.copy()
    for t in range(x.shape[0]):
        ad = int(idx[t])
        off, r = int(offsets[ad]), int(ranks[ad])
        if r == 0:
            continue
        out[t] += (x[t] @ a_flat[off:off + r].T) @ b_flat[off:off + r]
    return out


def segmented_branch(x, y, a_flat, b_flat, offsets, ranks, request_ids, tokens_per_request):
    """segmented_branch.py:50-60 (uniform segments; ValueError otherwise)."""
    total = np.asarray(x).shape[0]
    if total != len(request_ids) * tokens_per_request:
        raise ValueError("Invalid contiguous request segments")
    idx = np.repeat(np.asarray(request_ids, dtype=np.int64), tokens_per_request)
    return ragged_branch(x, y, a_flat, b_flat, offsets, ranks, idx)


def segments_to_ids(seg_start, seg_adapter):
    seg_start = np.asarray(seg_start, dtype=np.int64)
    lens = np.diff(seg_start)
    return np.repeat(np.asarray(seg_adapter, dtype=np.int64), lens)


def shrink_ragged(x, a_flat, offsets, ranks, idx, r_max):
    """multilora.py:128-182: z[t, :r_t] = x[t] @ A[off_t:off_t+r_t].T, zeros beyond, fp32 out."""
    x, a_flat = _f64(x, a_flat)
    z = np.zeros((x.shape[0], r_max))
    for t in range(x.shape[0]):
        ad = int(idx[t])
        off, r = int(offsets[ad]), int(ranks[ad])
        z[t, :r] = x[t] @ a_flat[off:off + r].T
    return z


def shrink_padded(x, a_stack, idx):
    """multilora.py:51-104: z[t] = x[t] @ A[idx[t]].T."""
    x, a_stack = _f64(x, a_stack)
    return np.stack([x[t] @ a_stack[int(idx[t])].T for t in range(x.shape[0])]) if x.shape[0] else \
        np.zeros((0, a_stack.shape[1]))


def expand_padded(y, z, b_stack, idx, scale=1.0):
    """multilora.py:295-347: out[t] = y[t] + scale * z[t, :r] @ B[idx[t]].T, B stack [n, N, r]."""
    y, z, b_stack = _f64(y, z, b_stack)
    r = b_stack.shape[2]
    out = y.copy()
    for t in range(y.shape[0]):
        out[t] += scale * (z[t, :r] @ b_stack[int(idx[t])].T)
    return out


# ---------------------------------------------------------- tile schedule


def tile_schedule(ids=None, seg_start=None, seg_adapter=None, n_adapters=None, tile=64):
    """Expected device tile list: a tile starts at every multiple of ``tile`` and
    wherever the adapter changes.  Returns (starts + [T], adapters); ids out of
    [0, n_adapters) map to -1."""
    if ids is None:
        ids = segments_to_ids(seg_start, seg_adapter)
    ids = [int(v) for v in ids]
    if n_adapters is not None:
        ids = [v if 0 <= v < n_adapters else -1 for v in ids]
    starts, adapters = [], []
    prev = None
    for t, a in enumerate(ids):
        if t % tile == 0 or a != prev:
            starts.append(t)
            adapters.append(a)
        prev = a
    starts.append(len(ids))
    return starts, adapters


# ----------------------------------------------------------- parity metrics


def excess_abs_error(got, want, dtype="bf16"):
    """max(|got - want| - half_ulp(want)): the arithmetic error beyond the rounding
    of a correctly rounded output in `dtype` (never negative)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    if got.size == 0:
        return 0.0
    return float(np.maximum(np.abs(got - want) - half_ulp(want, dtype), 0.0).max())


def parity(got, want):
    """(max-abs error, relative Frobenius error) of got against want, float64."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    err = got - want
    max_abs = float(np.abs(err).max()) if err.size else 0.0
    denom = float(np.linalg.norm(want))
    rel_fro = float(np.linalg.norm(err) / denom) if denom > 0 else float(np.linalg.norm(err))
    return max_abs, rel_fro
