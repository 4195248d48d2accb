"""Whole-output parity checks of a LoRA linear -- TEST INFRASTRUCTURE ONLY.

The float64 oracle (``lora_oracle``) cannot form the output of a full-size
benchmark projection (32760 x 13824 values) in seconds, so a full-size output
is checked three ways, each against the oracle on the same bf16 inputs:

* sampled rows (the first, the last, tile edges, random ones) against
  ``naive_linear`` element by element, with the bf16 bars;
* every row sum against ``row_sums`` (linearity: one matrix-vector product);
* a signed token sketch ``v^T out`` (v = +-1 per token) against
  ``token_sketch``, which mixes every row into every column.

A missing or misplaced tile changes a row sum or a sketch column by about
sqrt(tile width) output magnitudes, far above the rounding noise of a correct
output; the bounds are 6 sigma of that noise (each bf16 output carries a
rounding error of variance ulp^2/12), computed from the product's own values.

Only the tests and ``bench.py``'s parity report use this module.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import lora_oracle as orc

ROW_CHUNK = 4096
ALL_ROWS_MAX = 256  # outputs of at most this many rows are compared row by row in full


def np64(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


def _ulp_var(out: torch.Tensor, mant: int) -> torch.Tensor:
    """Per-element variance ulp^2/12 of rounding to a format with ``mant`` mantissa bits."""
    v = out.double().abs().clamp_min(1e-30)
    ulp = torch.exp2(torch.floor(torch.log2(v)) - (mant - 1))
    return ulp * ulp / 12.0


def sample_rows(m: int, n_random: int = 24, seed: int = 0, tile: int = 256) -> list[int]:
    """Row indices to check: first, last, tile edges, and seeded random rows."""
    if m <= 0:
        return []
    rows = {0, m - 1}
    for edge in (tile - 1, tile, 2 * tile - 1, m // 2, m - tile, m - tile - 1):
        if 0 <= edge < m:
            rows.add(edge)
    rng = np.random.default_rng(seed)
    rows.update(int(r) for r in rng.integers(0, m, size=min(n_random, m)))
    return sorted(rows)


def linear_report(out: torch.Tensor, x: torch.Tensor, w: torch.Tensor, bias, a, b, scale: float,
                  dtype: str = "bf16", n_random: int = 24, seed: int = 0, full_checks: bool = True) -> dict:
    """Parity of ``out`` against ``x W^T + bias + scale (x a^T) b^T`` (float64).

    ``a`` / ``b`` are the factors the reference would hold (numpy or torch,
    e.g. the stacked factors of ``lora_oracle.stack_adapters``).  Returns a dict
    with ``ok`` and the measured errors; ``full_checks`` adds the row sums and
    the token sketch over the whole output."""
    m, n = out.shape
    a64 = None if a is None else (a if isinstance(a, np.ndarray) else np64(a))
    b64 = None if b is None else (b if isinstance(b, np.ndarray) else np64(b))
    w64 = np64(w)
    bias64 = None if bias is None else np64(bias)
    rows = list(range(m)) if m <= ALL_ROWS_MAX else sample_rows(m, n_random, seed)
    idx = torch.as_tensor(rows, device=out.device)
    got = np64(out.index_select(0, idx))
    want = orc.naive_linear(np64(x.index_select(0, idx)), w64, bias64, a64, b64, scale)
    excess = orc.excess_abs_error(got, want, dtype)
    raw, fro = orc.parity(got, want)
    report = {"rows_checked": len(rows), "max_abs_excess": excess, "max_abs_raw": raw, "rel_fro": fro,
              "bars": {"max_abs_excess": 2e-2, "rel_fro": 5e-3}}
    ok = excess <= 2e-2 and fro <= 5e-3 and bool(np.isfinite(got).all())
    if full_checks:
        mant = {"bf16": 8, "f16": 11}[dtype]
        gen = torch.Generator(device="cpu")
        gen.manual_seed(seed + 17)
        signs = (torch.randint(0, 2, (m,), generator=gen) * 2 - 1).to(torch.float64)
        row_dev, sketch_got = 0.0, torch.zeros(n, dtype=torch.float64, device=out.device)
        sketch_var = torch.zeros(n, dtype=torch.float64, device=out.device)
        u = np.zeros(x.shape[1])
        signs_dev = signs.to(out.device)
        for r0 in range(0, m, ROW_CHUNK):
            r1 = min(m, r0 + ROW_CHUNK)
            oc = out[r0:r1].double()
            var = _ulp_var(out[r0:r1], mant)
            got_sum = oc.sum(1).cpu().numpy()
            sigma = var.sum(1).sqrt().cpu().numpy()
            xc = np64(x[r0:r1])
            want_sum = orc.row_sums(xc, w64, bias64, a64, b64, scale)
            bound = 6.0 * sigma + 1e-4 * math.sqrt(n)
            row_dev = max(row_dev, float((np.abs(got_sum - want_sum) / bound).max()))
            sc = signs_dev[r0:r1]
            sketch_got += sc @ oc
            sketch_var += var.sum(0)
            u += signs[r0:r1].numpy() @ xc
        want_sketch = orc.token_sketch(np.ones(1), u[None, :], w64, bias64, a64, b64, scale)
        if bias64 is not None:  # token_sketch added sum(weights) * bias for one unit weight
            want_sketch = want_sketch - bias64 + float(signs.sum()) * bias64
        bound = 6.0 * sketch_var.sqrt().cpu().numpy() + 1e-4 * math.sqrt(m)
        sketch_dev = float((np.abs(sketch_got.cpu().numpy() - want_sketch) / bound).max())
        report.update({"row_sum_dev": row_dev, "sketch_dev": sketch_dev,
                       "full_check_note": "row sums and a +-1 token sketch over the whole output, "
                                          "deviation / (6 sigma of bf16 rounding noise); ok below 1"})
        ok = ok and row_dev <= 1.0 and sketch_dev <= 1.0
    report["ok"] = bool(ok)
    return report


def branch_report(out: torch.Tensor, x: torch.Tensor, y: torch.Tensor, a_flat, b_flat, offsets, ranks, ids,
                  dtype: str = "bf16", n_random: int = 48, seed: int = 0) -> dict:
    """Parity of a multi-adapter branch output against ``ragged_branch`` on sampled
    tokens: the first and last token of every segment boundary sampled, plus
    random ones (``ids`` gives each token's adapter; the scale is in b_flat)."""
    t = out.shape[0]
    ids_np = ids.detach().cpu().numpy().astype(np.int64) if isinstance(ids, torch.Tensor) else np.asarray(ids)
    edges = np.flatnonzero(np.diff(ids_np)) if t > 1 else np.zeros(0, dtype=np.int64)
    rng = np.random.default_rng(seed)
    picks = set(int(v) for v in rng.choice(edges, size=min(len(edges), n_random), replace=False)) if len(edges) else set()
    rows = {0, t - 1}
    for e in picks:
        rows.update((e, e + 1))
    rows.update(int(r) for r in rng.integers(0, t, size=min(n_random, t)))
    rows = sorted(r for r in rows if 0 <= r < t)
    idx = torch.as_tensor(rows, device=out.device)
    offs = offsets.detach().cpu().numpy() if isinstance(offsets, torch.Tensor) else np.asarray(offsets)
    rks = ranks.detach().cpu().numpy() if isinstance(ranks, torch.Tensor) else np.asarray(ranks)
    want = orc.ragged_branch(np64(x.index_select(0, idx)), np64(y.index_select(0, idx)), np64(a_flat),
                             np64(b_flat), offs, rks, ids_np[rows])
    got = np64(out.index_select(0, idx))
    excess = orc.excess_abs_error(got, want, dtype)
    raw, fro = orc.parity(got, want)
    return {"rows_checked": len(rows), "max_abs_excess": excess, "max_abs_raw": raw, "rel_fro": fro,
            "ok": bool(excess <= 2e-2 and fro <= 5e-3 and np.isfinite(got).all())}


def seg_linear_report(out: torch.Tensor, x: torch.Tensor, w: torch.Tensor, bias, a_flat, b_flat, offsets, ranks,
                      ids, dtype: str = "bf16", n_random: int = 48, seed: int = 0) -> dict:
    """Parity of a fused base + multi-adapter linear against ``ragged_branch``
    applied to the exact base ``x W^T + bias`` (float64), on the tokens
    ``branch_report`` samples (segment edges and random ones)."""
    t = out.shape[0]
    ids_np = ids.detach().cpu().numpy().astype(np.int64) if isinstance(ids, torch.Tensor) else np.asarray(ids)
    edges = np.flatnonzero(np.diff(ids_np)) if t > 1 else np.zeros(0, dtype=np.int64)
    rng = np.random.default_rng(seed)
    picks = set(int(v) for v in rng.choice(edges, size=min(len(edges), n_random), replace=False)) if len(edges) else set()
    rows = {0, t - 1}
    for e in picks:
        rows.update((e, e + 1))
    for edge in (255, 256, t - 256, t - 257):
        rows.add(edge)
    rows.update(int(r) for r in rng.integers(0, t, size=min(n_random, t)))
    rows = sorted(r for r in rows if 0 <= r < t)
    idx = torch.as_tensor(rows, device=out.device)
    xs = np64(x.index_select(0, idx))
    base = xs @ np64(w).T + (0.0 if bias is None else np64(bias))
    offs = offsets.detach().cpu().numpy() if isinstance(offsets, torch.Tensor) else np.asarray(offsets)
    rks = ranks.detach().cpu().numpy() if isinstance(ranks, torch.Tensor) else np.asarray(ranks)
    want = orc.ragged_branch(xs, base, np64(a_flat), np64(b_flat), offs, rks, ids_np[rows])
    got = np64(out.index_select(0, idx))
    excess = orc.excess_abs_error(got, want, dtype)
    raw, fro = orc.parity(got, want)
    return {"rows_checked": len(rows), "max_abs_excess": excess, "max_abs_raw": raw, "rel_fro": fro,
            "ok": bool(excess <= 2e-2 and fro <= 5e-3 and np.isfinite(got).all())}
