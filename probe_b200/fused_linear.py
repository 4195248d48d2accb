"""Single-adapter LoRA linear on B200:  ``x @ W.T + bias + scale * (x @ A.T) @ B.T``.

Drop-in for ``loraforge_kernels.fused_linear`` (same names, signatures and
error behaviour).  The implementations are this package's sm_100a kernels:

``kconcat``  (default for M > 256)
    rank shrink ``z = scale * x @ A.T`` (split-K kernel, or the tcgen05 GEMM
    for ranks above 128), then ONE tcgen05 GEMM whose mainloop runs over
    ``[x | z]`` against ``[W | B]`` -- the LoRA expand is an extra K-slice, so
    the output is written once and no concatenated copy of x or W is built.
    The reference reached the same algebra by materialising ``[x | s.z]`` and
    ``[W | B]`` for cuBLAS (fused_linear.py:622-677).
``decode``   (default for M <= 256; M <= 64 when K is not a multiple of 8)
    shrink, then W streamed once through TMA into tcgen05 MMAs with the tokens
    as the narrow operand, K split over a cluster and the expand as a K tail
    (decode_linear.py:13-100).
``hybrid``   tcgen05 base GEMM, shrink, expand-add epilogue (fused_linear.py:370-373).
``concat``   tcgen05 GEMM on ``[W; A; 0]`` then expand-add (fused_linear.py:336-367).

With ``LORAFORGE_TUNE=1`` ``select_variant`` races the eligible candidates
once per shape, as the reference does (fused_linear.py:445-465); by default a
shape rule picks; ``LORAFORGE_VARIANT`` forces one.
Unlike the reference there is no CPU or cuBLAS path: CPU tensors raise.
"""

from __future__ import annotations

import os
import statistics

import torch

from . import kernels
from .kernels import round_up

# Rank tile constants kept for API compatibility (fused_linear.py:61-72).
MIN_RANK_TILE = 16
FUSED_MAX_RANK = 64
MIN_GEMM_ROWS = 128
# Rows at or below which the W-streaming decode kernel is the default: up to
# 256 on the tensor-core path (K a multiple of 8), 64 on the register path.
DECODE_MAX_ROWS = 64
SKINNY_MAX_ROWS = 256
# Ranks above this use the tensor-core GEMM for the shrink.
SHRINK_MMA_MAX_RANK = 128

VARIANTS = ("kconcat", "fused", "concat", "hybrid", "decode")

PACK_ALIGN = 16


def next_power_of_2(n: int) -> int:
    n = int(n)
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def pad_rank(r: int) -> int:
    """Round a rank up to the next power of two, at least 16 (fused_linear.py:77-79)."""
    return max(MIN_RANK_TILE, next_power_of_2(r))


def packed_rank(r: int) -> int:
    """Rank rows appended by ``augment_weight``: r rounded up to 16 (fused_linear.py:331-333)."""
    return ((r + PACK_ALIGN - 1) // PACK_ALIGN) * PACK_ALIGN


def _half(dtype) -> bool:
    return dtype in (torch.float16, torch.bfloat16)


def _require_half(x: torch.Tensor, where: str) -> None:
    if not x.is_cuda:
        raise RuntimeError(f"{where}: CUDA tensors required (this B200 build has no CPU path)")
    if not _half(x.dtype):
        raise TypeError(f"{where}: float16/bfloat16 required, got {x.dtype}")


# --------------------------------------------------------------------------- #
# Epilogue and GEMM entry points
# --------------------------------------------------------------------------- #

def expand_add(y, z, b, scale):
    """``out = y + scale * z @ b.T`` for y [M,N], z [M,R], b [N,R]; fresh output.

    y and z may be strided views (the concat path slices one GEMM result).
    Reference: fused_linear.py:176-200.
    """
    m, r = z.shape
    n = b.shape[0]
    assert b.shape[1] == r and y.shape == (m, n)
    return kernels.expand_add(y, z, b, scale)


class _KConcat:
    """Plan-time state of the kconcat variant.

    The tail of the fused GEMM is ``[hi | lo]`` of ``s.z = scale * x @ A.T``
    (each part r16 = roundup(r, 16) wide, zero beyond r) against
    ``[B | B]``: hi = round(s.z) and lo = round(s.z - hi) in the input dtype, so
    the expand keeps ~16 mantissa bits of z for twice the (small) tail width.
    """

    def __init__(self, weight, bias, a, b, scale):
        self.weight = weight.contiguous()
        self.bias = None if bias is None else bias.contiguous()
        self.a = a.contiguous()
        self.r = a.shape[0]
        self.r16 = round_up(self.r, 16)
        self.tail = 2 * self.r16
        b = b.to(weight.dtype)
        self.b_dup = torch.zeros((weight.shape[0], self.tail), device=weight.device, dtype=weight.dtype)
        self.b_dup[:, : self.r] = b
        self.b_dup[:, self.r16: self.r16 + self.r] = b
        self.scale = float(scale)
        self.a_pad = None
        if self.r > SHRINK_MMA_MAX_RANK:
            self.a_pad = torch.zeros((self.r16, self.a.shape[1]), device=a.device, dtype=a.dtype)
            self.a_pad[: self.r] = self.a

    def shrink(self, x):
        """``[hi | lo]`` of ``scale * x @ A.T``, shape [M, 2 * r16]."""
        if self.a_pad is None:
            return kernels.shrink(x, self.a, self.scale, z_dtype=x.dtype, z_width=self.r16, z_split=True)
        z = torch.empty((x.shape[0], self.tail), device=x.device, dtype=x.dtype)
        kernels.gemm(x, self.a_pad, alpha=self.scale, out=z[:, : self.r16], lo_offset=self.r16)
        return z

    def __call__(self, x, out=None):
        z = self.shrink(x)
        return kernels.gemm(x, self.weight, z, self.b_dup, rank=self.tail, bias=self.bias, out=out)


def fused_gemm(x, weight, bias, a, b, scale, out=None):
    """``x @ weight.T + bias + scale * (x @ a.T) @ b.T`` with one output write.

    Reference: fused_linear.py:296-317 (a single Triton kernel there; here the
    shrink kernel plus one tcgen05 GEMM with the expand as a K-slice).
    """
    _require_half(x, "fused_gemm")
    if a is None:
        return kernels.gemm(x, weight, bias=bias, out=out)
    return _KConcat(weight, bias, a, b, scale)(x, out=out)


def augment_weight(weight: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
    """``[W; A; 0]``: the shrink factor packed as extra output rows (fused_linear.py:336-343)."""
    a = a.to(device=weight.device, dtype=weight.dtype)
    pad = packed_rank(a.shape[0]) - a.shape[0]
    blocks = [weight, a]
    if pad:
        blocks.append(a.new_zeros(pad, a.shape[1]))
    return torch.cat(blocks, dim=0).contiguous()


def augment_bias(bias: torch.Tensor | None, rank: int) -> torch.Tensor | None:
    """Bias extended with zeros for the packed rows (fused_linear.py:346-350)."""
    if bias is None:
        return None
    return torch.cat([bias, bias.new_zeros(packed_rank(rank))]).contiguous()


def kconcat_weight(weight: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``[W | B]`` widened along K, zero-padded to ``K + packed_rank(r)`` (fused_linear.py:652-659)."""
    n, k = weight.shape
    r = b.shape[1]
    out = weight.new_zeros((n, k + packed_rank(r)))
    out[:, :k] = weight
    out[:, k: k + r] = b.to(device=weight.device, dtype=weight.dtype)
    return out.contiguous()


def build_ext(x, a, scale, rank_pad):
    """Materialise ``[x | scale * x @ a.T]`` contiguously (fused_linear.py:662-673).

    The shrink kernel writes the rank columns (and their zero padding) in
    place; only the copy of x is a plain device copy.
    """
    _require_half(x, "build_ext")
    m, k = x.shape
    ext = torch.empty((m, k + rank_pad), device=x.device, dtype=x.dtype)
    ext[:, :k].copy_(x)
    kernels.shrink(x, a, scale, z_dtype=x.dtype, z_width=rank_pad, out=ext[:, k:])
    return ext


def _kconcat(x, weight_kcat, bias, a, scale, rank_pad):
    """The reference's kconcat: one GEMM over the materialised ``[x | s.z]``."""
    return kernels.gemm(build_ext(x, a, scale, rank_pad), weight_kcat, bias=bias)


def _concat(x, weight_aug, bias_aug, b, scale, n):
    """GEMM on ``[W; A; 0]`` gives ``[y | z]``; the expand-add consumes both views."""
    y_aug = kernels.gemm(x, weight_aug, bias=bias_aug)
    return expand_add(y_aug[:, :n], y_aug[:, n: n + b.shape[1]], b, scale)


def _hybrid(x, weight, bias, a, b, scale):
    """Base GEMM, fp32 shrink, expand-add epilogue."""
    y = kernels.gemm(x, weight, bias=bias)
    z = kernels.shrink(x, a, 1.0, z_dtype=torch.float32)
    return expand_add(y, z, b, scale)


def _decode(x, weight, bias, a, b, scale):
    """Small-M path: one kernel streaming W with the shrink fused and the expand
    as a K tail; shapes outside it take the fp32 shrink then the decode kernel."""
    out = kernels.linear_small(x, weight, a, b, bias, scale)
    if out is not None:
        return out
    z = kernels.shrink(x, a, 1.0, z_dtype=torch.float32)
    return kernels.decode_linear(x, weight, z, b, bias, scale)


def _decode_rows(k: int) -> int:
    """Largest token count of one decode-kernel call for inner dimension k."""
    return SKINNY_MAX_ROWS if _gemm_aligned(k) else DECODE_MAX_ROWS


def _base_linear(x, weight, bias):
    """``x @ W.T + bias`` with this package's kernels (the r == 0 / scale == 0 path)."""
    if x.shape[0] <= _decode_rows(x.shape[1]) or not _gemm_aligned(x.shape[1]):
        return _rowwise(lambda xs: kernels.decode_linear(xs, weight, None, None, bias, 0.0), x)
    return kernels.gemm(x, weight, bias=bias)


def _rowwise(fn, x):
    """Apply a decode-sized kernel to any number of rows (odd-K fallback)."""
    step = _decode_rows(x.shape[1])
    if x.shape[0] <= step:
        return fn(x)
    return torch.cat([fn(x[i: i + step]) for i in range(0, x.shape[0], step)])


def _gemm_aligned(k: int) -> bool:
    return k % 8 == 0


def eligible(variant, m, k, n, r, dtype, has_augmented):
    """Which variants may run on a shape (reference gate: fused_linear.py:385-406)."""
    if not _half(dtype):
        return False
    if variant == "decode":
        return m <= _decode_rows(k) and r <= SHRINK_MMA_MAX_RANK
    if not _gemm_aligned(k):
        return False
    if variant in ("kconcat", "fused"):
        return True
    if variant == "concat":
        return has_augmented and m >= MIN_GEMM_ROWS and r <= 256
    if variant == "hybrid":
        return m >= MIN_GEMM_ROWS and r <= SHRINK_MMA_MAX_RANK
    return False


# --------------------------------------------------------------------------- #
# Variant selection
# --------------------------------------------------------------------------- #

class _VariantRace:
    """The per-shape timing race of ``LORAFORGE_TUNE=1`` (reference behaviour:
    fused_linear.py:413-473 times every eligible variant once per shape and
    keeps the fastest).

    Candidates are timed round-robin -- each round runs every candidate once
    between CUDA events -- so clock and power drift during the race touch all
    of them alike; the median round decides.  With ``LORAFORGE_TUNE_MODE=graph``
    shapes of at most 8 rows are timed as a captured chain of 20 calls (the
    replay cost a graph-serving caller pays).  A candidate that raises drops
    out.  Results are kept per key together with the candidate set and tune
    mode they were measured under; a change of either re-runs the race.
    """

    ROUNDS = 15
    WARMUP = 5
    CHAIN = 20

    def __init__(self):
        self.results: dict[tuple, dict] = {}

    @staticmethod
    def _as_chain(fn, length):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(length):
                fn()
        return graph.replay, graph

    def _clock(self, runners: dict, graph_mode: bool) -> dict:
        live, per_call, keep = {}, {}, []
        for name, fn in runners.items():
            try:
                for _ in range(self.WARMUP):
                    fn()
                if graph_mode:
                    replay, graph = self._as_chain(fn, self.CHAIN)
                    keep.append(graph)
                    live[name], per_call[name] = replay, self.CHAIN
                else:
                    live[name], per_call[name] = fn, 1
            except Exception:  # noqa: BLE001 -- a failing variant is not a candidate
                continue
        torch.cuda.synchronize()
        samples = {name: [] for name in live}
        for _ in range(self.ROUNDS):
            for name, fn in live.items():
                t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                t0.record()
                fn()
                t1.record()
                t1.synchronize()
                samples[name].append(t0.elapsed_time(t1) / per_call[name])
        del keep
        return {name: statistics.median(v) for name, v in samples.items()}

    def pick(self, runners: dict, key: tuple) -> str:
        forced = _forced_variant()
        if forced in runners:
            return forced
        if len(runners) == 1:
            return next(iter(runners))
        mode = os.environ.get("LORAFORGE_TUNE_MODE", "eager")
        context = (tuple(sorted(runners)), mode)
        known = self.results.get(key)
        if known is not None and known["context"] == context:
            return known["winner"]
        timings = self._clock(runners, graph_mode=(mode == "graph" and key[0] <= 8))
        if not timings:
            raise RuntimeError(f"no LoRA variant ran for shape {key}")
        winner = min(timings, key=timings.get)
        self.results[key] = {"winner": winner, "timings_ms": timings, "context": context}
        return winner

    def report(self) -> dict:
        out = {}
        for (m, k, n, r, dtype, _device), res in self.results.items():
            out[f"m{m}_k{k}_n{n}_r{r}_{str(dtype).split('.')[-1]}"] = res["winner"]
        return out


_RACE = _VariantRace()


def _forced_variant() -> str | None:
    choice = os.environ.get("LORAFORGE_VARIANT", "").strip().lower()
    return choice if choice in VARIANTS else None


def select_variant(runners: dict, key: tuple) -> str:
    """Name of the variant to run for shape ``key`` (forced, only, or raced once)."""
    return _RACE.pick(runners, key)


def selection_report() -> dict:
    """Which variant won the race for each shape seen so far (fused_linear.py:468-473)."""
    return _RACE.report()


def _default_variant(rows, k, r):
    if rows <= _decode_rows(k) and r <= SHRINK_MMA_MAX_RANK:
        return "decode"
    return "kconcat"


def build_plan(probe, weight, bias, a, b, scale, base_layer=None):
    """Resolve the variant for this shape once and return a specialised callable.

    Reference: fused_linear.py:476-524.  With ``LORAFORGE_TUNE=1`` every
    eligible variant is timed on ``probe`` (the reference's behaviour);
    otherwise the shape rule picks decode for M <= 256 (64 with K not a multiple of
    8) and kconcat above.
    ``base_layer`` is accepted for signature compatibility; no packed weight
    aliases it here because kconcat needs no packed copy of W.
    """
    _require_half(probe, "build_plan")
    n, k = weight.shape
    r = a.shape[0]
    dtype = probe.dtype
    rows = probe.shape[0]
    if r == 0 or scale == 0:
        return lambda x: _base_linear(x, weight, bias)
    if weight.dtype != dtype or a.dtype != dtype or b.dtype != dtype:
        raise TypeError("build_plan: x, weight, a and b must share one dtype")

    # Factories, not runners: a variant's plan-time state (kconcat's [B | B],
    # concat's [W; A; 0]) is built only for the variant that will run (or for
    # every candidate of a timing race), never on a call that picks another.
    makers = {}
    if eligible("decode", rows, k, n, r, dtype, False):
        makers["decode"] = lambda: (lambda x: _decode(x, weight, bias, a, b, scale))
    if eligible("kconcat", rows, k, n, r, dtype, False):
        makers["kconcat"] = lambda: _KConcat(weight, bias, a, b, scale)
    tune = os.environ.get("LORAFORGE_TUNE", "0") == "1"
    forced = _forced_variant()
    if tune or forced in ("hybrid", "concat"):
        if eligible("hybrid", rows, k, n, r, dtype, False):
            makers["hybrid"] = lambda: (lambda x: _hybrid(x, weight, bias, a, b, scale))
        pack = os.environ.get("LORAFORGE_PACK", "view").strip().lower()
        if pack not in ("0", "off", "none") and eligible("concat", rows, k, n, r, dtype, True):
            def make_concat():
                weight_aug = augment_weight(weight, a)
                bias_aug = augment_bias(bias, r)
                return lambda x: _concat(x, weight_aug, bias_aug, b, scale, n)
            makers["concat"] = make_concat
    if not makers:
        # Odd K with many rows: the decode kernel over 64-row chunks.
        return lambda x: _rowwise(lambda xs: _decode(xs, weight, bias, a, b, scale), x)

    if forced in makers:
        return makers[forced]()
    if not tune:
        choice = _default_variant(rows, k, r)
        return makers[choice]() if choice in makers else next(iter(makers.values()))()
    runners = {nm: make() for nm, make in makers.items()}
    key = (rows, k, n, r, dtype, torch.cuda.current_device())
    variant = select_variant({nm: (lambda f=fn: f(probe)) for nm, fn in runners.items()}, key)
    return runners[variant]


def fused_lora_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    a: torch.Tensor,
    b: torch.Tensor,
    scale: float = 1.0,
) -> torch.Tensor:
    """``x @ weight.T + bias + scale * (x @ a.T) @ b.T``; x may have leading dims.

    ``a`` is ``[r, k]`` and ``b`` is ``[n, r]`` (lora_A / lora_B weights).
    Reference: fused_linear.py:527-551 (minus its CPU fallback).
    """
    shape = x.shape
    n = weight.shape[0]
    x2 = x.reshape(-1, shape[-1])
    _require_half(x2, "fused_lora_linear")
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    if a.shape[0] == 0 or scale == 0:
        return _base_linear(x2, weight, bias).reshape(*shape[:-1], n)
    return build_plan(x2, weight, bias, a, b, scale)(x2).reshape(*shape[:-1], n)


class FusedLoRALinear(torch.nn.Module):
    """Drop-in replacement for an ``nn.Linear`` carrying a LoRA sidecar.

    Nothing is merged into the base weight, so the adapter stays swappable.
    Reference: fused_linear.py:554-615.
    """

    def __init__(self, base: torch.nn.Linear, a: torch.Tensor, b: torch.Tensor, scale: float = 1.0):
        super().__init__()
        if a.shape[1] != base.in_features or b.shape[0] != base.out_features or a.shape[0] != b.shape[1]:
            raise ValueError(
                f"LoRA factors {tuple(a.shape)}/{tuple(b.shape)} do not match "
                f"Linear({base.in_features}, {base.out_features})"
            )
        self.in_features = base.in_features
        self.out_features = base.out_features
        self.scale = float(scale)
        device, dtype = base.weight.device, base.weight.dtype
        self.register_buffer("weight", base.weight.detach())
        self.register_buffer("bias", None if base.bias is None else base.bias.detach())
        self.register_buffer("lora_a", a.detach().to(device=device, dtype=dtype).contiguous())
        self.register_buffer("lora_b", b.detach().to(device=device, dtype=dtype).contiguous())
        self._plan = None
        self._plan_rows = -1

    @property
    def rank(self) -> int:
        return self.lora_b.shape[1]

    def set_factors(self, a: torch.Tensor, b: torch.Tensor, scale: float | None = None) -> None:
        """Swap the adapter in place; the plan is rebuilt around the new factors."""
        device, dtype = self.weight.device, self.weight.dtype
        self.lora_a = a.detach().to(device=device, dtype=dtype).contiguous()
        self.lora_b = b.detach().to(device=device, dtype=dtype).contiguous()
        if scale is not None:
            self.scale = float(scale)
        self._plan = None
        self._plan_rows = -1

    def extra_repr(self) -> str:
        return (
            f"in_features={self.in_features}, out_features={self.out_features}, "
            f"bias={self.bias is not None}, rank={self.rank}, scale={self.scale}"
        )

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        rows = x.numel() // shape[-1]
        x2 = x.reshape(-1, shape[-1])
        _require_half(x2, "FusedLoRALinear")
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        if self._plan_rows != rows:
            self._plan = build_plan(x2, self.weight, self.bias, self.lora_a, self.lora_b, self.scale)
            self._plan_rows = rows
        return self._plan(x2).reshape(*shape[:-1], self.out_features)
