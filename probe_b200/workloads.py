"""Seeded synthetic workloads C1-C5 of the LoRA-linear benchmark.

Shapes, value distributions and seeds follow the benchmark definition of the
reference comparison (x ~ N(0,1); W, A ~ N(0, 1/fan_in); B ~ N(0, 1/r)).  No
public dataset or checkpoint is involved: every tensor is drawn from a
``torch.Generator`` with a fixed seed, in the reference's storage layouts
(W [N,K], A [r,K], B [N,r]).  Generation may run on the CPU (bit-reproducible
small cases for parity tests) or directly on the GPU (the multi-GB bench
inputs).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

HIDDEN_LLAMA = 4096
FFN_LLAMA = 11008
HIDDEN_WAN = 5120
FFN_WAN = 13824


@dataclass
class Projection:
    name: str
    k: int
    n: int
    x: torch.Tensor
    w: torch.Tensor
    a: torch.Tensor          # [r, K] (stacked adapters for C5)
    b: torch.Tensor          # [N, r]
    scale: float
    bias: torch.Tensor | None = None
    # the adapters behind a stacked (a, b): (down [r_i, K], up [N, r_i], alpha_i), input dtype
    adapters: list = field(default_factory=list)

    @property
    def m(self) -> int:
        return self.x.shape[0]

    @property
    def r(self) -> int:
        return self.a.shape[0]

    def flops(self) -> float:
        """Algorithmic FLOPs: base GEMM + shrink + expand."""
        return 2.0 * self.m * self.k * self.n + 2.0 * self.m * self.r * (self.k + self.n)

    def bytes(self, elem: int = 2) -> float:
        """Compulsory HBM bytes: x, W, A, B read once, out written once."""
        return elem * (self.m * self.k + self.n * self.k + self.r * (self.k + self.n) + self.m * self.n)


def _randn(gen, shape, std, device, dtype):
    t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    return t.to(dtype)


def _gen(seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def c1(device="cpu", dtype=torch.float32) -> Projection:
    """C1: x[256,4096], W[4096,4096], A[16,4096], B[4096,16], scale 2.0, seed 0."""
    g = _gen(0, device)
    k = n = 4096
    x = _randn(g, (256, k), 1.0, device, dtype)
    w = _randn(g, (n, k), 1 / math.sqrt(k), device, dtype)
    a = _randn(g, (16, k), 1 / math.sqrt(k), device, dtype)
    b = _randn(g, (n, 16), 1 / math.sqrt(16), device, dtype)
    return Projection("c1", k, n, x, w, a, b, 2.0)


def c2(m: int, device="cpu", dtype=torch.float32) -> Projection:
    """C2: decode M in {1,4,16,64}; Llama up_proj W[11008,4096], r=16, scale 2.0.

    One generator seeded 1 with the M loop outermost: the draws for M are
    preceded by the draws of every smaller M in (1, 4, 16, 64).
    """
    g = _gen(1, device)
    k, n = HIDDEN_LLAMA, FFN_LLAMA
    for mm in (1, 4, 16, 64):
        x = _randn(g, (mm, k), 1.0, device, dtype)
        w = _randn(g, (n, k), 1 / math.sqrt(k), device, dtype)
        a = _randn(g, (16, k), 1 / math.sqrt(k), device, dtype)
        b = _randn(g, (n, 16), 1 / math.sqrt(16), device, dtype)
        if mm == m:
            return Projection(f"c2_m{m}", k, n, x, w, a, b, 2.0)
    raise ValueError(f"C2 is defined for M in (1, 4, 16, 64), not {m}")


def zipf_lengths(total: int, segments: int, s: float, gen: torch.Generator) -> list[int]:
    """Segment lengths with weights k^-s (k = 1..segments), shuffled by gen, each >= 1,
    summing exactly to total (remainder to the largest fractional parts)."""
    w = torch.tensor([k ** -s for k in range(1, segments + 1)], dtype=torch.float64)
    perm = torch.randperm(segments, generator=gen, device=gen.device).cpu()
    w = w[perm]
    real = w / w.sum() * total
    base = torch.clamp(torch.floor(real), min=1).to(torch.int64)
    rem = total - int(base.sum())
    frac = real - torch.floor(real)
    if rem > 0:
        order = torch.argsort(frac, descending=True, stable=True)
        for i in range(rem):
            base[order[i % segments]] += 1
    elif rem < 0:
        order = torch.argsort(frac, descending=False, stable=True)
        i = 0
        while rem < 0:
            j = order[i % segments]
            if base[j] > 1:
                base[j] -= 1
                rem += 1
            i += 1
    return [int(v) for v in base]


@dataclass
class Segmented:
    """C3: segmented multi-LoRA batch in the flat-table layout of segmented/ragged_branch."""
    x: torch.Tensor            # [T, K]
    w: torch.Tensor            # [N, K] base weight (y = x W^T)
    a_flat: torch.Tensor       # [sum r, K]
    b_flat: torch.Tensor       # [sum r, N] rank-major, scale folded
    offsets: torch.Tensor      # [n_adapters] int64
    ranks: torch.Tensor        # [n_adapters] int64
    seg_start: torch.Tensor    # [S+1] int64
    seg_adapter: torch.Tensor  # [S] int64
    scales: list = field(default_factory=list)
    a_list: list = field(default_factory=list)   # per adapter [r_a, K]
    b_list: list = field(default_factory=list)   # per adapter [N, r_a] (unscaled)

    @property
    def r_max(self) -> int:
        return int(self.ranks.max())

    def token_ids(self) -> torch.Tensor:
        lens = self.seg_start[1:] - self.seg_start[:-1]
        return torch.repeat_interleave(self.seg_adapter, lens)

    def branch_flops(self) -> float:
        ids = self.token_ids().cpu()
        r = self.ranks.cpu()[ids]
        k, n = self.x.shape[1], self.w.shape[0]
        return float(2 * r.sum() * (k + n))

    def branch_bytes(self, elem=2) -> float:
        t, k = self.x.shape
        n = self.w.shape[0]
        used = torch.unique(self.seg_adapter.cpu())
        r_used = int(self.ranks.cpu()[used].sum())
        return float(elem * (t * k + 2 * t * n + r_used * (k + n)))


def c3(device="cpu", dtype=torch.float32, tokens=4096, segments=128, n_adapters=64, k=4096, n=4096,
       seed=2) -> Segmented:
    """C3: 4096 tokens, 128 Zipf(1.1) segments, 64 adapters with ranks in {4,8,16,32,64}."""
    g = _gen(seed, device)
    lens = zipf_lengths(tokens, segments, 1.1, g)
    seg_adapter = torch.randint(0, n_adapters, (segments,), generator=g, device=device)
    choices = torch.tensor([4, 8, 16, 32, 64], device=device)
    ranks = choices[torch.randint(0, 5, (n_adapters,), generator=g, device=device)]
    a_list, b_list, scales = [], [], []
    for ad in range(n_adapters):
        r = int(ranks[ad])
        a_list.append(_randn(g, (r, k), 1 / math.sqrt(k), device, dtype))
        b_list.append(_randn(g, (n, r), 1 / math.sqrt(r), device, dtype))
        scales.append(2.0 * r / r)  # alpha_a / r_a with alpha_a = 2 r_a
    x = _randn(g, (tokens, k), 1.0, device, dtype)
    w = _randn(g, (n, k), 1 / math.sqrt(k), device, dtype)
    offsets = torch.zeros(n_adapters, dtype=torch.int64, device=device)
    offsets[1:] = torch.cumsum(ranks.to(torch.int64), 0)[:-1]
    a_flat = torch.cat(a_list, 0)
    b_flat = torch.cat([(bl.float() * s).t().to(dtype) for bl, s in zip(b_list, scales)], 0).contiguous()
    seg_start = torch.zeros(segments + 1, dtype=torch.int64, device=device)
    seg_start[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64, device=device), 0)
    return Segmented(x, w, a_flat, b_flat, offsets, ranks.to(torch.int64), seg_start, seg_adapter.to(torch.int64),
                     scales, a_list, b_list)


def stack_folded(adapters, dtype):
    """Stack adapters the way ``attach_fused_lora`` does: the first alpha is the
    layer's scale, every later down factor is multiplied by alpha_i / alpha_0 in
    fp32 and rounded back to ``dtype``, and the factors are concatenated along
    the rank.  Returns (a [sum r, K], b [N, sum r], scale)."""
    scale = float(adapters[0][2])
    a_parts = [adapters[0][0].to(dtype)]
    for down, _, alpha in adapters[1:]:
        a_parts.append(((float(alpha) / scale) * down.float()).to(dtype))
    a = torch.cat(a_parts, 0).contiguous()
    b = torch.cat([up.to(dtype) for _, up, _ in adapters], 1).contiguous()
    return a, b, scale


def _projection(g, name, m, k, n, ranks_scales, device, dtype, x=None):
    """One projection whose adapters (drawn per rank, stored in ``dtype`` like
    adapter files) are stacked with attach_fused_lora semantics."""
    if x is None:
        x = _randn(g, (m, k), 1.0, device, dtype)
    w = _randn(g, (n, k), 1 / math.sqrt(k), device, dtype)
    adapters = []
    for r, s in ranks_scales:
        down = _randn(g, (r, k), 1 / math.sqrt(k), device, dtype)
        up = _randn(g, (n, r), 1 / math.sqrt(r), device, dtype)
        adapters.append((down, up, s))
    a, b, scale = stack_folded(adapters, dtype)
    return Projection(name, k, n, x, w, a, b, scale, adapters=adapters)


def c4(device="cuda", dtype=torch.bfloat16, m=8192) -> list[Projection]:
    """C4: Llama-7B layer prefill, M = 8192, r = 16 LoRA on q,k,v,o,gate,up,down, scale 2.0."""
    g = _gen(3, device)
    h, f = HIDDEN_LLAMA, FFN_LLAMA
    shapes = [("q", h, h), ("k", h, h), ("v", h, h), ("o", h, h), ("gate", h, f), ("up", h, f), ("down", f, h)]
    return [_projection(g, nm, m, k, n, [(16, 2.0)], device, dtype) for nm, k, n in shapes]


C5_STACK = ((32, 1.0), (64, 0.7), (128, 0.4))
C5_SHAPES = (("q", HIDDEN_WAN, HIDDEN_WAN), ("k", HIDDEN_WAN, HIDDEN_WAN), ("v", HIDDEN_WAN, HIDDEN_WAN),
             ("o", HIDDEN_WAN, HIDDEN_WAN), ("ffn_up", HIDDEN_WAN, FFN_WAN), ("ffn_down", FFN_WAN, HIDDEN_WAN))


def c5(device="cuda", dtype=torch.bfloat16, m=32760, only=None, rows=None) -> list[Projection]:
    """C5: Wan DiT projections, M = 32760 tokens, 3-LoRA stack r = 32/64/128 with weights 1.0/0.7/0.4.

    ``only`` keeps a subset of the projection names; the draws of the others
    still happen (on the device they are cheap), so every projection's values
    do not depend on which ones are kept.  ``rows = (start, stop)`` keeps that
    token range of each projection's x (the rank's shard of the batch); the
    weights and adapters, drawn after the full batch's x, are the same on
    every rank.
    """
    g = _gen(4, device)
    out = []
    for nm, k, n in C5_SHAPES:
        x = _randn(g, (m, k), 1.0, device, dtype)
        if rows is not None:
            x = x[rows[0]:rows[1]].clone()
        p = _projection(g, nm, m, k, n, C5_STACK, device, dtype, x=x)
        if only is None or nm in only:
            out.append(p)
        del p, x
    return out


def c5_flops(m=32760) -> float:
    h, f = HIDDEN_WAN, FFN_WAN
    shapes = [(h, h)] * 4 + [(h, f), (f, h)]
    return sum(2.0 * m * k * n + 2.0 * m * 224 * (k + n) for k, n in shapes)
