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


def _projection(g, name, m, k, n, ranks_scales, device, dtype, x=None):
    """One projection; adapters stacked with attach_fused_lora semantics (first alpha = layer scale)."""
    if x is None:
        x = _randn(g, (m, k), 1.0, device, dtype)
    w = _randn(g, (n, k), 1 / math.sqrt(k), device, dtype)
    a_blocks, b_blocks = [], []
    base_scale = ranks_scales[0][1]
    for r, s in ranks_scales:
        a = _randn(g, (r, k), 1 / math.sqrt(k), device, torch.float32)
        b = _randn(g, (n, r), 1 / math.sqrt(r), device, torch.float32)
        a_blocks.append((s / base_scale) * a)
        b_blocks.append(b)
    a = torch.cat(a_blocks, 0).to(dtype)
    b = torch.cat(b_blocks, 1).to(dtype).contiguous()
    return Projection(name, k, n, x, w, a, b, base_scale)


def c4(device="cuda", dtype=torch.bfloat16, m=8192) -> list[Projection]:
    """C4: Llama-7B layer prefill, M = 8192, r = 16 LoRA on q,k,v,o,gate,up,down, scale 2.0."""
    g = _gen(3, device)
    h, f = HIDDEN_LLAMA, FFN_LLAMA
    shapes = [("q", h, h), ("k", h, h), ("v", h, h), ("o", h, h), ("gate", h, f), ("up", h, f), ("down", f, h)]
    return [_projection(g, nm, m, k, n, [(16, 2.0)], device, dtype) for nm, k, n in shapes]


def c5(device="cuda", dtype=torch.bfloat16, m=32760) -> list[Projection]:
    """C5: Wan DiT projections, M = 32760 tokens, 3-LoRA stack r = 32/64/128 with weights 1.0/0.7/0.4."""
    g = _gen(4, device)
    h, f = HIDDEN_WAN, FFN_WAN
    stack = [(32, 1.0), (64, 0.7), (128, 0.4)]
    shapes = [("q", h, h), ("k", h, h), ("v", h, h), ("o", h, h), ("ffn_up", h, f), ("ffn_down", f, h)]
    return [_projection(g, nm, m, k, n, stack, device, dtype) for nm, k, n in shapes]


def c5_flops(m=32760) -> float:
    h, f = HIDDEN_WAN, FFN_WAN
    shapes = [(h, h)] * 4 + [(h, f), (f, h)]
    return sum(2.0 * m * k * n + 2.0 * m * 224 * (k + n) for k, n in shapes)
