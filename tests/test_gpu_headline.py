"""Parity at the benchmarked configurations' own shapes.

The bench times C5 (M = 32760, q/k/v/o 5120->5120, FFN 5120->13824->5120, a
3-LoRA stack r = 32 + 64 + 128 = 224) and C4 (M = 8192, the seven Llama-7B
projections at r = 16); C2 is the decode shape at M = 1, 4, 16, 64.  These
tests run those exact shapes through the public API -- ``attach_fused_lora``
three times for the C5 stack, ``fused_lora_linear`` for C2 and C4 -- and check
the whole output against the float64 oracle: sampled rows element by element
(the bf16 bars), every row sum, and a signed token sketch that mixes every row
into every column (``oracle/checks.py``).  The shard sizes of the multi-GPU
split (4095 and 8190 tokens of C5) are checked the same way.
Reference check being mirrored: test_fused_linear.py:49-78 (variants against
the naive path on seeded inputs).
"""

import numpy as np
import pytest
import torch
from torch import nn

from oracle import checks
from oracle import lora_oracle as orc
from probe_b200 import attach_fused_lora, fused_lora_linear, total_fused_rank, workloads
from tests.helpers import assert_parity, np64

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _stacked_oracle_factors(p):
    """The stacked factors the reference's attach_fused_lora builds from p's adapters."""
    a64, b64, scale = orc.stack_adapters([(np64(d), np64(u), al) for d, u, al in p.adapters], dtype="bf16")
    return a64, b64, scale


def _attach_three(p):
    holder = nn.Module()
    lin = nn.Linear(p.k, p.n, bias=False, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(p.w)
    holder.proj = lin
    for down, up, alpha in p.adapters:
        attach_fused_lora(holder, "proj", down, up, alpha=alpha)
    return holder


@pytest.mark.parametrize("name", ["q", "ffn_up", "ffn_down"])
@pytest.mark.parametrize("m", [32760, 4095])
def test_c5_projection_full_size(name, m):
    (p,) = workloads.c5(device=DEV, m=m, only={name})
    holder = _attach_three(p)
    assert holder.proj.rank == 224 and total_fused_rank(holder) == 224
    # the module's stacked factors are the reference's, bit for bit
    a64, b64, scale = _stacked_oracle_factors(p)
    assert np.array_equal(np64(holder.proj.lora_a), a64) and np.array_equal(np64(holder.proj.lora_b), b64)
    assert scale == holder.proj.scale == 1.0
    with torch.no_grad():
        out = holder.proj(p.x)
    torch.cuda.synchronize()
    rep = checks.linear_report(out, p.x, p.w, None, a64, b64, scale, seed=m)
    assert rep["ok"], rep
    # the bench's own path (pre-stacked factors, same kernels) gives the same bits
    from probe_b200.fused_linear import _KConcat

    same = _KConcat(p.w, None, p.a, p.b, p.scale)(p.x)
    assert torch.equal(same, out)


def test_c5_shard_8190_q():
    (p,) = workloads.c5(device=DEV, m=8190, only={"q"})
    a64, b64, scale = _stacked_oracle_factors(p)
    out = fused_lora_linear(p.x, p.w, None, p.a, p.b, p.scale)
    rep = checks.linear_report(out, p.x, p.w, None, a64, b64, scale, seed=3)
    assert rep["ok"], rep


def test_c4_all_projections():
    projs = workloads.c4(device=DEV)
    assert [p.name for p in projs] == ["q", "k", "v", "o", "gate", "up", "down"]
    for i, p in enumerate(projs):
        out = fused_lora_linear(p.x, p.w, None, p.a, p.b, p.scale)
        rep = checks.linear_report(out, p.x, p.w, None, p.a, p.b, p.scale, seed=i)
        assert rep["ok"], (p.name, rep)
        del out


@pytest.mark.parametrize("m", [1, 4, 16, 64])
def test_c2_decode_shapes(m):
    p = workloads.c2(m, device="cpu")
    x, w, a, b = (t.to(DEV, torch.bfloat16) for t in (p.x, p.w, p.a, p.b))
    out = fused_lora_linear(x, w, None, a, b, p.scale)
    assert_parity(out, orc.naive_linear(np64(x), np64(w), None, np64(a), np64(b), p.scale))


def test_c1_through_module():
    p = workloads.c1(device="cpu")
    lin = nn.Linear(p.k, p.n, bias=False, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(p.w)
    holder = nn.Module()
    holder.proj = lin
    attach_fused_lora(holder, "proj", p.a.to(DEV, torch.bfloat16), p.b.to(DEV, torch.bfloat16), alpha=p.scale)
    x = p.x.to(DEV, torch.bfloat16)
    out = holder.proj(x)
    assert_parity(out, orc.naive_linear(np64(x), np64(holder.proj.weight), None, np64(holder.proj.lora_a),
                                        np64(holder.proj.lora_b), p.scale))
