"""Launch ordering under programmatic dependent launch (GPU).

Most kernels of this library launch with programmatic stream serialization:
they may start while the kernel launched just before them on the stream is
still running, and read only weights before griddepcontrol.wait.  Each case
here puts the producer of a kernel's activations (or of its tile table)
IMMEDIATELY before it on the stream, with nothing in between, and checks the
consumer against the float64 oracle evaluated on what the producer wrote:

* the register-path decode kernel (K not a multiple of 8), base only and with
  a z input, reading an x that the small-M linear has just written (that
  linear signals its dependents as soon as it starts);
* the tcgen05 z-consuming form of the small-M linear reading a just-written x;
* the segmented expand launched straight after a schedule that rewrote the
  tile table it reads (the buffer still holding another batch's table);
* back-to-back segmented branches whose segment tables differ.
"""

import math

import pytest
import torch

from oracle import lora_oracle as orc
from probe_b200 import _lib, kernels
from tests.helpers import assert_parity, np64, randn

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _producer(m, k_in, n_out, seed):
    """x0 and the weights of a small-M LoRA linear writing an [m, n_out] x."""
    x0 = randn((m, k_in), 1.0, seed=seed)
    w1 = randn((n_out, k_in), 1 / math.sqrt(k_in), seed=seed + 1)
    a1 = randn((16, k_in), 1 / math.sqrt(k_in), seed=seed + 2)
    b1 = randn((n_out, 16), 0.25, seed=seed + 3)
    return x0, w1, a1, b1


@pytest.mark.parametrize("with_z", [False, True])
def test_decode_kernel_waits_for_its_x(with_z):
    m, k_in, k, n, r = 64, 1024, 1002, 520, 8  # K = 1002: the register-path decode kernel
    w2 = randn((n, k), 1 / math.sqrt(k), seed=11)
    bias = randn((n,), 1.0, seed=12)
    b2 = randn((n, r), 0.25, seed=13)
    for it in range(6):
        x0, w1, a1, b1 = _producer(m, k_in, k, seed=100 + 10 * it)
        z = randn((m, r), 1.0, torch.float32, seed=200 + it) if with_z else None
        torch.cuda.synchronize()
        x1 = kernels.linear_small(x0, w1, a1, b1, None, 1.0)  # writes x, signals dependents at once
        out = kernels.decode_linear(x1, w2, z, b2 if with_z else None, bias, 0.5 if with_z else 0.0)
        torch.cuda.synchronize()
        want = np64(x1) @ np64(w2).T + np64(bias)
        if with_z:
            want += 0.5 * np64(z) @ np64(b2).T
        assert_parity(out, want)
    assert _lib.device_error() == 0


def test_skinny_z_form_waits_for_its_x():
    m, k, n, r = 64, 1024, 2048, 16
    w2 = randn((n, k), 1 / math.sqrt(k), seed=21)
    b2 = randn((n, r), 0.25, seed=22)
    for it in range(6):
        x0, w1, a1, b1 = _producer(m, 2048, k, seed=300 + 10 * it)
        z = randn((m, r), 1.0, torch.float32, seed=400 + it)
        torch.cuda.synchronize()
        x1 = kernels.linear_small(x0, w1, a1, b1, None, 1.0)
        out = kernels.decode_linear(x1, w2, z, b2, None, 0.75)  # tcgen05 form fed a z
        torch.cuda.synchronize()
        want = np64(x1) @ np64(w2).T + 0.75 * np64(z) @ np64(b2).T
        assert_parity(out, want)
    assert _lib.device_error() == 0


def _tables(ranks, k, n, seed):
    g = torch.Generator().manual_seed(seed)
    ranks_t = torch.tensor(ranks, dtype=torch.int64)
    offs = torch.zeros_like(ranks_t)
    offs[1:] = torch.cumsum(ranks_t, 0)[:-1]
    tot = int(ranks_t.sum())
    a = (torch.randn(tot, k, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    b = (torch.randn(tot, n, generator=g) * 0.2).to(torch.bfloat16)
    return a.to(DEV), b.to(DEV), offs.to(DEV), ranks_t.to(DEV)


def _segments(t, count, n_adapters, seed, skew):
    """``count`` segments over t tokens (the same table layout for every call
    with the same count), lengths skewed by ``skew``; valid adapter ids."""
    gen = torch.Generator().manual_seed(seed)
    weights = torch.rand(count, generator=gen) ** skew + 1e-3
    lens = torch.clamp((weights / weights.sum() * (t - count)).floor().long(), min=0) + 1
    lens[-1] += t - int(lens.sum())
    seg = torch.zeros(count + 1, dtype=torch.int64)
    seg[1:] = torch.cumsum(lens, 0)
    seg_ad = torch.randint(0, n_adapters, (count,), generator=gen)
    return seg.to(DEV), seg_ad.to(DEV)


def _want_branch(x, y, a, b, offs, ranks, ids):
    xv, yv, av, bv = np64(x), np64(y), np64(a), np64(b)
    o, r = offs.cpu().numpy(), ranks.cpu().numpy()
    out = yv.copy()
    for t, ad in enumerate(ids):
        if 0 <= ad < len(r) and r[ad] > 0:
            rows = slice(int(o[ad]), int(o[ad] + r[ad]))
            out[t] += (xv[t] @ av[rows].T) @ bv[rows]
    return out


def _schedule_into(buf, t, n_adapters, seg_start, seg_ad):
    _lib.call("lora_sgmv_schedule", None, _lib.ptr(seg_start), _lib.ptr(seg_ad), t, seg_ad.numel(), n_adapters,
              _lib.ptr(buf), buf.numel() * 4, _lib.stream_handle(buf.device))


def test_expand_right_after_a_schedule_that_rewrote_its_table():
    t, k, n = 1024, 512, 384
    ranks = [4, 8, 16, 32, 64] * 2
    a, b, offs, rk = _tables(ranks, k, n, seed=5)
    x = randn((t, k), 1.0, seed=6)
    y = randn((t, n), 1.0, seed=7)
    lib = _lib.load()
    buf = torch.zeros((lib.lora_sgmv_tiles_size(t, 96) + 3) // 4, dtype=torch.int32, device=DEV)
    for it in range(4):
        # the same segment count (one table layout), different boundaries and adapters
        seg_a = _segments(t, 96, len(ranks), seed=40 + it, skew=6.0)
        seg_b = _segments(t, 96, len(ranks), seed=60 + it, skew=0.5)
        ids_b = orc.segments_to_ids(seg_b[0].cpu().numpy(), seg_b[1].cpu().numpy())
        tiles_b, s_b = kernels.sgmv_schedule(t, len(ranks), seg_start=seg_b[0], seg_adapter=seg_b[1])
        z_b = kernels.sgmv_shrink(x, a, offs, rk, tiles_b, s_b, max(ranks), z_dtype=torch.float32)
        _schedule_into(buf, t, len(ranks), *seg_a)  # the shared buffer holds batch a's table
        torch.cuda.synchronize()
        _schedule_into(buf, t, len(ranks), *seg_b)  # rewritten, and read by the very next launch
        out = kernels.sgmv_expand(y, z_b, b, n, 1, offs, rk, buf, seg_b[1].numel(), n, max(ranks))
        torch.cuda.synchronize()
        assert_parity(out, _want_branch(x, y, a, b, offs, rk, ids_b))
    assert _lib.device_error() == 0


def test_back_to_back_branches_with_different_segments():
    from probe_b200.segmented_branch import segmented_branch_varlen

    t, k, n = 2048, 1024, 256
    ranks = [4, 8, 16, 32, 64] * 3
    a, b, offs, rk = _tables(ranks, k, n, seed=8)
    x = randn((t, k), 1.0, seed=9)
    y = randn((t, n), 1.0, seed=10)
    cases = [_segments(t, 128, len(ranks), seed=80 + i, skew=(0.3, 3.0, 8.0)[i % 3]) for i in range(6)]
    torch.cuda.synchronize()
    outs = [segmented_branch_varlen(x, y, a, b, offs, rk, s, ad, max(ranks)) for s, ad in cases]
    torch.cuda.synchronize()
    for out, (s, ad) in zip(outs, cases):
        ids = orc.segments_to_ids(s.cpu().numpy(), ad.cpu().numpy())
        assert_parity(out, _want_branch(x, y, a, b, offs, rk, ids))
    assert _lib.device_error() == 0


def test_plain_stream_order_switch_is_read():
    """LORA_B200_PDL=0 (plain stream order) gives the same bits as the default,
    through the small-M linear, the decode kernel, the schedule, both
    segmented shrinks (tensor-core, and the cluster block kernel reached with a
    row indirection) and the segmented expand."""
    import os
    import subprocess
    import sys

    code = (
        "import torch, math\n"
        "from probe_b200 import kernels\n"
        "from tests.helpers import randn\n"
        "x = randn((64, 1024), 1.0, seed=1)\n"
        "w = randn((1002, 1024), 1 / 32, seed=2)\n"
        "a = randn((16, 1024), 1 / 32, seed=3)\n"
        "b = randn((1002, 16), 0.25, seed=4)\n"
        "w2 = randn((300, 1002), 1 / 32, seed=5)\n"
        "y = kernels.decode_linear(kernels.linear_small(x, w, a, b, None, 1.0), w2, None, None, None, 0.0)\n"
        "ranks = torch.tensor([4, 8, 16, 32, 64, 16], device='cuda')\n"
        "offs = torch.cumsum(ranks, 0) - ranks\n"
        "af = randn((140, 512), 1 / 23, seed=6)\n"
        "bf = randn((140, 256), 0.2, seed=7)\n"
        "xs = randn((700, 512), 1.0, seed=8)\n"
        "ys = randn((700, 256), 1.0, seed=9)\n"
        "seg = torch.tensor([0, 3, 90, 91, 300, 310, 512, 700], device='cuda')\n"
        "sad = torch.tensor([1, 5, 0, 4, 2, 3, 4], device='cuda')\n"
        "tiles, s = kernels.sgmv_schedule(700, 6, seg_start=seg, seg_adapter=sad)\n"
        "z_tc = kernels.sgmv_shrink(xs, af, offs, ranks, tiles, s, 64)\n"
        "z_blk = kernels.sgmv_shrink(xs, af, offs, ranks, tiles, s, 64, rows=torch.arange(700, device='cuda'))\n"
        "o = kernels.sgmv_expand(ys, z_tc, bf, 256, 1, offs, ranks, tiles, s, 256, 64)\n"
        "torch.save([t.cpu() for t in (y, z_tc, z_blk, o)], __import__('sys').argv[1])\n"
    )
    results = []
    for flag in ("1", "0"):
        path = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"pdl_{flag}_{os.getpid()}.pt")
        env = dict(os.environ, LORA_B200_PDL=flag)
        subprocess.run([sys.executable, "-c", code, path], check=True, env=env, timeout=300,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        results.append(torch.load(path))
        os.remove(path)
    for got, want in zip(results[1], results[0]):
        assert torch.equal(got, want)
