#!/usr/bin/env python3
"""Generate the golden vectors in this directory by running the reference itself.

Usage:  python tests/golden/make_golden.py --reference <checkout of lishenghui/probe>

The reference (``loraforge_kernels``) is imported from that checkout and run
on the CPU:
  * its CPU LoRA-linear path: ``fused_lora_linear`` on CPU tensors dispatches
    to ``_torch_naive`` (fused_linear.py:527-551, :376-378), in fp32;
  * its segmented / ragged branch Triton kernels (segmented_branch.py,
    ragged_branch.py) under the Triton interpreter (TRITON_INTERPRET=1), in
    fp32 -- the interpreter mis-evaluates bf16, so inputs are bf16-representable
    values held in fp32;
  * its multi-adapter stacking (attach_fused_lora, runtime_lora.py:29-61) on a
    CPU nn.Linear, whose forward again takes the _torch_naive path;
  * its integer helpers (pad_rank, packed_rank, align_to_deploy_rank,
    rank_tile, auto_split_k).
Every floating-point input is rounded to bfloat16 first, so the same values
can be fed to the bf16 GPU kernels exactly; inputs are stored as bfloat16 bit
patterns (uint16), outputs as float32.
The generated files are committed; nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def bf16(t):
    import torch

    return t.to(torch.bfloat16).to(torch.float32)


def bits(t):
    """bfloat16 bit patterns (uint16) of a bf16-representable float tensor."""
    import numpy as np
    import torch

    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the lishenghui/probe checkout")
    args = ap.parse_args()

    os.environ["TRITON_INTERPRET"] = "1"
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(Path(args.reference).resolve()))
    sys.path.insert(0, str(REPO))

    import numpy as np
    import torch

    from loraforge_kernels import fused_linear as ref_fl
    from loraforge_kernels import multilora as ref_ml
    from loraforge_kernels import ragged_branch as ref_rb
    from loraforge_kernels import runtime_lora as ref_rt
    from loraforge_kernels import segmented_branch as ref_sb
    from loraforge_kernels import splitk_lora as ref_sl
    from loraforge_kernels import splitk_shrink as ref_ss

    from probe_b200 import workloads

    torch.set_num_threads(os.cpu_count() or 1)

    # ---------------------------------------------------------- integer helpers
    ints = {
        "pad_rank": {r: ref_fl.pad_rank(r) for r in range(1, 301)},
        "packed_rank": {r: ref_fl.packed_rank(r) for r in range(0, 301)},
        "align_to_deploy_rank": {r: ref_sl.align_to_deploy_rank(r) for r in range(1, 301)},
        "splitk_rank_tile": {r: ref_ss.rank_tile(r) for r in range(1, 301)},
        "multilora_rank_tile": {r: ref_ml.rank_tile(r) for r in range(1, 301)},
        "auto_split_k": {n: ref_ml.auto_split_k(n) for n in list(range(0, 130)) + [255, 256, 257, 1000, 2048,
                                                                               4096, 5000, 32760]},
        "deploy_rank_buckets": list(ref_sl.DEPLOY_RANK_BUCKETS),
        "constants": {"MIN_GEMM_ROWS": ref_fl.MIN_GEMM_ROWS, "FUSED_MAX_RANK": ref_fl.FUSED_MAX_RANK,
                      "MIN_RANK_TILE": ref_fl.MIN_RANK_TILE, "PACK_ALIGN": ref_fl.PACK_ALIGN},
    }
    (HERE / "int_helpers.json").write_text(json.dumps(ints, indent=0, sort_keys=True))

    # -------------------------------------------------- single-adapter linear
    g = torch.Generator().manual_seed(20240)
    cases = [  # m, k, n, r, bias, scale  (shapes from test_fused_linear.py:53-54 and odd sizes)
        (64, 256, 192, 16, True, 2.0),
        (33, 128, 96, 7, True, 0.75),
        (16, 512, 320, 40, False, -0.7),
        (130, 320, 320, 17, True, 0.75),
        (8, 384, 512, 64, True, 0.5),
        (200, 256, 136, 1, False, 1.25),
    ]
    lin = {}
    for i, (m, k, n, r, has_bias, scale) in enumerate(cases):
        x = bf16(torch.randn(m, k, generator=g))
        w = bf16(torch.randn(n, k, generator=g) / math.sqrt(k))
        a = bf16(torch.randn(r, k, generator=g) / math.sqrt(k))
        b = bf16(torch.randn(n, r, generator=g) / math.sqrt(r))
        bias = bf16(torch.randn(n, generator=g)) if has_bias else None
        out = ref_fl.fused_lora_linear(x, w, bias, a, b, scale)
        lin[f"c{i}_x"], lin[f"c{i}_w"], lin[f"c{i}_a"], lin[f"c{i}_b"] = bits(x), bits(w), bits(a), bits(b)
        lin[f"c{i}_bias"] = bits(bias) if bias is not None else np.zeros(0, np.uint16)
        lin[f"c{i}_scale"] = np.float32(scale)
        lin[f"c{i}_out"] = out.numpy()
    # leading dimensions: fused_lora_linear reshapes [..., K]
    x3 = bf16(torch.randn(2, 5, 128, generator=g))
    w3 = bf16(torch.randn(64, 128, generator=g) / math.sqrt(128))
    a3 = bf16(torch.randn(8, 128, generator=g) / math.sqrt(128))
    b3 = bf16(torch.randn(64, 8, generator=g) / math.sqrt(8))
    lin["nd_x"], lin["nd_w"], lin["nd_a"], lin["nd_b"] = bits(x3), bits(w3), bits(a3), bits(b3)
    lin["nd_out"] = ref_fl.fused_lora_linear(x3, w3, None, a3, b3, 0.8).numpy()
    lin["n_cases"] = np.int64(len(cases))
    np.savez_compressed(HERE / "linear_cases.npz", **lin)

    # ------------------------------------------------ C1 (full size) checksums
    p = workloads.c1(device="cpu", dtype=torch.float32)
    c1 = {"x_head": p.x.flatten()[:16].numpy(), "w_head": p.w.flatten()[:16].numpy(),
          "a_head": p.a.flatten()[:16].numpy(), "b_head": p.b.flatten()[:16].numpy()}
    rows = np.array([0, 1, 100, 255])
    for tag, cast in (("f32", lambda t: t), ("bf16in", bf16)):
        out = ref_fl.fused_lora_linear(cast(p.x), cast(p.w), None, cast(p.a), cast(p.b), p.scale)
        c1[f"{tag}_rows"] = out[rows].numpy()
        c1[f"{tag}_row_sums"] = out.sum(1).numpy()
        c1[f"{tag}_fro"] = np.float64(torch.linalg.vector_norm(out.double()).item())
    c1["rows"] = rows
    np.savez_compressed(HERE / "c1_checksums.npz", **c1)

    # ------------------------------------------- multi-adapter branch kernels
    g = torch.Generator().manual_seed(777)
    k, n = 128, 96
    ranks = torch.tensor([4, 8, 0, 16, 3], dtype=torch.int64)
    offsets = torch.zeros_like(ranks)
    offsets[1:] = torch.cumsum(ranks, 0)[:-1]
    tot = int(ranks.sum())
    a_flat = bf16(torch.randn(tot, k, generator=g) / math.sqrt(k))
    b_flat = bf16(torch.randn(tot, n, generator=g) * 0.3)  # scale folded into B
    # ragged: per-token ids with runs and isolated tokens, including the rank-0 adapter
    ids = torch.tensor([0] * 5 + [3] * 9 + [1] + [2] * 4 + [4] * 7 + [1] * 3 + [0] + [3] * 18, dtype=torch.int64)
    t = ids.numel()
    x = bf16(torch.randn(t, k, generator=g))
    y = bf16(torch.randn(t, n, generator=g))
    rag = ref_rb.branch(x, y, a_flat, b_flat, offsets, ranks, ids, int(ranks.max()))
    rag_noskip = ref_rb.branch(x, y, a_flat, b_flat, offsets, ranks, ids, int(ranks.max()), skip_zero=False)
    # segmented: 4 requests x 12 tokens
    req = torch.tensor([3, 0, 4, 1], dtype=torch.int64)
    xs = bf16(torch.randn(48, k, generator=g))
    ys = bf16(torch.randn(48, n, generator=g))
    seg = ref_sb.segmented_branch(xs, ys, a_flat, b_flat, offsets, ranks, req, 12, int(ranks.max()))
    np.savez_compressed(
        HERE / "branch_cases.npz", a_flat=bits(a_flat), b_flat=bits(b_flat), offsets=offsets.numpy(),
        ranks=ranks.numpy(), ids=ids.numpy(), x=bits(x), y=bits(y), ragged_out=rag.numpy(),
        ragged_noskip_out=rag_noskip.numpy(), req=req.numpy(), xs=bits(xs), ys=bits(ys), seg_out=seg.numpy())

    # ------------------------------------------------------ adapter stacking
    g = torch.Generator().manual_seed(4242)
    base = torch.nn.Linear(64, 48, bias=True)
    with torch.no_grad():
        base.weight.copy_(bf16(torch.randn(48, 64, generator=g) / 8))
        base.bias.copy_(bf16(torch.randn(48, generator=g)))
    holder = torch.nn.Module()
    holder.proj = base
    adapters = []
    for r, alpha in ((4, 1.0), (8, 0.7), (16, 0.4)):
        down = bf16(torch.randn(r, 64, generator=g) / 8)
        up = bf16(torch.randn(48, r, generator=g) / math.sqrt(r))
        adapters.append((down, up, alpha))
        ref_rt.attach_fused_lora(holder, "proj", down, up, alpha)
    xq = bf16(torch.randn(10, 64, generator=g))
    with torch.no_grad():
        stacked_out = holder.proj(xq)
    st = {"w": bits(base.weight.detach()), "bias": bits(base.bias.detach()), "x": bits(xq),
          "out": stacked_out.numpy(), "lora_a": holder.proj.lora_a.numpy(), "lora_b": holder.proj.lora_b.numpy(),
          "scale": np.float32(holder.proj.scale), "rank": np.int64(holder.proj.rank)}
    for i, (down, up, alpha) in enumerate(adapters):
        st[f"down{i}"], st[f"up{i}"], st[f"alpha{i}"] = bits(down), bits(up), np.float32(alpha)
    np.savez_compressed(HERE / "stack_case.npz", **st)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
