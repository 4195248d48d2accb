"""Compact adapters and their SGMV tables (CPU).

Follows the reference's own test (test_compact_adapter.py:18-80): heterogeneous
ranks 0 / 1 / 3 cut from padded rank 8, plain LoRA and rsLoRA, a per-module
alpha pattern, an all-zero adapter (base only) and a refused cut of a live
coordinate.  PEFT is not installed here, so the compact adapter is checked by
the LoRA math in fp64 instead of a PEFT reload.  Then the packing of several
adapters into the flat tables the segmented kernels read.
"""

import json

import pytest
import torch

from probe_b200 import compact_adapter as ca


def _padded(ranks, k=7, n=5, r=8, seed=83):
    g = torch.Generator().manual_seed(seed)
    tensors = {}
    for i, rank in enumerate(ranks):
        a, b = torch.zeros(r, k), torch.zeros(n, r)
        a[:rank] = torch.randn(rank, k, generator=g)
        b[:, :rank] = torch.randn(n, rank, generator=g)
        tensors[f"base_model.model.blocks.{i}.lora_A.weight"] = a
        tensors[f"base_model.model.blocks.{i}.lora_B.weight"] = b
    return tensors


def _config(rslora):
    return dict(peft_type="LORA", r=8, lora_alpha=16, lora_dropout=0.05, target_modules=["0", "1", "2"],
                bias="none", use_rslora=rslora, alpha_pattern={r"blocks\.1": 5.5})


def _lora_sum(tensors, config, x):
    out = torch.zeros(x.shape[0], 5, dtype=torch.float64)
    for key in sorted(k for k in tensors if k.endswith(".lora_A.weight")):
        name = ca.module_name(key)
        a = tensors[key].double()
        b = tensors[key.replace(".lora_A.", ".lora_B.")].double()
        out += ca.lora_scale(config, name) * ((x @ a.T) @ b.T)
    return out


@pytest.mark.parametrize("rslora", [False, True])
def test_compaction_keeps_outputs(tmp_path, rslora):
    ranks = [0, 1, 3]
    tensors, config = _padded(ranks), _config(rslora)
    compact, cfg, manifest = ca.compact_zero_padded(tensors, config, ranks)
    assert manifest["compact_elements"] == 4 * (7 + 5)
    assert manifest["padded_elements"] == 3 * 8 * (7 + 5)
    assert manifest["zero_modules"] == 1 and manifest["active_modules"] == 2
    assert len(compact) == 4
    x = torch.randn(4, 7, dtype=torch.float64)
    torch.testing.assert_close(_lora_sum(compact, cfg, x), _lora_sum(tensors, config, x), rtol=1e-10, atol=1e-11)
    # the same through the files: export, then read back
    from safetensors.torch import load_file, save_file

    src = tmp_path / "source"
    src.mkdir()
    save_file(tensors, src / "adapter_model.safetensors")
    (src / "adapter_config.json").write_text(json.dumps(config))
    ca.export_compact(src, tmp_path / "compact", ranks)
    back = load_file(tmp_path / "compact" / "adapter_model.safetensors")
    back_cfg = json.loads((tmp_path / "compact" / "adapter_config.json").read_text())
    assert back["base_model.model.blocks.2.lora_A.weight"].shape == (3, 7)
    assert back["base_model.model.blocks.1.lora_B.weight"].shape == (5, 1)
    assert "base_model.model.blocks.0.lora_A.weight" not in back
    torch.testing.assert_close(_lora_sum(back, back_cfg, x), _lora_sum(tensors, config, x), rtol=1e-10, atol=1e-11)
    with pytest.raises(ValueError):
        ca.export_compact(src, tmp_path / "compact", ranks)  # refuses to overwrite


def test_all_zero_is_base_only_and_live_tail_is_refused():
    ranks = [0, 1, 3]
    tensors, config = _padded(ranks), _config(False)
    zeros = {k: torch.zeros_like(v) for k, v in tensors.items()}
    out, _, info = ca.compact_zero_padded(zeros, config, [0, 0, 0])
    assert not out and info["base_only"] and info["compact_elements"] == 0
    bad = {k: v.clone() for k, v in tensors.items()}
    bad["base_model.model.blocks.1.lora_A.weight"][7].fill_(1)
    bad["base_model.model.blocks.1.lora_B.weight"][:, 7].fill_(1)
    with pytest.raises(ValueError, match="nonzero"):
        ca.compact_zero_padded(bad, config, ranks)
    with pytest.raises(ValueError, match="Allocation"):
        ca.compact_zero_padded(tensors, config, [1, 2])
    with pytest.raises(ValueError, match="bias-free"):
        ca.compact_zero_padded(tensors, dict(config, use_dora=True), ranks)


def test_bucket_zero_pad_is_exact():
    g = torch.Generator().manual_seed(5)
    tensors = {}
    pattern = {}
    for i, r in enumerate([3, 5, 16]):
        tensors[f"m.layer{i}.lora_A.weight"] = torch.randn(r, 6, generator=g)
        tensors[f"m.layer{i}.lora_B.weight"] = torch.randn(4, r, generator=g)
        pattern[f"layer{i}"] = r
    config = dict(r=16, lora_alpha=16, rank_pattern=pattern)
    out, cfg, report = ca.bucket_zero_pad(tensors, config, maximum=32)
    assert [d["new_rank"] for d in report] == [4, 8, 16]
    assert cfg["rank_pattern"] == {"layer0": 4, "layer1": 8, "layer2": 16}
    x = torch.randn(2, 6)
    for i in range(3):
        a, b = out[f"m.layer{i}.lora_A.weight"], out[f"m.layer{i}.lora_B.weight"]
        a0, b0 = tensors[f"m.layer{i}.lora_A.weight"], tensors[f"m.layer{i}.lora_B.weight"]
        torch.testing.assert_close((x @ a.T) @ b.T, (x @ a0.T) @ b0.T)
    with pytest.raises(ValueError, match="largest bucket"):
        ca.bucket_zero_pad(tensors, config, maximum=8)


def test_sgmv_tables_from_compact_adapters(tmp_path):
    """Three adapters of one module (one with the module cut to rank 0) packed
    into the flat tables; the ragged-branch math on them equals each adapter's
    own LoRA output."""
    from safetensors.torch import save_file

    dirs = []
    for j, ranks in enumerate([[2, 1, 3], [0, 0, 0], [1, 2, 0]]):
        tensors, config = _padded(ranks, seed=10 + j), _config(j == 2)
        src = tmp_path / f"src{j}"
        src.mkdir()
        save_file(tensors, src / "adapter_model.safetensors")
        (src / "adapter_config.json").write_text(json.dumps(config))
        ca.export_compact(src, tmp_path / f"compact{j}", ranks)
        dirs.append((tmp_path / f"compact{j}", tensors, config))
    a_flat, b_flat, offsets, rk = ca.load_sgmv_tables([d for d, _, _ in dirs], "blocks.1", device="cpu",
                                                      dtype=torch.float64)
    assert rk.tolist() == [1, 0, 2] and offsets.tolist() == [0, 1, 1]
    x = torch.randn(6, 7, dtype=torch.float64)
    ids = [0, 0, 1, 2, 2, 0]
    for t, ad in enumerate(ids):
        o, r = int(offsets[ad]), int(rk[ad])
        got = (x[t] @ a_flat[o:o + r].T) @ b_flat[o:o + r] if r else torch.zeros(5, dtype=torch.float64)
        _, tensors, config = dirs[ad]
        a = tensors["base_model.model.blocks.1.lora_A.weight"].double()
        b = tensors["base_model.model.blocks.1.lora_B.weight"].double()
        want = ca.lora_scale(config, "blocks.1") * ((x[t] @ a.T) @ b.T)
        torch.testing.assert_close(got, want, rtol=1e-9, atol=1e-9)


@pytest.mark.gpu
def test_compact_tables_drive_segmented_branch(tmp_path):
    """On disk to device: three adapters of one module (ranks 4, 0 after
    compaction, 16), their tables loaded by load_sgmv_tables, the segmented
    branch on the GPU against each token's own adapter in fp64."""
    import numpy as np
    from safetensors.torch import save_file

    from probe_b200 import segmented_branch
    from tests.helpers import assert_parity, np64

    k, n, t = 256, 192, 150
    dirs, per = [], []
    for j, rank in enumerate([4, 0, 16]):
        g = torch.Generator().manual_seed(40 + j)
        a, b = torch.zeros(16, k), torch.zeros(n, 16)
        a[:rank] = torch.randn(rank, k, generator=g) / k ** 0.5
        b[:, :rank] = torch.randn(n, rank, generator=g) / 4
        tensors = {"base_model.model.layer.lora_A.weight": a, "base_model.model.layer.lora_B.weight": b}
        config = dict(peft_type="LORA", r=16, lora_alpha=8 * (j + 1), target_modules=["layer"], bias="none")
        src = tmp_path / f"src{j}"
        src.mkdir()
        save_file(tensors, src / "adapter_model.safetensors")
        (src / "adapter_config.json").write_text(json.dumps(config))
        ca.export_compact(src, tmp_path / f"c{j}", [rank])
        dirs.append(tmp_path / f"c{j}")
        per.append((a.double(), b.double(), ca.lora_scale(config, "layer")))
    a_flat, b_flat, offsets, ranks = ca.load_sgmv_tables(dirs, "layer", device="cuda", dtype=torch.bfloat16)
    assert ranks.tolist() == [4, 0, 16]
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(t, k, generator=gen).to("cuda", torch.bfloat16)
    y = torch.randn(t, n, generator=gen).to("cuda", torch.bfloat16)
    seg_start = torch.tensor([0, 40, 41, 100, 150], device="cuda")
    seg_ad = torch.tensor([2, 0, 1, 2], device="cuda")
    out = segmented_branch.segmented_branch_varlen(x, y, a_flat, b_flat, offsets, ranks, seg_start, seg_ad, 16)
    want = np64(y).copy()
    xs = np64(x)
    for s in range(4):
        a, b, scale = per[int(seg_ad[s])]
        lo, hi = int(seg_start[s]), int(seg_start[s + 1])
        want[lo:hi] += scale * (xs[lo:hi] @ a.numpy().T) @ b.numpy().T
    assert_parity(out, np.asarray(want))
