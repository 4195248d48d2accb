"""The CPU oracle against the reference's own outputs (golden vectors).

These tests pin the oracle: every golden file was produced by running the
reference implementation (see tests/golden/make_golden.py).  CPU only.
"""

import numpy as np
import pytest
import torch

from oracle import lora_oracle as orc
from probe_b200 import fused_linear, multilora, splitk_lora, splitk_shrink, workloads
from tests.golden_io import from_bits, ints, load

# fp64 oracle vs the reference's fp32 CPU arithmetic
REL = 2e-6


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_known_answer_rank_tables():
    """The reference's own known-answer tables (test_fused_linear.py:171-185)."""
    for r, want in {1: 16, 8: 16, 16: 16, 17: 32, 24: 32, 40: 64, 64: 64, 65: 128}.items():
        assert orc.pad_rank(r) == want
        assert fused_linear.pad_rank(r) == want
    for r, want in {1: 16, 16: 16, 17: 32, 40: 48, 64: 64}.items():
        assert orc.packed_rank(r) == want
        assert fused_linear.packed_rank(r) == want


def test_integer_helpers_match_reference():
    g = ints()
    for r, v in g["pad_rank"].items():
        assert orc.pad_rank(int(r)) == v and fused_linear.pad_rank(int(r)) == v
    for r, v in g["packed_rank"].items():
        assert orc.packed_rank(int(r)) == v and fused_linear.packed_rank(int(r)) == v
    for r, v in g["align_to_deploy_rank"].items():
        assert orc.align_to_deploy_rank(int(r)) == v and splitk_lora.align_to_deploy_rank(int(r)) == v
    for r, v in g["splitk_rank_tile"].items():
        assert orc.rank_tile(int(r)) == v and splitk_shrink.rank_tile(int(r)) == v
    for r, v in g["multilora_rank_tile"].items():
        assert multilora.rank_tile(int(r)) == v
    for n, v in g["auto_split_k"].items():
        assert orc.auto_split_k(int(n)) == v and multilora.auto_split_k(int(n)) == v
    assert list(splitk_lora.DEPLOY_RANK_BUCKETS) == g["deploy_rank_buckets"]
    c = g["constants"]
    assert fused_linear.MIN_GEMM_ROWS == c["MIN_GEMM_ROWS"]
    assert fused_linear.FUSED_MAX_RANK == c["FUSED_MAX_RANK"]
    assert fused_linear.MIN_RANK_TILE == c["MIN_RANK_TILE"]
    assert fused_linear.PACK_ALIGN == c["PACK_ALIGN"]


def test_oracle_linear_matches_reference_cpu_path():
    d = load("linear_cases.npz")
    for i in range(int(d["n_cases"])):
        bias = from_bits(d[f"c{i}_bias"]) if d[f"c{i}_bias"].size else None
        got = orc.naive_linear(from_bits(d[f"c{i}_x"]), from_bits(d[f"c{i}_w"]), bias, from_bits(d[f"c{i}_a"]),
                               from_bits(d[f"c{i}_b"]), float(d[f"c{i}_scale"]))
        assert rel(got, d[f"c{i}_out"]) < REL, i
    x = from_bits(d["nd_x"])
    got = orc.naive_linear(x.reshape(-1, x.shape[-1]), from_bits(d["nd_w"]), None, from_bits(d["nd_a"]),
                           from_bits(d["nd_b"]), 0.8)
    assert rel(got, d["nd_out"].reshape(got.shape)) < REL


def test_workload_c1_generator_and_oracle_match_reference():
    d = load("c1_checksums.npz")
    p = workloads.c1(device="cpu", dtype=torch.float32)
    for name in ("x", "w", "a", "b"):
        assert np.array_equal(getattr(p, name).flatten()[:16].numpy(), d[f"{name}_head"])
    rows = d["rows"]
    xr = p.x.numpy()[rows]
    got = orc.naive_linear(xr, p.w.numpy(), None, p.a.numpy(), p.b.numpy(), p.scale)
    assert rel(got, d["f32_rows"]) < REL
    xb = orc.round_bf16(p.x.numpy())
    got_b = orc.naive_linear(xb[rows], orc.round_bf16(p.w.numpy()), None, orc.round_bf16(p.a.numpy()),
                             orc.round_bf16(p.b.numpy()), p.scale)
    assert rel(got_b, d["bf16in_rows"]) < REL


def test_oracle_branches_match_reference_triton_kernels():
    d = load("branch_cases.npz")
    a, b = from_bits(d["a_flat"]), from_bits(d["b_flat"])
    got = orc.ragged_branch(from_bits(d["x"]), from_bits(d["y"]), a, b, d["offsets"], d["ranks"], d["ids"])
    assert rel(got, d["ragged_out"]) < 5e-6
    assert rel(got, d["ragged_noskip_out"]) < 5e-6
    got = orc.segmented_branch(from_bits(d["xs"]), from_bits(d["ys"]), a, b, d["offsets"], d["ranks"], d["req"], 12)
    assert rel(got, d["seg_out"]) < 5e-6
    with pytest.raises(ValueError):
        orc.segmented_branch(from_bits(d["xs"]), from_bits(d["ys"]), a, b, d["offsets"], d["ranks"], d["req"], 11)


def test_oracle_stacking_matches_reference_attach():
    d = load("stack_case.npz")
    adapters = [(from_bits(d[f"down{i}"]), from_bits(d[f"up{i}"]), float(d[f"alpha{i}"])) for i in range(3)]
    a_st, b_st, scale = orc.stack_adapters(adapters)
    assert scale == float(d["scale"])
    assert int(d["rank"]) == a_st.shape[0] == 28
    # the reference folds alpha in fp32 then casts back to the layer dtype (fp32 here)
    assert rel(a_st, d["lora_a"]) < 1e-6
    assert np.array_equal(b_st.astype(np.float32), d["lora_b"])
    got = orc.naive_linear(from_bits(d["x"]), from_bits(d["w"]), from_bits(d["bias"]), a_st, b_st, scale)
    assert rel(got, d["out"]) < REL


def test_tile_schedule_oracle():
    starts, adapters = orc.tile_schedule(ids=[0] * 70 + [1] * 3 + [0] * 2, tile=64)
    assert starts == [0, 64, 70, 73, 75]
    assert adapters == [0, 0, 1, 0]
    starts, adapters = orc.tile_schedule(seg_start=[0, 5, 5, 9], seg_adapter=[2, 7, 2], n_adapters=4)
    assert starts == [0, 9] and adapters == [2]
    starts, adapters = orc.tile_schedule(ids=[5, 5, 1], n_adapters=4)
    assert adapters == [-1, 1]


def test_bf16_rounding_helper():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38], np.float32)
    want = torch.tensor(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(orc.round_bf16(x), want)
    r = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 10
    assert np.array_equal(orc.round_bf16(r), torch.tensor(r).to(torch.bfloat16).float().numpy())
