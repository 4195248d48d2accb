"""The whole-output parity checker itself (CPU): a correctly rounded output
passes, outputs with a planted mistake fail."""

import numpy as np
import torch

from oracle import checks
from oracle import lora_oracle as orc


def _case(m=600, k=64, n=96, r=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    x = torch.randn(m, k, generator=g).to(bf)
    w = (torch.randn(n, k, generator=g) / 8).to(bf)
    a = (torch.randn(r, k, generator=g) / 8).to(bf)
    b = (torch.randn(n, r, generator=g) / 3).to(bf)
    f = lambda t: t.double().numpy()  # noqa: E731
    ref = orc.naive_linear(f(x), f(w), None, f(a), f(b), 1.5)
    out = torch.from_numpy(ref).to(bf)  # correctly rounded product
    return out, x, w, a, b


def test_correct_output_passes():
    out, x, w, a, b = _case()
    rep = checks.linear_report(out, x, w, None, a, b, 1.5, seed=1)
    assert rep["ok"], rep
    assert rep["row_sum_dev"] < 1 and rep["sketch_dev"] < 1


def test_missing_tile_fails():
    out, x, w, a, b = _case()
    bad = out.clone()
    bad[300:316, 32:48] = 0  # a 16 x 16 block never written (no sampled row needs to hit it)
    rep = checks.linear_report(bad, x, w, None, a, b, 1.5, seed=1)
    assert not rep["ok"] and (rep["row_sum_dev"] > 1 or rep["sketch_dev"] > 1)


def test_wrong_scale_fails():
    out, x, w, a, b = _case()
    rep = checks.linear_report(out, x, w, None, a, b, 1.4, seed=1)
    assert not rep["ok"]


def test_small_output_checked_in_full():
    out, x, w, a, b = _case(m=40)
    bad = out.clone()
    bad[17, 5] += 0.5
    assert checks.linear_report(out, x, w, None, a, b, 1.5, full_checks=False)["ok"]
    rep = checks.linear_report(bad, x, w, None, a, b, 1.5, full_checks=False)
    assert rep["rows_checked"] == 40 and not rep["ok"]


def test_branch_report_detects_wrong_adapter():
    g = torch.Generator().manual_seed(3)
    bf = torch.bfloat16
    t, k, n = 200, 32, 48
    ranks = np.array([4, 8, 0, 16])
    offsets = np.concatenate([[0], np.cumsum(ranks)[:-1]])
    x = torch.randn(t, k, generator=g).to(bf)
    y = torch.randn(t, n, generator=g).to(bf)
    a_flat = (torch.randn(int(ranks.sum()), k, generator=g) / 4).to(bf)
    b_flat = (torch.randn(int(ranks.sum()), n, generator=g) / 3).to(bf)
    ids = np.repeat([0, 1, 2, 3, 1], [30, 50, 20, 60, 40])
    f = lambda v: v.double().numpy()  # noqa: E731
    ref = orc.ragged_branch(f(x), f(y), f(a_flat), f(b_flat), offsets, ranks, ids)
    out = torch.from_numpy(ref).to(bf)
    assert checks.branch_report(out, x, y, a_flat, b_flat, offsets, ranks, ids)["ok"]
    wrong = ids.copy()
    wrong[wrong == 3] = 0  # the product routed segment 4 to adapter 0
    out_wrong = torch.from_numpy(orc.ragged_branch(f(x), f(y), f(a_flat), f(b_flat), offsets, ranks, wrong)).to(bf)
    assert not checks.branch_report(out_wrong, x, y, a_flat, b_flat, offsets, ranks, ids)["ok"]
