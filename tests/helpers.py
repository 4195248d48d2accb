"""Shared helpers of the parity tests (tolerances are the bf16 bar of the spec)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import lora_oracle as orc

# bf16 bar: max-abs error <= 2e-2 and relative Frobenius error <= 5e-3 against
# the float64 reference.  The output is itself bf16, so even a correctly
# rounded result differs from the reference by up to half an ulp (0.03 at
# |y| >= 8, more than 2e-2); the max-abs bound therefore applies to the error
# beyond that half ulp: max(|out - ref| - ulp(ref)/2) <= 2e-2.  The raw max-abs
# is reported alongside.  fp16 has 3 more mantissa bits; the same bounds hold.
MAX_ABS = 2e-2
REL_FRO = 5e-3


def np64(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


def dtype_tag(dtype) -> str:
    return "bf16" if dtype == torch.bfloat16 else "f16"


def assert_parity(got: torch.Tensor, want: np.ndarray, dtype=torch.bfloat16, max_abs=MAX_ABS, rel_fro=REL_FRO,
                  scale_abs: float | None = None):
    g = np64(got)
    want = np.asarray(want, dtype=np.float64)
    assert g.shape == want.shape, (g.shape, want.shape)
    assert np.isfinite(g).all(), "non-finite output"
    err_abs = orc.excess_abs_error(g, want, dtype_tag(dtype))
    raw, fro = orc.parity(g, want)
    bound = max_abs if scale_abs is None else max_abs * scale_abs
    assert err_abs <= bound, f"max-abs beyond half-ulp {err_abs:.3e} > {bound:.1e} (raw {raw:.3e})"
    assert fro <= rel_fro, f"rel-Frobenius {fro:.3e} > {rel_fro:.1e}"
    return err_abs, fro


def randn(shape, std=1.0, dtype=torch.bfloat16, seed=0, device="cuda"):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(dtype).to(device)
