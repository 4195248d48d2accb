"""Single-launch-class base + LoRA linear for small decode batches.

Drop-in for ``loraforge_kernels.decode_linear`` (decode_linear.py:1-100).  The
reference computes base GEMV + shrink + expand + bias in one Triton launch per
output tile, re-deriving x.A^T in every tile.  Here the shrink runs once (split-K
kernel, z rounded to the input dtype exactly where the reference rounds it,
decode_linear.py:42-44) and the decode kernel streams W once with the expand as
a K tail; programmatic dependent launch overlaps the two.
"""

from __future__ import annotations

import torch

from . import kernels
from .fused_linear import _base_linear


def build_decode_linear(weight, bias, a, b, scale=1.0, *, block_n=16, block_k=256):
    """Bind the invariant operands once (decode_linear.py:53-78).

    ``block_n`` / ``block_k`` are accepted for compatibility; the B200 kernel
    picks its own split of K and N.
    """
    r, k = a.shape
    if r == 0 or scale == 0:
        return lambda x: _base_linear(x, weight, bias)
    scale = float(scale)
    weight = weight.contiguous()
    a = a.contiguous()
    b = b.contiguous()

    def run(x):
        if x.shape[0] == 0:
            return torch.empty((0, weight.shape[0]), device=x.device, dtype=x.dtype)
        outs = []
        step = 256 if x.shape[1] % 8 == 0 else 64
        for i in range(0, x.shape[0], step):
            xs = x[i: i + step]
            z = kernels.shrink(xs, a, 1.0, z_dtype=torch.float32)
            outs.append(kernels.decode_linear(xs, weight, z, b, bias, scale))
        return outs[0] if len(outs) == 1 else torch.cat(outs)

    return run


def decode_lora_linear(x, weight, bias, a, b, scale=1.0, *, block_n=16, block_k=256):
    """Evaluate the complete Linear without packing W (decode_linear.py:81-100).

    Raises ``ValueError`` for incompatible shapes, a rank outside [0, 64], or
    tensors that are not CUDA fp16/bf16 of one dtype and device.
    """
    r, k = a.shape
    n = weight.shape[0]
    if (x.ndim != 2 or weight.shape[1] != k or x.shape[1] != k
            or b.shape != (n, r) or not 0 <= r <= 64):
        raise ValueError("Incompatible decode Linear shapes or rank outside [0, 64]")
    tensors = (weight, a, b) + (() if bias is None else (bias,))
    if (not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16)
            or any(t.device != x.device or t.dtype != x.dtype for t in tensors)):
        raise ValueError("decode Linear requires CUDA fp16/bf16 tensors of one dtype/device")
    if r == 0 or scale == 0:
        return _base_linear(x.contiguous() if not x.is_contiguous() else x, weight, bias)
    if bias is not None and bias.shape != (n,):
        raise ValueError("bias must be a vector of out_features elements")
    return build_decode_linear(weight, bias, a, b, scale, block_n=block_n, block_k=block_k)(x)
