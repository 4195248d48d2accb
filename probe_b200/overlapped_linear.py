"""Base GEMM and LoRA shrink on two streams (drop-in for overlapped_linear.py:10-61).

The memory-bound shrink ``x @ A.T`` runs on a side stream while the tensor-core
base GEMM runs on the caller's stream; the join is the expand-add epilogue,
which reads the base output once and writes the result once.
"""

from __future__ import annotations

import torch

from . import kernels
from .fused_linear import _base_linear


class DualStreamOverlappedLinear(torch.nn.Module):
    """Linear with a LoRA branch overlapped on a second CUDA stream."""

    def __init__(self, in_features: int, out_features: int, rank: int, bias: bool = False,
                 dtype=torch.float16, device="cuda"):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.rank = rank
        self.weight = torch.nn.Parameter(
            torch.randn(out_features, in_features, device=device, dtype=dtype) / in_features**0.5)
        self.lora_A = torch.nn.Parameter(torch.randn(rank, in_features, device=device, dtype=dtype) / in_features**0.5)
        self.lora_B = torch.nn.Parameter(torch.randn(out_features, rank, device=device, dtype=dtype) / max(rank, 1)**0.5)
        self.bias = torch.nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype)) if bias else None
        self.stream_lora = torch.cuda.Stream(device=device)
        self.event_input_ready = torch.cuda.Event()
        self.event_lora_done = torch.cuda.Event()

    @torch.no_grad()
    def forward(self, x: torch.Tensor, scale: float = 1.0, use_splitk: bool = False) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        current = torch.cuda.current_stream()
        self.event_input_ready.record(current)
        with torch.cuda.stream(self.stream_lora):
            self.stream_lora.wait_event(self.event_input_ready)
            z = kernels.shrink(x2, self.lora_A, 1.0, z_dtype=torch.float32)
            self.event_lora_done.record(self.stream_lora)
        y = _base_linear(x2, self.weight, self.bias)
        current.wait_event(self.event_lora_done)
        z.record_stream(current)
        out = kernels.expand_add(y, z, self.lora_B, scale)
        return out.reshape(*shape[:-1], self.out_features)
