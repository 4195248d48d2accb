"""CUDA-graph greedy decoding for a fixed Transformers model and adapter.

Drop-in for ``loraforge_kernels.static_decode`` (static_decode.py:1-120): the
prompt is prefilled eagerly into a Transformers ``StaticCache``; every decode
step after it -- the model forward at one token per sequence, the argmax, the
position and the additive attention mask -- is one captured CUDA graph that
is replayed.  The LoRA linears of this package run inside it (their plans are
resolved by the warm-up steps before capture; the small-M decode kernels need
no workspace).

Fixed-length greedy only: no EOS stop, sampling, beams, padding or adapter
switching.  Build a new runner after changing weights, adapters, batch size or
length.  The model must support ``StaticCache`` and a 4-D additive mask.
"""

from __future__ import annotations

import torch


class StaticDecodeRunner:
    """Greedy generation of exactly ``new_tokens`` tokens for a fixed batch
    and prompt length (static_decode.py:11-120).  Returned token tensors belong
    to the caller; the graph's buffers stay inside the runner."""

    @torch.inference_mode()
    def __init__(self, model, example_ids: torch.Tensor, new_tokens: int):
        from transformers import StaticCache

        if example_ids.ndim != 2 or not example_ids.is_cuda or example_ids.dtype != torch.long or new_tokens < 1:
            raise ValueError("Expected CUDA [batch, prefix] IDs and new_tokens >= 1")
        if model.training:
            raise ValueError("Call model.eval() before capturing inference")
        self.model = model
        self.batch, self.prefix = example_ids.shape
        if self.prefix == 0:
            raise ValueError("A nonempty unpadded prefix is required")
        self.new_tokens = new_tokens
        self.capacity = self.prefix + new_tokens + 4
        dev = example_ids.device
        self.cache = StaticCache(config=model.config, max_cache_len=self.capacity)
        # graph inputs / outputs: fixed addresses, updated in place
        self.token = torch.empty((self.batch, 1), device=dev, dtype=torch.long)
        self.position = torch.full_like(self.token, self.prefix)
        self.columns = torch.arange(self.capacity, device=dev)
        self.mask = torch.empty((self.batch, 1, 1, self.capacity), device=dev, dtype=model.dtype)
        self.prefix_mask = torch.ones_like(example_ids)
        self._prefill(example_ids)
        # Plans, lazily built tables and cache allocations must exist before
        # capture: two eager steps on throw-away cache state.
        for _ in range(2):
            self._step()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        self.graph_logits = self.step_logits
        # The graph holds device addresses, not Python references: keep every
        # parameter and buffer it read alive as long as the runner.
        self._captured = tuple(model.parameters()) + tuple(model.buffers())

    def _update_mask(self):
        visible = self.columns[None, :] <= self.position  # [batch, capacity]
        self.mask.copy_(torch.where(visible, 0.0, torch.finfo(self.mask.dtype).min)[:, None, None, :])

    def _prefill(self, input_ids):
        self.cache.reset()
        out = self.model(input_ids=input_ids, attention_mask=self.prefix_mask, past_key_values=self.cache,
                         use_cache=True, logits_to_keep=1)
        self.token.copy_(out.logits[:, -1].argmax(-1, keepdim=True))
        self.position.fill_(self.prefix)
        self._update_mask()

    def _step(self):
        out = self.model(input_ids=self.token, position_ids=self.position, attention_mask=self.mask,
                         past_key_values=self.cache, use_cache=True, logits_to_keep=1)
        self.step_logits = out.logits[:, -1]
        self.token.copy_(self.step_logits.argmax(-1, keepdim=True))
        self.position.add_(1)
        self._update_mask()

    @torch.inference_mode()
    def validate(self, input_ids, tolerance: float = 0.01) -> float:
        """Largest relative L2 difference between replayed and eager logits on
        the same teacher-forced tokens (argmax ties may flip under rounding, so
        the trajectories are matched rather than compared).  Raises above
        ``tolerance``."""
        self._prefill(input_ids)
        tokens, logits = [], []
        for _ in range(1, self.new_tokens):
            tokens.append(self.token.clone())
            self._step()
            logits.append(self.step_logits.clone())
        self._prefill(input_ids)
        worst = 0.0
        for tok, ref in zip(tokens, logits):
            self.token.copy_(tok)
            self.graph.replay()
            err = float(torch.linalg.vector_norm(self.graph_logits.float() - ref.float())
                        / torch.linalg.vector_norm(ref.float()).clamp_min(1e-8))
            worst = max(worst, err)
        if worst > tolerance:
            raise AssertionError(f"Captured decode logit relative L2 error {worst:.4g} > {tolerance}")
        return worst

    @torch.inference_mode()
    def __call__(self, input_ids, *, replay: bool = True) -> torch.Tensor:
        if (input_ids.shape != (self.batch, self.prefix) or input_ids.device != self.token.device
                or input_ids.dtype != torch.long):
            raise ValueError("Input must match the captured batch, prefix, device and int64 dtype")
        self._prefill(input_ids)
        result = torch.empty((self.batch, self.prefix + self.new_tokens), device=input_ids.device, dtype=torch.long)
        result[:, : self.prefix].copy_(input_ids)
        result[:, self.prefix: self.prefix + 1].copy_(self.token)
        for step in range(1, self.new_tokens):
            if replay:
                self.graph.replay()
            else:
                self._step()
            result[:, self.prefix + step: self.prefix + step + 1].copy_(self.token)
        return result
