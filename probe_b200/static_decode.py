"""Greedy decoding replayed from one CUDA graph per step.

Drop-in for ``loraforge_kernels.static_decode`` (static_decode.py:1-120).  The
prompt is prefilled eagerly into a Transformers ``StaticCache``; the decode
step -- model forward at one token per sequence, argmax, the new token's
write into the output row, position and additive-mask update -- is captured
once and replayed for every further token, so a step costs one graph launch
instead of hundreds of kernel launches.  This package's LoRA linears run
inside the graph (their plans and workspaces are set up by the warm-up steps,
which run on the capture stream before capture).

Design: every tensor the step touches lives in the runner at a fixed address.
``history`` holds the whole output sequence; the captured step scatters its
new token to column ``position + 1``, so a generation is a prefill, replays
and one copy of ``history`` -- no per-step host work.

Limits: fixed batch, prompt length and token count; greedy only (no EOS stop,
sampling, beams, padding or adapter switching).  Build a new runner after
changing weights, adapters, batch size or lengths.  The model must accept a
``StaticCache`` and a 4-D additive attention mask.
"""

from __future__ import annotations

import torch

_WARMUP_STEPS = 2      # eager steps on the capture stream before capture
_SPARE_POSITIONS = 4   # cache slots beyond the generated tokens (warm-up and capture steps write there)


def _check_prompt(ids: torch.Tensor, new_tokens: int) -> None:
    shaped = ids.ndim == 2 and ids.is_cuda and ids.dtype == torch.long
    if not shaped or new_tokens < 1:
        raise ValueError("Expected CUDA [batch, prefix] IDs and new_tokens >= 1")
    if ids.shape[1] == 0:
        raise ValueError("A nonempty unpadded prefix is required")


class StaticDecodeRunner:
    """Generate exactly ``new_tokens`` greedy tokens for a fixed batch and
    prompt length (static_decode.py:11-120).

    ``runner(ids)`` returns a fresh ``[batch, prefix + new_tokens]`` int64
    tensor owned by the caller; ``runner(ids, replay=False)`` runs the same
    steps eagerly; ``validate(ids)`` compares replayed and eager logits.
    """

    @torch.inference_mode()
    def __init__(self, model, example_ids: torch.Tensor, new_tokens: int):
        from transformers import StaticCache

        _check_prompt(example_ids, new_tokens)
        if model.training:
            raise ValueError("Call model.eval() before capturing inference")
        self.model = model
        self.batch, self.prefix = (int(v) for v in example_ids.shape)
        self.new_tokens = int(new_tokens)
        self.capacity = self.prefix + self.new_tokens + _SPARE_POSITIONS
        device = example_ids.device
        self.cache = StaticCache(config=model.config, max_cache_len=self.capacity)
        # fixed-address state read and written by the captured step
        self.history = torch.zeros((self.batch, self.capacity), device=device, dtype=torch.long)
        self.token = torch.zeros((self.batch, 1), device=device, dtype=torch.long)
        self.position = torch.zeros((self.batch, 1), device=device, dtype=torch.long)
        self._columns = torch.arange(self.capacity, device=device)
        self.mask = torch.zeros((self.batch, 1, 1, self.capacity), device=device, dtype=model.dtype)
        self._prompt_mask = torch.ones((self.batch, self.prefix), device=device, dtype=torch.long)
        self._mask_fill = torch.finfo(model.dtype).min
        self.step_logits = None

        self._start(example_ids)
        capture_stream = torch.cuda.Stream(device)
        capture_stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(capture_stream):
            for _ in range(_WARMUP_STEPS):  # plans, workspaces and cache buffers appear here, not in capture
                self._advance()
        torch.cuda.current_stream(device).wait_stream(capture_stream)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=capture_stream):
            self._advance()
        self.graph_logits = self.step_logits
        # The graph refers to device addresses only; hold the tensors behind them.
        self._keepalive = (tuple(model.parameters()), tuple(model.buffers()))

    # -------------------------------------------------------------- steps
    def _refresh_mask(self) -> None:
        hidden = self._columns[None, :] > self.position  # [batch, capacity]: columns not yet visible
        self.mask.zero_()
        self.mask.masked_fill_(hidden[:, None, None, :], self._mask_fill)

    def _start(self, ids: torch.Tensor) -> None:
        """Prefill the prompt; the first new token goes to column ``prefix``."""
        self.cache.reset()
        logits = self.model(input_ids=ids, attention_mask=self._prompt_mask, past_key_values=self.cache,
                            use_cache=True, logits_to_keep=1).logits[:, -1]
        self.token.copy_(torch.argmax(logits, dim=-1, keepdim=True))
        self.history[:, : self.prefix].copy_(ids)
        self.history[:, self.prefix: self.prefix + 1].copy_(self.token)
        self.position.fill_(self.prefix)
        self._refresh_mask()

    def _advance(self) -> None:
        """Feed ``token`` at ``position``; write the next token to column position + 1."""
        logits = self.model(input_ids=self.token, position_ids=self.position, attention_mask=self.mask,
                            past_key_values=self.cache, use_cache=True, logits_to_keep=1).logits[:, -1]
        self.step_logits = logits
        self.token.copy_(torch.argmax(logits, dim=-1, keepdim=True))
        self.history.scatter_(1, self.position + 1, self.token)
        self.position.add_(1)
        self._refresh_mask()

    # ------------------------------------------------------------ public
    def _check_request(self, ids: torch.Tensor) -> None:
        if tuple(ids.shape) != (self.batch, self.prefix) or ids.device != self.token.device \
                or ids.dtype != torch.long:
            raise ValueError("Input must match the captured batch, prefix, device and int64 dtype")

    @torch.inference_mode()
    def __call__(self, input_ids: torch.Tensor, *, replay: bool = True) -> torch.Tensor:
        self._check_request(input_ids)
        self._start(input_ids)
        for _ in range(self.new_tokens - 1):
            if replay:
                self.graph.replay()
            else:
                self._advance()
        return self.history[:, : self.prefix + self.new_tokens].clone()

    @torch.inference_mode()
    def validate(self, input_ids: torch.Tensor, tolerance: float = 0.01) -> float:
        """Worst relative L2 distance between replayed and eager step logits.

        Both runs are fed the same (eager) tokens: near an argmax tie bf16
        rounding could send free-running trajectories apart, which would say
        nothing about the graph.  Raises ``AssertionError`` above ``tolerance``.
        """
        self._check_request(input_ids)
        self._start(input_ids)
        fed, eager = [], []
        for _ in range(self.new_tokens - 1):
            fed.append(self.token.clone())
            self._advance()
            eager.append(self.step_logits.float().clone())
        self._start(input_ids)
        worst = 0.0
        for token, ref in zip(fed, eager):
            self.token.copy_(token)
            self.graph.replay()
            diff = torch.linalg.vector_norm(self.graph_logits.float() - ref)
            worst = max(worst, float(diff / torch.linalg.vector_norm(ref).clamp_min(1e-8)))
        if worst > tolerance:
            raise AssertionError(f"Captured decode logit relative L2 error {worst:.4g} > {tolerance}")
        return worst
