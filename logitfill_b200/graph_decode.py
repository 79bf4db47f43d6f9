"""CUDA-graph decode loop for a model driven by ``DeepSeekQwenKVAdapter``.

The reference samples one token at a time by calling the model eagerly with
its cache handle (``src/logitfill/benchmarks/generate.py:28-57``): every step
pays the Python dispatch of every layer and a host-side commit.  Here the
prompt is prefilled eagerly (dense attention, K1 for the completed pages) and
one decode step -- the whole model forward for one token, with the packed
attention (K2 + K3) and the device-side commit of the token (append to the
residual page, K1 when the page fills, lengths advanced on the device,
``lf_commit_token``) -- is captured once in a CUDA graph and replayed for every
following token.  Positions are fed through static device tensors; the host
lengths are advanced after each replay by the same rule the device applies.

The packed history is allocated for ``max_tokens`` up front (a capture cannot
survive a reallocation); the split plan of the captured step is the one chosen
at capture time (correct for any history length up to the capacity).
"""
from __future__ import annotations

import torch

from logitfill_b200.adapter import DeepSeekQwenKVAdapter


class GraphDecoder:
    """Prefill eagerly, then decode one token per :meth:`step` by replaying a
    captured graph.  Batch 1, like the reference's manager."""

    def __init__(self, model, adapter: DeepSeekQwenKVAdapter, max_tokens: int):
        if not adapter._attached:
            raise RuntimeError("attach the adapter first")
        self.model, self.adapter = model, adapter
        self.max_tokens = int(max_tokens)
        self.device = next(model.parameters()).device
        self.manager = adapter.packed_manager()
        self.cache = adapter.make_cache()
        self.graph = None
        self.ids = torch.zeros(1, 1, dtype=torch.long, device=self.device)
        self.pos = torch.zeros(1, 1, dtype=torch.long, device=self.device)
        self.cpos = torch.zeros(1, dtype=torch.long, device=self.device)
        self.logits = None

    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Dense prefill of ``input_ids`` ``[1, T]`` (a new sequence); returns the
        last position's logits ``[1, vocab]``."""
        if input_ids.shape[0] != 1 or input_ids.shape[1] >= self.max_tokens:
            raise ValueError("one sequence shorter than max_tokens")
        self.cache.reset()
        self.manager.cache.grow_to(self.max_tokens)
        out = self.model(input_ids=input_ids, use_cache=True, past_key_values=self.cache)
        return out.logits[:, -1]

    def _forward(self) -> torch.Tensor:
        self.adapter.graph_step = True
        try:
            out = self.model(input_ids=self.ids, position_ids=self.pos, cache_position=self.cpos,
                             past_key_values=self.cache, use_cache=True)
        finally:
            self.adapter.graph_step = False
        return out.logits[:, -1]

    def _set_inputs(self, token: torch.Tensor) -> None:
        n = self.manager.seq_len
        if n + 1 > self.max_tokens:
            raise RuntimeError(f"the sequence reached max_tokens={self.max_tokens}")
        self.ids.copy_(token.reshape(1, 1))
        self.pos.fill_(n)
        self.cpos.fill_(n)

    @torch.inference_mode()
    def step(self, token: torch.Tensor) -> torch.Tensor:
        """Decode ``token`` (``[1, 1]`` or a scalar tensor on the device):
        returns its logits ``[1, vocab]`` (a static buffer, overwritten by the
        next step)."""
        if self.manager.seq_len == 0:
            raise RuntimeError("prefill first")
        self._set_inputs(token)
        if self.graph is None:
            # First step eagerly (allocates the workspaces, loads the kernels),
            # then capture the same step for the following tokens.
            logits = self._forward().clone()
            self.manager.advance_host()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.logits = self._forward()
            return logits
        self.graph.replay()
        self.manager.advance_host()
        return self.logits

    def release(self) -> None:
        """Drop the captured graph (its memory pool goes with it)."""
        self.graph = None
        self.logits = None
