"""Greedy decoding with a static KV cache, one token per step, each step replayed from a
CUDA graph.

The reference measures its patch end to end with HuggingFace ``generate()`` (eager, a
dynamic KV cache; ``benchmarks/e2e_decode.py:60-148``: prompt 128, 256 new tokens, batch
1 and 16, tokens per second over the decode phase).  On B200 a decode step of a Llama
layer stack is a few hundred microseconds of GPU work and about as much Python; launched
eagerly, the host is the bottleneck and the fused kernels cannot show.  This driver keeps
the methodology (prefill of the prompt, then greedy decode, tokens per second over the
decode steps) and removes the host from the loop: the prompt is prefilled eagerly into a
``transformers.StaticCache``, one decode step (embedding, every decoder layer with its KV
cache update, final norm, LM head, argmax, position advance) is captured in a CUDA graph,
and each further token is one replay.  The patched and unpatched models run the same
driver, so their tokens can be compared step by step.
"""
from __future__ import annotations

import torch
from transformers import StaticCache


class GraphedGreedyDecoder:
    """Greedy decoder for a ``LlamaForCausalLM`` (patched or not) on one CUDA device.

    ``generate(prompt, n_new)`` returns the ``n_new`` greedy tokens after ``prompt``
    (``(batch, prompt_len)`` int64 on the model's device) as ``(batch, n_new)``.  The first
    new token comes from the eager prefill; every later one from a replay of the captured
    step.  ``decode_seconds`` holds the CUDA-event time of those replays."""

    def __init__(self, model, batch: int, max_len: int):
        self.model = model
        self.batch = batch
        self.max_len = max_len
        self.device = next(model.parameters()).device
        self.decode_seconds = 0.0
        self._graph = None

    def _new_cache(self) -> StaticCache:
        return StaticCache(config=self.model.config, max_cache_len=self.max_len)

    @torch.no_grad()
    def _step(self):
        """One decode step on the static buffers: logits of the last token, argmax into
        ``self._tok``, position advanced in place."""
        out = self.model(input_ids=self._tok, position_ids=self._pos, past_key_values=self._cache, use_cache=True)
        self._tok.copy_(out.logits[:, -1, :].argmax(dim=-1, keepdim=True))
        self._pos.add_(1)

    @torch.no_grad()
    def forced_logits(self, prompt: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
        """Teacher forcing, eagerly: the fp32 logits that predict ``tokens[:, t]`` for every t
        ((batch, n, vocab)), when ``tokens[:, :t]`` follow ``prompt``.  Comparing two models on
        the same token sequence separates numerical differences from the divergence of their
        own greedy paths."""
        B, P = prompt.shape
        n = tokens.shape[1]
        cache = self._new_cache()
        pos = torch.arange(P, device=self.device)[None].expand(B, P)
        out = self.model(input_ids=prompt, position_ids=pos, past_key_values=cache, use_cache=True)
        logits = [out.logits[:, -1, :].float()]
        for t in range(n - 1):
            p = torch.full((B, 1), P + t, dtype=torch.long, device=self.device)
            out = self.model(input_ids=tokens[:, t:t + 1], position_ids=p, past_key_values=cache, use_cache=True)
            logits.append(out.logits[:, -1, :].float())
        return torch.stack(logits, dim=1)

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, n_new: int) -> torch.Tensor:
        B, P = prompt.shape
        if B != self.batch or P + n_new > self.max_len:
            raise ValueError(f"prompt {tuple(prompt.shape)} + {n_new} tokens does not fit batch {self.batch}, "
                             f"max_len {self.max_len}")
        self._cache = self._new_cache()
        pos = torch.arange(P, device=self.device)[None].expand(B, P)
        out = self.model(input_ids=prompt, position_ids=pos, past_key_values=self._cache, use_cache=True)
        self._tok = out.logits[:, -1, :].argmax(dim=-1, keepdim=True).contiguous()
        self._pos = torch.full((B, 1), P, dtype=torch.long, device=self.device)
        tokens = [self._tok.clone()]
        if n_new == 1:
            return torch.cat(tokens, dim=1)
        # The first decode step runs eagerly on a side stream (library and allocator
        # warm-up), then one step is captured; the cache and position buffers stay in place.
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._step()
        torch.cuda.current_stream(self.device).wait_stream(side)
        tokens.append(self._tok.clone())
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph, stream=side):
            self._step()
        torch.cuda.synchronize(self.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        outs = torch.empty(B, n_new - 2, dtype=torch.long, device=self.device)
        e0.record()
        for i in range(n_new - 2):
            self._graph.replay()
            outs[:, i:i + 1].copy_(self._tok)
        e1.record()
        torch.cuda.synchronize(self.device)
        self.decode_seconds = e0.elapsed_time(e1) / 1e3
        self._graph = None
        return torch.cat(tokens + [outs], dim=1)
