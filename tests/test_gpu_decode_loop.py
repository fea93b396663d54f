"""End-to-end check of the integration in a KV-cache decode loop: greedy decoding with a
static KV cache, one token per step replayed from a CUDA graph
(``integration.GraphedGreedyDecoder``), on a Llama-3-8B-shaped model with random weights.
The patched model (the reference's Q/K/V patch, and the fullest mode: cross-layer fusion
with the one-launch rotary split) must produce the unpatched model's greedy tokens for
every step."""
from __future__ import annotations

import pytest
import torch

from integration import GraphedGreedyDecoder, build_llama3_8b, fused_patch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [1, 4])
def test_patched_greedy_decode_matches_unpatched(batch):
    model = build_llama3_8b(dtype=torch.bfloat16, device="cuda", num_hidden_layers=2)
    gen = torch.Generator(device="cuda").manual_seed(3 + batch)
    prompt = torch.randint(0, model.config.vocab_size, (batch, 12), generator=gen, device="cuda")
    n_new = 20
    ref = GraphedGreedyDecoder(model, batch, 64).generate(prompt, n_new)
    assert ref.shape == (batch, n_new)
    for kw in ({}, {"cross_layer": True, "rope": True}):
        with fused_patch(model, **kw):
            got = GraphedGreedyDecoder(model, batch, 64).generate(prompt, n_new)
        assert torch.equal(got, ref), (kw, got, ref)
    del model
    torch.cuda.empty_cache()
