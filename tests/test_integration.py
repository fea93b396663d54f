"""The Llama-3 integration: packing and patch bookkeeping on the CPU, end-to-end logits
of a patched model against the unpatched one on the GPU."""
from __future__ import annotations

import pytest
import torch
from transformers import LlamaConfig, LlamaForCausalLM

from integration import LLAMA3_8B_CONFIG, apply_fused_patch, build_llama3_8b, fused_patch, remove_fused_patch
from integration.llama3_patch import pack_gate_up_weight, pack_qkv_weight


def tiny_llama(device="cpu", dtype=torch.float32, layers=2):
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=layers, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, vocab_size=500, max_position_embeddings=128,
                      rms_norm_eps=1e-5, tie_word_embeddings=False)
    torch.manual_seed(0)
    saved = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device(device):
            return LlamaForCausalLM(cfg).eval()
    finally:
        torch.set_default_dtype(saved)


def test_pack_is_q_then_k_then_v_without_padding():
    model = tiny_llama()
    attn = model.model.layers[0].self_attn
    packed = pack_qkv_weight(attn)
    assert packed.shape == (256 + 2 * 128, 256)
    assert torch.equal(packed[:256], attn.q_proj.weight)
    assert torch.equal(packed[256:384], attn.k_proj.weight)
    assert torch.equal(packed[384:], attn.v_proj.weight)


def test_patch_and_unpatch_bookkeeping():
    model = tiny_llama()
    originals = [layer.forward for layer in model.model.layers]
    apply_fused_patch(model)
    apply_fused_patch(model)  # idempotent
    for layer in model.model.layers:
        assert hasattr(layer, "_fused_packed_qkv") and layer._fused_H_kv == 128
    remove_fused_patch(model)
    for layer, fwd in zip(model.model.layers, originals):
        assert not hasattr(layer, "_fused_packed_qkv")
        assert layer.forward == fwd
    with fused_patch(model):
        assert all(hasattr(layer, "_fused_packed_qkv") for layer in model.model.layers)
    assert not any(hasattr(layer, "_fused_packed_qkv") for layer in model.model.layers)


def test_pack_gate_up_is_gate_then_up():
    model = tiny_llama()
    mlp = model.model.layers[1].mlp
    packed = pack_gate_up_weight(mlp)
    assert packed.shape == (2 * 512, 256)
    assert torch.equal(packed[:512], mlp.gate_proj.weight)
    assert torch.equal(packed[512:], mlp.up_proj.weight)


def test_mlp_patch_bookkeeping():
    model = tiny_llama()
    originals = [layer.forward for layer in model.model.layers]
    with fused_patch(model, mlp=True):
        for layer in model.model.layers:
            assert layer._fused_packed_gate_up.shape == (1024, 256) and layer._fused_intermediate == 512
            assert hasattr(layer, "_fused_packed_qkv")
    for layer, fwd in zip(model.model.layers, originals):
        assert not hasattr(layer, "_fused_packed_gate_up") and not hasattr(layer, "_fused_intermediate")
        assert layer.forward == fwd
    apply_fused_patch(model)  # the reference's default: Q/K/V only
    assert not any(hasattr(layer, "_fused_packed_gate_up") for layer in model.model.layers)
    remove_fused_patch(model)


def test_cross_layer_patch_bookkeeping():
    model = tiny_llama(layers=3)
    with fused_patch(model, cross_layer=True):
        layers = model.model.layers
        assert all(hasattr(layer, "_fused_packed_gate_up") for layer in layers)  # implies mlp
        assert layers[0]._fused_carry is layers[2]._fused_carry
        assert [layer._fused_first for layer in layers] == [True, False, False]
        assert [layer._fused_last for layer in layers] == [False, False, True]
    assert not any(hasattr(layer, "_fused_carry") for layer in model.model.layers)


def test_rope_patch_bookkeeping():
    model = tiny_llama()
    with fused_patch(model, rope=True):
        assert all(getattr(layer, "_fused_rope", False) for layer in model.model.layers)
        assert not any(hasattr(layer, "_fused_packed_gate_up") for layer in model.model.layers)
    assert not any(hasattr(layer, "_fused_rope") for layer in model.model.layers)


def test_llama3_8b_config_shape():
    assert LLAMA3_8B_CONFIG["hidden_size"] + 2 * LLAMA3_8B_CONFIG["num_key_value_heads"] * \
        LLAMA3_8B_CONFIG["head_dim"] == 6144


MODES = {"qkv": {}, "qkv+mlp": {"mlp": True}, "cross-layer": {"cross_layer": True},
         "all": {"cross_layer": True, "rope": True}}


@pytest.mark.gpu
@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("fixed", [False, True], ids=["auto", "fixed"])
def test_patched_tiny_llama_matches_unpatched(fixed, mode, monkeypatch):
    if fixed:
        monkeypatch.setenv("TRITON_FUSED_DISABLE_AUTOTUNE", "1")
    model = tiny_llama("cuda", torch.bfloat16)
    ids = torch.randint(0, 500, (2, 24), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    with torch.no_grad():
        ref = model(ids).logits.float()
        with fused_patch(model, **MODES[mode]):
            got = model(ids).logits.float()
    rel = (got - ref).norm() / ref.norm()
    assert rel < 2e-2, float(rel)


def _prefill_then_decode(model, ids, cont):
    """Last-position logits of a prefill of ``ids`` and then one decode step per token of
    ``cont`` through the KV cache (teacher forcing: both runs see the same tokens)."""
    out = model(ids, use_cache=True)
    logits, cache = [out.logits[:, -1].float()], out.past_key_values
    for j in range(cont.shape[1]):
        out = model(cont[:, j:j + 1], past_key_values=cache, use_cache=True)
        logits.append(out.logits[:, -1].float())
        cache = out.past_key_values
    return logits


@pytest.mark.gpu
@pytest.mark.parametrize("mode", list(MODES))
def test_patched_llama3_8b_two_layers_decode_and_prefill(mode):
    """The Llama-3-8B layer shape (2 layers): prefill of 32 tokens (M = 32), then 4 decode
    steps (M = 1) through the KV cache, patched vs unpatched on the same token sequence.
    With "qkv+mlp" the post-attention add + norm + gate/up (N = 2 x 14336) runs through the
    fused op too; with "cross-layer" the second layer's input call also takes the first
    layer's MLP output and residual stream (R = 1).  (Greedy generation is not compared: with random weights the logits are
    nearly flat, and a rounding-level difference can change the argmax and so every later
    step's input.)"""
    model = build_llama3_8b(dtype=torch.bfloat16, device="cuda", num_hidden_layers=2)
    gen = torch.Generator(device="cuda").manual_seed(2)
    ids = torch.randint(0, 128256, (1, 32), device="cuda", generator=gen)
    cont = torch.randint(0, 128256, (1, 4), device="cuda", generator=gen)
    with torch.no_grad():
        ref = _prefill_then_decode(model, ids, cont)
        with fused_patch(model, **MODES[mode]):
            got = _prefill_then_decode(model, ids, cont)
    for a, b in zip(got, ref):
        rel = (a - b).norm() / b.norm()
        assert rel < 3e-2, float(rel)
    del model
    torch.cuda.empty_cache()


def test_cross_layer_carry_is_cleared_on_first_layer_and_on_error(monkeypatch):
    """The cross-layer carry holds the residual stream between layers: the first layer of a
    forward starts from an empty carry, and a layer that raises leaves it empty."""
    from integration import llama3_patch

    model = tiny_llama()
    apply_fused_patch(model, cross_layer=True)
    first, second = model.model.layers[0], model.model.layers[1]
    carry = first._fused_carry
    assert carry is second._fused_carry

    seen = {}

    def fake_body(self, hidden_states, attention_mask, past_key_values, position_embeddings, carry_, pending, *a,
                  **kw):
        seen["pending"] = pending
        if self is second:
            raise RuntimeError("boom")
        return hidden_states

    monkeypatch.setattr(llama3_patch, "_patched_body", fake_body)
    h = torch.zeros(1, 1, 256)
    carry["stream"] = "stale"
    first(h, position_embeddings=(None, None))
    assert seen["pending"] is None and "stream" not in carry   # stale entry dropped by the first layer
    carry["stream"] = "from layer 0"
    with pytest.raises(RuntimeError):
        second(h, position_embeddings=(None, None))
    assert seen["pending"] == "from layer 0" and carry == {}
    remove_fused_patch(model)
