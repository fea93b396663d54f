"""Route each Llama decoder layer's input RMSNorm + Q/K/V projections through the fused op.

Same public surface and behaviour as the reference's ``integration/llama3_patch.py``:

* ``apply_fused_patch(model)`` stores, per ``LlamaDecoderLayer``, the packed GQA weight
  ``[Wq; Wk; Wv]`` of shape ``(H + 2 * H_kv, H)`` (no zero padding, llama3_patch.py:111-127)
  and rebinds the layer's ``forward`` (llama3_patch.py:206-215);
* the patched forward calls ``fused_rmsnorm_residual_matmul(hidden_states, None,
  input_layernorm.weight, packed, eps)`` -- Llama adds its residual after attention, so
  the fused call has none (llama3_patch.py:148-154) -- then splits Q/K/V by their real
  widths and runs the unchanged rest of the layer (RoPE, KV cache, attention, o_proj,
  residual, post-attention norm, MLP, residual; llama3_patch.py:156-196);
* ``TRITON_FUSED_DISABLE_AUTOTUNE=1`` selects the ``_fixed`` entry point
  (llama3_patch.py:61-65);
* ``remove_fused_patch`` / ``fused_patch`` undo it (llama3_patch.py:218-239).

Beyond the reference, ``apply_fused_patch(model, mlp=True)`` also routes the layer's
second half through the op.  ``fused_add_rmsnorm_matmul(attn_out, residual,
post_attention_layernorm.weight, [W_gate; W_up])`` forms the updated residual stream
``residual + attn_out`` (bit-exact, returned), normalises it and projects it onto the
packed gate/up weight in one launch.  The layer then applies ``down_proj(act(gate) * up)``
and adds the MLP output to the returned stream (llama3_patch.py:190-194).

``cross_layer=True`` (implies ``mlp=True``) also fuses across layer boundaries.  A layer
other than the last returns its MLP output alone and leaves the updated residual stream
in a per-model carry.  The next layer's input call is then
``fused_add_rmsnorm_matmul(mlp_out, stream, input_layernorm.weight, [Wq; Wk; Wv])``: one
launch adds the two (bit-exact), normalises and projects.  The last layer returns the
full stream, so the final norm is unchanged.  The stream between layers therefore exists
only inside that carry: ``cross_layer`` is for plain forward passes.  Hidden states
collected between layers (``output_hidden_states``) and forward hooks on single layers
see the MLP outputs, not the stream, and a single layer called on its own returns a
partial value.  The first layer of each forward clears the carry, and a layer that raises
clears it too.

``rope=True`` replaces the fused Q/K/V call and the split / view / transpose /
``apply_rotary_pos_emb`` sequence after it by ``fused_add_rmsnorm_qkv_rope``: at decode sizes
one launch whose epilogue writes head-major Q, K, V with Q and K rotated, bit-identical to
that sequence (other sizes: the fused call and ``qkv_rope_split``).

Written against transformers 5.5 (``LlamaDecoderLayer.forward`` / ``LlamaAttention``).
"""
from __future__ import annotations

import os
from contextlib import contextmanager
from typing import Optional

import torch
from transformers import LlamaConfig, LlamaForCausalLM
from transformers.models.llama.modeling_llama import (
    ALL_ATTENTION_FUNCTIONS,
    LlamaAttention,
    apply_rotary_pos_emb,
    eager_attention_forward,
)

from triton_fused_rmsnorm_qkv import (
    fused_add_rmsnorm_matmul,
    fused_add_rmsnorm_qkv_rope,
    fused_rmsnorm_residual_matmul,
    fused_rmsnorm_residual_matmul_fixed,
    qkv_rope_split,
)

LLAMA3_8B_CONFIG = dict(
    hidden_size=4096,
    intermediate_size=14336,
    num_hidden_layers=32,
    num_attention_heads=32,
    num_key_value_heads=8,
    head_dim=128,
    max_position_embeddings=8192,
    rms_norm_eps=1e-5,
    vocab_size=128256,
    rope_theta=500000.0,
    tie_word_embeddings=False,
    attention_bias=False,
    mlp_bias=False,
)

_ORIGINAL = "_fused_original_forward"
_LAYER_ATTRS = ("_fused_packed_qkv", "_fused_H_kv", "_fused_packed_gate_up", "_fused_intermediate",
                "_fused_carry", "_fused_first", "_fused_last", "_fused_rope")


def _fixed() -> bool:
    """TRITON_FUSED_DISABLE_AUTOTUNE=1 selects the fixed-tile (``_fixed``) kernels."""
    return os.environ.get("TRITON_FUSED_DISABLE_AUTOTUNE") == "1"


def _fused_op():
    """The fused entry point for this call (env TRITON_FUSED_DISABLE_AUTOTUNE=1 -> _fixed)."""
    return fused_rmsnorm_residual_matmul_fixed if _fixed() else fused_rmsnorm_residual_matmul


def _fused_add(x, residual, rms_weight, weight, eps):
    """(out, x + residual) in one launch, on the fixed-tile kernel when _fixed()."""
    return fused_add_rmsnorm_matmul(x, residual, rms_weight, weight, eps=eps, schedule="simt" if _fixed() else None)


def build_llama3_8b(dtype: torch.dtype = torch.float16, device: str = "cuda",
                    num_hidden_layers: Optional[int] = None) -> LlamaForCausalLM:
    """A Llama-3-8B-shaped ``LlamaForCausalLM`` with random weights, in eval mode."""
    cfg = dict(LLAMA3_8B_CONFIG)
    if num_hidden_layers is not None:
        cfg["num_hidden_layers"] = num_hidden_layers
    saved = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device(device):
            model = LlamaForCausalLM(LlamaConfig(**cfg))
    finally:
        torch.set_default_dtype(saved)
    return model.eval()


def pack_qkv_weight(attn: LlamaAttention) -> torch.Tensor:
    """``[Wq; Wk; Wv]`` stacked along the output dimension, without padding."""
    wq, wk, wv = attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight
    hidden = wq.shape[1]
    if wq.shape[0] != hidden:
        raise ValueError(f"q_proj must map {hidden} -> {hidden}, got {tuple(wq.shape)}")
    if wk.shape != wv.shape:
        raise ValueError(f"k_proj {tuple(wk.shape)} and v_proj {tuple(wv.shape)} must have the same shape")
    return torch.cat([wq.detach(), wk.detach(), wv.detach()], dim=0).contiguous()


def pack_gate_up_weight(mlp) -> torch.Tensor:
    """``[W_gate; W_up]`` stacked along the output dimension (2 * intermediate rows)."""
    wg, wu = mlp.gate_proj.weight, mlp.up_proj.weight
    if wg.shape != wu.shape:
        raise ValueError(f"gate_proj {tuple(wg.shape)} and up_proj {tuple(wu.shape)} must have the same shape")
    if getattr(mlp.gate_proj, "bias", None) is not None or getattr(mlp.up_proj, "bias", None) is not None:
        raise ValueError("the fused gate/up projection has no bias")
    return torch.cat([wg.detach(), wu.detach()], dim=0).contiguous()


def _patched_forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                     use_cache=False, position_embeddings=None, **kwargs):
    """LlamaDecoderLayer.forward with input_layernorm + q/k/v_proj replaced by one fused op
    (and, when the layer was patched with ``mlp=True``, the post-attention residual add +
    post_attention_layernorm + gate/up projections by a second one)."""
    attn = self.self_attn
    lead = hidden_states.shape[:-1]
    h_kv = self._fused_H_kv
    h_q = self._fused_packed_qkv.shape[0] - 2 * h_kv
    carry = getattr(self, "_fused_carry", None)
    if carry is not None and self._fused_first:
        carry.clear()  # a forward that raised part-way leaves nothing behind for this one
    pending = None if carry is None else carry.pop("stream", None)
    try:
        return _patched_body(self, hidden_states, attention_mask, past_key_values, position_embeddings, carry,
                             pending, lead, attn, h_q, h_kv, **kwargs)
    except BaseException:
        if carry is not None:
            carry.clear()
        raise


def _patched_body(self, hidden_states, attention_mask, past_key_values, position_embeddings, carry, pending, lead,
                  attn, h_q, h_kv, **kwargs):
    """The patched layer's work (see _patched_forward)."""
    cos, sin = position_embeddings
    ln = self.input_layernorm
    if getattr(self, "_fused_rope", False) and not _fixed():
        # One launch: norm, projection, head split and rotary embedding (decode sizes; the
        # op runs the projection and the split as two launches otherwise).
        heads = (h_q // attn.head_dim, h_kv // attn.head_dim, attn.head_dim)
        if pending is None:
            q, k, v = fused_add_rmsnorm_qkv_rope(hidden_states, None, ln.weight, self._fused_packed_qkv, cos, sin,
                                                 *heads, ln.variance_epsilon, return_residual=False)
        else:
            q, k, v, hidden_states = fused_add_rmsnorm_qkv_rope(hidden_states, pending, ln.weight,
                                                                self._fused_packed_qkv, cos, sin, *heads,
                                                                ln.variance_epsilon)
        return _attend_and_mlp(self, hidden_states, q, k, v, attention_mask, past_key_values, carry, lead, attn,
                               **kwargs)
    if pending is None:
        qkv = _fused_op()(hidden_states, None, ln.weight, self._fused_packed_qkv, eps=ln.variance_epsilon)
    else:
        # The previous layer's MLP output arrives with the stream it belongs to.
        qkv, hidden_states = _fused_add(hidden_states, pending, ln.weight, self._fused_packed_qkv,
                                        ln.variance_epsilon)
    if getattr(self, "_fused_rope", False):
        q, k, v = qkv_rope_split(qkv, cos, sin, h_q // attn.head_dim, h_kv // attn.head_dim, attn.head_dim)
    else:
        q, k, v = torch.split(qkv, [h_q, h_kv, h_kv], dim=-1)
        q = q.reshape(*lead, -1, attn.head_dim).transpose(1, 2)
        k = k.reshape(*lead, -1, attn.head_dim).transpose(1, 2)
        v = v.reshape(*lead, -1, attn.head_dim).transpose(1, 2)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
    return _attend_and_mlp(self, hidden_states, q, k, v, attention_mask, past_key_values, carry, lead, attn, **kwargs)


def _attend_and_mlp(self, hidden_states, q, k, v, attention_mask, past_key_values, carry, lead, attn, **kwargs):
    """The rest of the layer after Q/K/V: KV cache, attention, o_proj, residual, MLP."""
    if past_key_values is not None:
        k, v = past_key_values.update(k, v, attn.layer_idx)
    attend = ALL_ATTENTION_FUNCTIONS.get_interface(attn.config._attn_implementation, eager_attention_forward)
    ctx, _ = attend(attn, q, k, v, attention_mask, dropout=0.0, scaling=attn.scaling, **kwargs)
    attn_out = attn.o_proj(ctx.reshape(*lead, -1).contiguous())
    gate_up_w = getattr(self, "_fused_packed_gate_up", None)
    if gate_up_w is None:
        hidden_states = hidden_states + attn_out
        return hidden_states + self.mlp(self.post_attention_layernorm(hidden_states))
    post = self.post_attention_layernorm
    gate_up, hidden_states = _fused_add(attn_out, hidden_states, post.weight, gate_up_w, post.variance_epsilon)
    gate, up = torch.split(gate_up, [self._fused_intermediate, self._fused_intermediate], dim=-1)
    mlp_out = self.mlp.down_proj(self.mlp.act_fn(gate) * up)
    if carry is not None and not self._fused_last:
        carry["stream"] = hidden_states  # added by the next layer's fused input call
        return mlp_out
    return hidden_states + mlp_out


def apply_fused_patch(model: LlamaForCausalLM, *, mlp: bool = False, cross_layer: bool = False,
                      rope: bool = False) -> LlamaForCausalLM:
    """Patch every decoder layer of ``model`` (idempotent).  ``mlp=True`` also fuses the
    post-attention residual add + norm + gate/up projections; ``cross_layer=True`` (which
    implies ``mlp``) also fuses each layer's MLP residual add into the next layer's input
    norm + Q/K/V projection; ``rope=True`` splits Q/K/V head-major and rotates Q and K in
    one launch."""
    mlp = mlp or cross_layer
    layers = model.model.layers
    n_run = min(len(layers), getattr(model.config, "num_hidden_layers", len(layers)))
    carry = {} if cross_layer else None
    for idx, layer in enumerate(layers):
        if hasattr(layer, _ORIGINAL):
            continue
        layer._fused_packed_qkv = pack_qkv_weight(layer.self_attn)
        layer._fused_H_kv = layer.self_attn.k_proj.weight.shape[0]
        if mlp:
            layer._fused_packed_gate_up = pack_gate_up_weight(layer.mlp)
            layer._fused_intermediate = layer.mlp.gate_proj.weight.shape[0]
        if rope:
            layer._fused_rope = True
        if carry is not None:
            layer._fused_carry = carry  # shared by the layers of this model
            layer._fused_first = idx == 0
            layer._fused_last = idx == n_run - 1
        setattr(layer, _ORIGINAL, layer.forward)
        layer.forward = _patched_forward.__get__(layer, type(layer))
    return model


def remove_fused_patch(model: LlamaForCausalLM) -> LlamaForCausalLM:
    """Restore the original forward of every patched layer and drop the packed weights."""
    for layer in model.model.layers:
        if not hasattr(layer, _ORIGINAL):
            continue
        layer.forward = getattr(layer, _ORIGINAL)
        delattr(layer, _ORIGINAL)
        for name in _LAYER_ATTRS:
            if hasattr(layer, name):
                delattr(layer, name)
    return model


@contextmanager
def fused_patch(model: LlamaForCausalLM, *, mlp: bool = False, cross_layer: bool = False, rope: bool = False):
    """Apply the patch for the duration of a ``with`` block."""
    apply_fused_patch(model, mlp=mlp, cross_layer=cross_layer, rope=rope)
    try:
        yield model
    finally:
        remove_fused_patch(model)
