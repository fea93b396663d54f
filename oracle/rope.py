"""CPU oracle for the Q/K/V split with the rotary position embedding (test infrastructure).

Restates what the reference's Llama integration does after the fused projection
(``integration/llama3_patch.py:156-168``): split the packed output by the real GQA widths,
view each part as heads, transpose to (B, heads, S, d), and apply transformers'
``apply_rotary_pos_emb`` (transformers 5.5, ``models/llama/modeling_llama.py``:
``rotate_half(x) = cat(-x[..., d/2:], x[..., :d/2])`` and
``x * cos + rotate_half(x) * sin`` with cos / sin unsqueezed on the head axis).  Every
step is a PyTorch elementwise op in the tensors' own 16-bit dtype, as in the model, so
the oracle rounds exactly where the model does.  ``tests/test_oracle.py`` pins it to
transformers' own function.
"""
from __future__ import annotations

from typing import Tuple

import torch


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def rope_split(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, n_q: int, n_kv: int,
               head_dim: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(q, k, v) head-major from qkv (B, S, (n_q + 2 n_kv) d); q and k rotated."""
    B, S, _ = qkv.shape
    q, k, v = torch.split(qkv, [n_q * head_dim, n_kv * head_dim, n_kv * head_dim], dim=-1)
    q = q.reshape(B, S, n_q, head_dim).transpose(1, 2)
    k = k.reshape(B, S, n_kv, head_dim).transpose(1, 2)
    v = v.reshape(B, S, n_kv, head_dim).transpose(1, 2)
    if cos.dim() == 2:
        cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    c, s = cos.unsqueeze(1), sin.unsqueeze(1)
    q = (q * c) + (rotate_half(q) * s)
    k = (k * c) + (rotate_half(k) * s)
    return q.contiguous(), k.contiguous(), v.contiguous()


def make_rope_case(B: int, S: int, n_q: int, n_kv: int, head_dim: int, dtype: torch.dtype, seed: int,
                   cos_batch: int = 1, theta: float = 500000.0):
    """Seeded qkv ~ N(0, 1) and the cos / sin tables of positions 0..S-1 (per batch row an
    offset of 3 * b when cos_batch == B), built the way the model's rotary embedding builds
    them: fp32 angles, cos / sin cast to the dtype."""
    gen = torch.Generator().manual_seed(seed)
    qkv = torch.randn(B, S, (n_q + 2 * n_kv) * head_dim, generator=gen, dtype=torch.float32).to(dtype)
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    pos = torch.arange(S, dtype=torch.float32)[None, :] + 3.0 * torch.arange(cos_batch, dtype=torch.float32)[:, None]
    freqs = pos[..., None] * inv_freq
    emb = torch.cat((freqs, freqs), dim=-1)
    return qkv, emb.cos().to(dtype), emb.sin().to(dtype)
