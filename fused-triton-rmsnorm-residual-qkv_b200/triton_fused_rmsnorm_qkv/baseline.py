"""Unfused PyTorch path: residual add, RMSNorm, packed linear, split into three.

Same function, arguments and results as the reference's ``baseline.py``
(``rmsnorm_residual_qkv``, baseline.py:25-70); it runs on whatever device its inputs
live on (cuBLAS on a GPU, the CPU BLAS otherwise) and is the comparator the fused
kernels are benchmarked against.

    hidden = x + residual                               (baseline.py:48)
    normed = dtype(fp32(hidden) * rsqrt(mean(fp32(hidden)^2) + eps) * fp32(rms_weight))
                                                        (baseline.py:58-62)
    Q, K, V = (normed @ qkv_weight^T).chunk(3, -1)      (baseline.py:67-68)

``residual`` may also be None here (the reference raises on None); the add is then
skipped.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn.functional as F


def _rms_normalize(hidden: torch.Tensor, rms_weight: torch.Tensor, eps: float) -> torch.Tensor:
    h32 = hidden.float()
    inv_rms = torch.rsqrt(h32.square().mean(dim=-1, keepdim=True) + eps)
    return ((h32 * inv_rms) * rms_weight.float()).to(hidden.dtype)


def rmsnorm_residual_qkv(
    x: torch.Tensor,
    residual: Optional[torch.Tensor],
    rms_weight: torch.Tensor,
    qkv_weight: torch.Tensor,
    eps: float = 1e-6,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Unfused residual add -> RMSNorm -> packed QKV linear -> ``chunk(3)``.

    Args:
        x: (B, S, H) activations.
        residual: (B, S, H) residual stream in x's dtype (or None).
        rms_weight: (H,) RMSNorm gain.
        qkv_weight: (3*H, H) packed [W_Q; W_K; W_V].
        eps: RMSNorm epsilon.

    Returns:
        (Q, K, V) in x's dtype.  For a GQA weight of another width, ``chunk(3)`` splits
        into near-equal thirds exactly as the reference does; take ``torch.cat`` of the
        three to recover the full projection.
    """
    hidden = x if residual is None else x + residual
    projected = F.linear(_rms_normalize(hidden, rms_weight, eps), qkv_weight)
    q, k, v = projected.chunk(3, dim=-1)
    return q, k, v
