"""CPU oracle for the FP8-weight (e4m3, one fp32 scale per weight row) variant of the path
(test infrastructure).

The residual add and the normalisation are the reference's (``baseline.py:48-62``,
restated in ``rmsnorm_qkv.py``).  The projection uses the exactly dequantised weight:
``out = dtype(scale[n] * sum_k normed[m, k] * float(w8[n, k]))``, summed in fp64 here.
There is no FP8 path in the reference (its README lists FP8 weights as future work); this
is the contract of the new path.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .rmsnorm_qkv import residual_add, rms_normalize


def forward_fp8w(x: torch.Tensor, residual: Optional[torch.Tensor], rms_weight: torch.Tensor, w8: torch.Tensor,
                 scale: torch.Tensor, eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """(out [..., N], hidden [..., H]) on the CPU."""
    hidden = residual_add(x, residual)
    normed = rms_normalize(hidden, rms_weight, eps)
    acc = normed.double() @ w8.double().T
    return (acc * scale.double()).to(x.dtype), hidden
