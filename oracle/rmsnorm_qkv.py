"""CPU oracle for residual add -> RMSNorm -> packed (GQA) projection.

TEST INFRASTRUCTURE.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg may use this module, and only as the checker or the timed CPU reference.

A restatement, step by step, of the reference's unfused PyTorch path
``rmsnorm_residual_qkv`` (src/triton_fused_rmsnorm_qkv/baseline.py:25-70), run with
PyTorch's CPU kernels, with the two corrections the north-star contract needs:

* the full projection is returned (``torch.cat`` of the three chunks, which is exactly
  ``F.linear(normed, W)``, baseline.py:67) and split by the real GQA widths
  (integration/llama3_patch.py:156-158) instead of ``chunk(3)`` (baseline.py:68),
  which splits a GQA width into wrong thirds;
* ``residual=None`` (HAS_RESIDUAL=0) is served as no add (the reference raises a
  TypeError at baseline.py:48 on None).

Pinned against the reference itself: tests/golden/golden.npz holds outputs of the
reference's baseline.py run in the build container on the inputs of ``make_case``
(script: tests/golden/make_golden.py); tests/test_oracle.py checks this module
reproduces them bit for bit.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


def residual_add(x: torch.Tensor, residual: Optional[torch.Tensor]) -> torch.Tensor:
    """hidden = x + residual in the working dtype (baseline.py:48).

    PyTorch adds two half-precision tensors by converting both to fp32, adding once and
    rounding to nearest-even: the updated residual the fused kernels must reproduce
    bit for bit.
    """
    return x if residual is None else x + residual


def rms_normalize(hidden: torch.Tensor, rms_weight: torch.Tensor, eps: float) -> torch.Tensor:
    """normed = dtype((fp32(h) * rsqrt(mean(fp32(h)^2) + eps)) * fp32(g)) (baseline.py:58-62)."""
    dt = hidden.dtype
    h32 = hidden.to(torch.float32)                               # baseline.py:59
    variance = h32.pow(2).mean(dim=-1, keepdim=True)            # baseline.py:60
    scaled = h32 * torch.rsqrt(variance + eps)                  # baseline.py:61
    return (scaled * rms_weight.to(torch.float32)).to(dt)       # baseline.py:62


def project(normed: torch.Tensor, weight: torch.Tensor, accumulate: str = "native") -> torch.Tensor:
    """out = normed @ weight^T (baseline.py:67).

    ``native``: ``F.linear`` in the working dtype, as the reference runs it (CPU BLAS,
    fp32 accumulation, one rounding).  ``fp32``: the same product with both operands
    widened to fp32 and one final rounding -- the fp32-accumulation result the fused
    kernels compute, and much faster on the CPU for large shapes.
    """
    if accumulate == "native" or normed.dtype == torch.float32:
        return F.linear(normed, weight)
    if accumulate == "fp32":
        return F.linear(normed.to(torch.float32), weight.to(torch.float32)).to(normed.dtype)
    raise ValueError(f"unknown accumulate mode {accumulate!r}")


def forward(x: torch.Tensor, residual: Optional[torch.Tensor], rms_weight: torch.Tensor, weight: torch.Tensor,
            eps: float, accumulate: str = "native") -> Tuple[torch.Tensor, torch.Tensor]:
    """The whole path: returns (out [..., N], hidden [..., H]) on the CPU."""
    hidden = residual_add(x, residual)
    return project(rms_normalize(hidden, rms_weight, eps), weight, accumulate), hidden


def split_qkv(out: torch.Tensor, h_q: int, h_kv: int):
    """Q, K, V views of a packed [q | k | v] output (integration/llama3_patch.py:156-158)."""
    return out[..., :h_q], out[..., h_q:h_q + h_kv], out[..., h_q + h_kv:h_q + 2 * h_kv]


def ulp(values: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Spacing of the ``dtype`` grid at each |value| (fp64), i.e. one unit in the last place."""
    mbits = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}[dtype]
    a = values.detach().to("cpu", torch.float64).abs()
    _, e = torch.frexp(a)                      # a = m * 2^e, m in [0.5, 1)
    u = torch.ldexp(torch.ones_like(a), (e - 1 - mbits).to(torch.int32))
    return torch.where(a > 0, u, torch.zeros_like(a))


def parity_metrics(got: torch.Tensor, ref: torch.Tensor, abs_bar: float = 2e-2) -> dict:
    """Error of ``got`` against ``ref`` (both taken in fp64).

    max_abs / rel_l2: the contract's metrics.  ``n_over_abs``: elements whose error is
    above ``abs_bar``; ``max_ulp_over_abs``: the largest of those errors in units of the
    reference's ulp -- 1.0 means the kernel rounded to the adjacent representable value,
    the smallest possible difference (bf16's ulp is 0.03125 for |x| in [4, 8), above a
    2e-2 bar).
    """
    g = got.detach().to("cpu", torch.float64)
    r = ref.detach().to("cpu", torch.float64)
    diff = (g - r).abs()
    denom = float(r.norm())
    over = diff > abs_bar
    n_over = int(over.sum())
    max_ulp = 0.0
    if n_over and ref.dtype in (torch.bfloat16, torch.float16, torch.float32):
        max_ulp = float((diff[over] / ulp(ref.detach().cpu()[over], ref.dtype)).max())
    return {
        "max_abs": float(diff.max()) if diff.numel() else 0.0,
        "rel_l2": float((g - r).norm()) / denom if denom > 0 else float((g - r).norm()),
        "nonfinite": int((~torch.isfinite(g)).sum()),
        "n_over_abs": n_over,
        "max_ulp_over_abs": max_ulp,
        "n": int(diff.numel()),
    }


def within_bars(m: dict, abs_bar: float = 2e-2, rel_bar: float = 5e-3) -> bool:
    """The parity bar: rel-L2 <= rel_bar and every element within max(abs_bar, 1 ulp)."""
    return (m["nonfinite"] == 0 and m["rel_l2"] <= rel_bar
            and (m["n_over_abs"] == 0 or m["max_ulp_over_abs"] <= 1.0))


def faithful_rounding_metrics(got: torch.Tensor, exact: torch.Tensor) -> dict:
    """How far a half-precision ``got`` is from the unrounded fp32 result ``exact``.

    A correctly rounded output is within 0.5 ulp of ``exact``; fp32 accumulation order
    and the odd normalised activation rounded the other way add a little.  ``n_bad``
    counts elements beyond 0.6 ulp + 2e-3 (the slack covers near-zero outputs, whose
    ulp is tiny); ``max_excess`` is the largest error beyond half an ulp.
    """
    g = got.detach().to("cpu", torch.float64)
    e = exact.detach().to("cpu", torch.float64)
    u = ulp(got.detach().cpu(), got.dtype)
    err = (g - e).abs()
    return {"n_bad": int((err > 0.6 * u + 2e-3).sum()),
            "max_excess": float((err - 0.5 * u).max()),
            "max_abs": float(err.max())}


def make_case(M: int, H: int, N: int, dtype: torch.dtype, seed: int, has_residual: bool = True,
              gain_dtype: Optional[torch.dtype] = None, w_std: float = 0.02):
    """Seeded synthetic inputs with the distributions the benchmark configs name.

    x, residual ~ N(0, 1); rms_weight = 1 + 0.1 N(0, 1); W ~ N(0, w_std).  Drawn on the
    CPU from ``torch.Generator().manual_seed(seed)`` in a fixed order, so every machine
    with this PyTorch version produces the same tensors.
    """
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(M, H, generator=gen, dtype=torch.float32).to(dtype)
    r = torch.randn(M, H, generator=gen, dtype=torch.float32).to(dtype) if has_residual else None
    g = (1.0 + 0.1 * torch.randn(H, generator=gen, dtype=torch.float32)).to(gain_dtype or dtype)
    w = (w_std * torch.randn(N, H, generator=gen, dtype=torch.float32)).to(dtype)
    return x, r, g, w


def tolerance_for(H: int) -> float:
    """Scaled max-abs bound of the reference's GPU tests (tests/test_correctness.py:305-306)."""
    return math.sqrt(H / 512)
