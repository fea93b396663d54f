"""The reference's own CUDA tests (tests/test_correctness.py:158-346), restated against
this package: the fused op versus the unfused PyTorch path on the GPU, with the
reference's shapes, seeds, distributions and tolerances."""
from __future__ import annotations

import pytest
import torch

from triton_fused_rmsnorm_qkv import (
    fused_rmsnorm_residual_matmul,
    fused_rmsnorm_residual_matmul_fixed,
    fused_rmsnorm_residual_qkv,
    fused_rmsnorm_residual_qkv_fixed,
    get_autotune_best_config,
    rmsnorm_residual_qkv,
)

pytestmark = pytest.mark.gpu

# tests/test_correctness.py:162-168
CUDA_SHAPES = [(1, 16, 512), (1, 128, 512), (2, 256, 1024), (4, 512, 2048), (1, 2048, 4096)]
# tests/test_correctness.py:255-263: (B, S, H, H_kv)
GQA_SHAPES = [(1, 1, 512, 128), (1, 16, 512, 128), (1, 128, 1024, 256), (2, 256, 1024, 256),
              (1, 1, 4096, 1024), (1, 32, 3584, 512)]
DTYPES = [torch.float16, torch.bfloat16]


def _tol(H, dtype):
    """tests/test_correctness.py:205-208."""
    return (2e-1 if dtype == torch.bfloat16 else 5e-2) * (H / 512) ** 0.5, 1e-1


def _manual_reference(x, residual, rms_weight, weight, eps):
    """tests/test_correctness.py:281-287, restated: optional add, fp32 RMS, cast, linear."""
    h = (x if residual is None else x + residual).float()
    h = h * torch.rsqrt(h.pow(2).mean(dim=-1, keepdim=True) + eps)
    return torch.nn.functional.linear((h * rms_weight.float()).to(x.dtype), weight)


@pytest.mark.parametrize("shape", CUDA_SHAPES, ids=lambda s: f"B{s[0]}_S{s[1]}_H{s[2]}")
@pytest.mark.parametrize("dtype", DTYPES, ids=["fp16", "bf16"])
@pytest.mark.parametrize("fixed", [False, True], ids=["auto", "fixed"])
def test_fused_matches_baseline(shape, dtype, fixed):
    B, S, H = shape
    torch.manual_seed(42)
    x = torch.randn(B, S, H, dtype=dtype, device="cuda")
    residual = torch.randn(B, S, H, dtype=dtype, device="cuda")
    rms_weight = torch.randn(H, dtype=dtype, device="cuda")
    qkv_weight = torch.randn(3 * H, H, dtype=dtype, device="cuda")
    base = rmsnorm_residual_qkv(x, residual, rms_weight, qkv_weight, 1e-5)
    fn = fused_rmsnorm_residual_qkv_fixed if fixed else fused_rmsnorm_residual_qkv
    fused = fn(x, residual, rms_weight, qkv_weight, 1e-5)
    atol, rtol = _tol(H, dtype)
    for f, b in zip(fused, base):
        assert f.shape == (B, S, H) and f.dtype == dtype
        torch.testing.assert_close(f, b, atol=atol, rtol=rtol)


@pytest.mark.parametrize("shape", CUDA_SHAPES, ids=lambda s: f"B{s[0]}_S{s[1]}_H{s[2]}")
@pytest.mark.parametrize("dtype", DTYPES, ids=["fp16", "bf16"])
def test_no_nans_with_zero_residual(shape, dtype):
    B, S, H = shape
    torch.manual_seed(0)
    x = torch.randn(B, S, H, dtype=dtype, device="cuda")
    q, k, v = fused_rmsnorm_residual_qkv(x, torch.zeros_like(x), torch.ones(H, dtype=dtype, device="cuda"),
                                         torch.randn(3 * H, H, dtype=dtype, device="cuda"))
    for t in (q, k, v):
        assert not torch.isnan(t).any()


@pytest.mark.parametrize("gqa", GQA_SHAPES, ids=lambda s: f"B{s[0]}_S{s[1]}_H{s[2]}_Hkv{s[3]}")
@pytest.mark.parametrize("dtype", DTYPES, ids=["fp16", "bf16"])
@pytest.mark.parametrize("with_residual", [True, False], ids=["residual", "none"])
def test_gqa_matches_reference(gqa, dtype, with_residual):
    B, S, H, H_kv = gqa
    torch.manual_seed(7 if with_residual else 11)
    N_OUT = H + 2 * H_kv
    x = torch.randn(B, S, H, dtype=dtype, device="cuda")
    residual = torch.randn(B, S, H, dtype=dtype, device="cuda") if with_residual else None
    rms_weight = torch.randn(H, dtype=dtype, device="cuda")
    weight = torch.randn(N_OUT, H, dtype=dtype, device="cuda") * 0.02
    out = fused_rmsnorm_residual_matmul(x, residual, rms_weight, weight, 1e-5)
    assert out.shape == (B, S, N_OUT)
    atol, rtol = _tol(H, dtype)
    torch.testing.assert_close(out, _manual_reference(x, residual, rms_weight, weight, 1e-5), atol=atol, rtol=rtol)
    out_fixed = fused_rmsnorm_residual_matmul_fixed(x, residual, rms_weight, weight, 1e-5)
    torch.testing.assert_close(out_fixed, out, atol=atol, rtol=rtol)


@pytest.mark.parametrize("gqa", GQA_SHAPES, ids=lambda s: f"B{s[0]}_S{s[1]}_H{s[2]}_Hkv{s[3]}")
def test_gqa_split_widths(gqa):
    B, S, H, H_kv = gqa
    torch.manual_seed(0)
    x = torch.randn(B, S, H, dtype=torch.bfloat16, device="cuda")
    weight = torch.randn(H + 2 * H_kv, H, dtype=torch.bfloat16, device="cuda") * 0.02
    out = fused_rmsnorm_residual_matmul(x, None, torch.ones(H, dtype=torch.bfloat16, device="cuda"), weight)
    q, k, v = out[..., :H], out[..., H:H + H_kv], out[..., H + H_kv:H + 2 * H_kv]
    assert q.shape == (B, S, H) and k.shape == (B, S, H_kv) and v.shape == (B, S, H_kv)
    assert not torch.isnan(out).any()


def test_get_autotune_best_config_describes_the_schedule():
    x = torch.randn(1, 16, 4096, dtype=torch.bfloat16, device="cuda")
    w = torch.randn(6144, 4096, dtype=torch.bfloat16, device="cuda") * 0.02
    fused_rmsnorm_residual_matmul(x, None, torch.ones(4096, device="cuda"), w)
    cfg = get_autotune_best_config(16, 4096)
    assert cfg is not None and {"BLOCK_M", "BLOCK_N", "BLOCK_K", "num_warps", "num_stages"} <= set(cfg)
    assert cfg["schedule"] == "decode"
    assert get_autotune_best_config(3, 77) is None


def test_mha_wrapper_rejects_gqa_weight():
    x = torch.randn(1, 4, 512, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(AssertionError, match="For GQA"):
        fused_rmsnorm_residual_qkv(x, None, torch.ones(512, device="cuda"),
                                   torch.randn(768, 512, dtype=torch.bfloat16, device="cuda"))
