"""The FP8-weight (e4m3 + fp32 row scale) decode path against its CPU oracle."""
from __future__ import annotations

import pytest
import torch

from oracle import forward_fp8w, make_case, parity_metrics, within_bars
from triton_fused_rmsnorm_qkv import _lib, device_status, fused_add_rmsnorm_matmul_fp8w, quantize_weight_e4m3

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 5e-3


def run_fp8(M, H, N, dtype, seed, res=True):
    x, r, g, w = make_case(M, H, N, dtype, seed, res)
    w8, scale = quantize_weight_e4m3(w)
    out, hidden = fused_add_rmsnorm_matmul_fp8w(x.cuda()[None], r.cuda()[None] if r is not None else None, g.cuda(),
                                                w8.cuda(), scale.cuda(), 1e-5)
    torch.cuda.synchronize()
    ref, ref_hidden = forward_fp8w(x, r, g, w8, scale, 1e-5)
    m = parity_metrics(out[0].cpu(), ref)
    assert within_bars(m, MAX_ABS, REL_L2), m
    assert torch.equal(hidden[0].cpu(), ref_hidden)
    assert device_status() == 0
    return m


@pytest.mark.parametrize("M", [1, 4, 16, 64])
def test_llama3_8b_decode_fp8w(M):
    run_fp8(M, 4096, 6144, torch.bfloat16, seed=300 + M)


def test_llama3_8b_decode_fp8w_fp16():
    run_fp8(16, 4096, 6144, torch.float16, seed=41)


@pytest.mark.parametrize("M", [1, 16])
def test_qwen2_fp8w_no_residual(M):
    run_fp8(M, 3584, 4608, torch.bfloat16, seed=50 + M, res=False)


@pytest.mark.parametrize("M", [1, 16])
def test_gate_up_fp8w(M):
    """N = 2 x 14336: the wide-weight configurations (more 128-row tiles per CTA)."""
    info = _lib.query_schedule(M, 4096, 28672, _lib.BF16)
    print(info)
    run_fp8(M, 4096, 28672, torch.bfloat16, seed=60 + M)


@pytest.mark.parametrize("M,H,N", [(5, 272, 200), (33, 512, 768), (1, 1024, 1280),
                                   (2, 272, 200), (3, 1040, 700), (4, 8192, 1024)])  # the spread norm phase
def test_ragged_fp8w(M, H, N):
    run_fp8(M, H, N, torch.bfloat16, seed=M + H)


@pytest.mark.parametrize("M", [1, 2, 4])
def test_spread_fp8w_fp16_three_terms(M):
    """fp16: three e4m3 terms per value, whose regions reach past their own 128 K of the
    16-bit buffer they overwrite; the spread norm phase (M <= 4) reads every h first."""
    run_fp8(M, 1040, 1280, torch.float16, seed=80 + M)


def test_fp8w_rejects_prefill_sizes():
    x = torch.zeros(1, 65, 256, dtype=torch.bfloat16, device="cuda")
    w8 = torch.zeros(512, 256, dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(ValueError):
        fused_add_rmsnorm_matmul_fp8w(x, None, torch.ones(256, device="cuda"), w8,
                                      torch.ones(512, device="cuda"), 1e-5)


@pytest.mark.parametrize("M", [1, 32, 64])
def test_llama3_8b_decode_fp8w_fp16_sizes(M):
    """fp16 activations take three e4m3 terms; above 32 rows they run as two launches."""
    run_fp8(M, 4096, 6144, torch.float16, seed=70 + M)


@pytest.mark.parametrize("M", [16, 1, 4])
@pytest.mark.parametrize("dtype,min_equal", [(torch.bfloat16, 0.99), (torch.float16, 0.97)])
def test_fp8w_term_split_is_exact(dtype, min_equal, M):
    """The activations' e4m3 terms hold the normalised values exactly, so the kernel differs
    from the fp64 oracle only by its fp32 accumulation: nearly every output is bit-identical,
    and none is further away than one unit in the last place plus the fp32 rounding of a
    4096-term sum (1e-5 of the largest output; it dominates only for outputs near zero).
    M = 1 and 4 run the spread norm phase."""
    H, N = 4096, 6144
    x, r, g, w = make_case(M, H, N, dtype, seed=91)
    w8, scale = quantize_weight_e4m3(w)
    out, _ = fused_add_rmsnorm_matmul_fp8w(x.cuda()[None], r.cuda()[None], g.cuda(), w8.cuda(), scale.cuda(), 1e-5)
    torch.cuda.synchronize()
    ref, _ = forward_fp8w(x, r, g, w8, scale, 1e-5)
    got = out[0].cpu()
    equal = (got == ref).float().mean().item()
    assert equal >= min_equal, equal
    # one unit in the last place of the dtype at each reference value (away from zero)
    away = torch.where(ref >= 0, torch.tensor(float("inf"), dtype=dtype), torch.tensor(float("-inf"), dtype=dtype))
    step = (torch.nextafter(ref, away).float() - ref.float()).abs()
    tol = step + 1e-5 * ref.float().abs().max()
    assert bool(((got.float() - ref.float()).abs() <= tol).all())
