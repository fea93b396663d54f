"""The CPU oracle against the reference's own outputs (golden vectors) and the
known-answer properties of the reference's tests.  CPU only."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from cases import CASES, as_bits, inputs_digest
from oracle import forward, make_case, parity_metrics, rms_normalize, split_qkv

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "golden.npz")


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_golden(case):
    """Bit-exact: the oracle reproduces the reference's baseline.py output and hidden."""
    torch.set_num_threads(1)
    x, r, g, w = make_case(case["M"], case["H"], case["N"], case["dtype"], case["seed"], case["res"])
    assert inputs_digest(x, r, g, w) == str(GOLDEN[case["name"] + "__digest"]), \
        "regenerated inputs differ from the ones the golden vectors were made from"
    out, hidden = forward(x, r, g, w, case["eps"])
    np.testing.assert_array_equal(as_bits(out), GOLDEN[case["name"] + "__out"])
    np.testing.assert_array_equal(as_bits(hidden), GOLDEN[case["name"] + "__hidden"])


@pytest.mark.parametrize("case", [c for c in CASES if c["dtype"] != torch.float32], ids=lambda c: c["name"])
def test_fp32_accumulation_mode_within_tolerance(case):
    """The fast fp32-accumulate projection stays within the parity bar of the native one."""
    x, r, g, w = make_case(case["M"], case["H"], case["N"], case["dtype"], case["seed"], case["res"])
    a, _ = forward(x, r, g, w, case["eps"], accumulate="native")
    b, _ = forward(x, r, g, w, case["eps"], accumulate="fp32")
    m = parity_metrics(b, a)
    assert m["max_abs"] <= 2e-2 and m["rel_l2"] <= 5e-3, m


def test_identity_projection_gives_equal_qkv():
    """tests/test_correctness.py:142-155: identity weight, unit gain -> Q == K == V."""
    torch.manual_seed(0)
    H = 128
    x = torch.randn(16, H)
    g = torch.ones(H)
    w = torch.eye(H).repeat(3, 1)
    out, _ = forward(x, torch.zeros_like(x), g, w, 1e-6)
    q, k, v = split_qkv(out, H, H)
    torch.testing.assert_close(q, k, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(k, v, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(q, rms_normalize(x, g, 1e-6), atol=1e-5, rtol=1e-5)


def test_zero_residual_has_no_nan():
    """tests/test_correctness.py:127-140."""
    x, _, _, w = make_case(128, 256, 768, torch.float16, 0)
    out, hidden = forward(x, torch.zeros_like(x), torch.ones(256, dtype=torch.float16), w, 1e-6)
    assert not torch.isnan(out).any()
    assert torch.equal(hidden, x)


def test_split_widths_gqa():
    """integration/llama3_patch.py:156-158 and tests/test_correctness.py:327-346."""
    H, H_kv = 512, 128
    x, r, g, w = make_case(4, H, H + 2 * H_kv, torch.bfloat16, 9)
    out, _ = forward(x, r, g, w, 1e-5)
    q, k, v = split_qkv(out, H, H_kv)
    assert q.shape == (4, H) and k.shape == (4, H_kv) and v.shape == (4, H_kv)


def test_residual_add_is_fp32_add_rounded():
    """hidden = RNE_dtype(fp32(x) + fp32(r)): the contract the kernels reproduce bit for bit."""
    for dt in (torch.float16, torch.bfloat16):
        x, r, _, _ = make_case(64, 512, 8, dt, 11)
        hidden, _ = forward(x, r, torch.ones(512, dtype=dt), torch.zeros(8, 512, dtype=dt), 1e-5)[::-1]
        assert torch.equal(hidden, (x.float() + r.float()).to(dt))


def test_parity_metrics():
    a = torch.tensor([1.0, 2.0, 3.0])
    m = parity_metrics(a + torch.tensor([0.0, 0.01, 0.0]), a)
    assert abs(m["max_abs"] - 0.01) < 1e-6 and m["nonfinite"] == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("B,S,n_q,n_kv,d,cb", [(1, 1, 32, 8, 128, 1), (2, 7, 4, 2, 64, 2), (3, 5, 8, 8, 128, 1)])
def test_rope_oracle_matches_transformers(B, S, n_q, n_kv, d, cb, dtype):
    """The Q/K/V split + rotary oracle is bit-identical to transformers' own
    apply_rotary_pos_emb on the same split (llama3_patch.py:156-168)."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

    from oracle import make_rope_case, rope_split

    qkv, cos, sin = make_rope_case(B, S, n_q, n_kv, d, dtype, seed=B * 100 + S, cos_batch=cb)
    q, k, v = rope_split(qkv, cos, sin, n_q, n_kv, d)
    qs, ks, vs = torch.split(qkv, [n_q * d, n_kv * d, n_kv * d], dim=-1)
    qh = qs.reshape(B, S, n_q, d).transpose(1, 2)
    kh = ks.reshape(B, S, n_kv, d).transpose(1, 2)
    qr, kr = apply_rotary_pos_emb(qh, kh, cos.expand(B, S, d), sin.expand(B, S, d))
    assert torch.equal(q, qr) and torch.equal(k, kr)
    assert torch.equal(v, vs.reshape(B, S, n_kv, d).transpose(1, 2))


def test_e4m3_quantizer_round_trip_bound():
    """quantize_weight_e4m3: w8 * scale is w to within e4m3's 3 mantissa bits (relative
    2^-4 for normal values, 2^-10 * scale absolute below the normal range)."""
    from triton_fused_rmsnorm_qkv import quantize_weight_e4m3

    w = (0.02 * torch.randn(64, 256, generator=torch.Generator().manual_seed(4))).bfloat16()
    w[3] = 0  # an all-zero row keeps scale 1
    w8, scale = quantize_weight_e4m3(w)
    assert w8.dtype == torch.float8_e4m3fn and scale.dtype == torch.float32 and scale[3] == 1
    deq = w8.float() * scale[:, None]
    err = (deq - w.float()).abs()
    bound = torch.maximum(w.float().abs() * 2.0 ** -4, scale[:, None] * 2.0 ** -10)
    assert bool((err <= bound).all())
    assert torch.allclose(w8.float().abs().amax(dim=1)[w.float().abs().amax(dim=1) > 0], torch.tensor(448.0))
