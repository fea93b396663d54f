"""qkv_rope_split (one CUDA launch: head-major Q/K/V with the rotary embedding on Q and K)
against the CPU oracle and transformers' apply_rotary_pos_emb: bit-exact."""
from __future__ import annotations

import pytest
import torch

from oracle import make_rope_case, rope_split
from triton_fused_rmsnorm_qkv import qkv_rope_split

pytestmark = pytest.mark.gpu

CASES = [  # B, S, n_q, n_kv, head_dim, cos batch rows
    (1, 1, 32, 8, 128, 1),     # Llama-3-8B decode
    (2, 7, 4, 2, 64, 2),       # per-batch positions
    (3, 5, 8, 8, 128, 1),      # MHA
    (4, 33, 32, 8, 128, 4),
    (1, 300, 28, 4, 128, 1),   # Qwen2-7B heads, prefill
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("B,S,n_q,n_kv,d,cb", CASES, ids=[f"B{c[0]}_S{c[1]}_q{c[2]}_kv{c[3]}_d{c[4]}" for c in CASES])
def test_rope_split_bit_exact(B, S, n_q, n_kv, d, cb, dtype):
    qkv, cos, sin = make_rope_case(B, S, n_q, n_kv, d, dtype, seed=7 * B + S, cos_batch=cb)
    q, k, v = qkv_rope_split(qkv.cuda(), cos.cuda(), sin.cuda(), n_q, n_kv, d)
    torch.cuda.synchronize()
    rq, rk, rv = rope_split(qkv, cos, sin, n_q, n_kv, d)
    assert q.shape == (B, n_q, S, d) and k.shape == v.shape == (B, n_kv, S, d) and q.is_contiguous()
    assert torch.equal(q.cpu(), rq) and torch.equal(k.cpu(), rk) and torch.equal(v.cpu(), rv)


def test_rope_split_matches_transformers_on_gpu():
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

    B, S, n_q, n_kv, d = 2, 9, 32, 8, 128
    qkv, cos, sin = make_rope_case(B, S, n_q, n_kv, d, torch.bfloat16, seed=3, cos_batch=B)
    qkv, cos, sin = qkv.cuda(), cos.cuda(), sin.cuda()
    q, k, v = qkv_rope_split(qkv, cos, sin, n_q, n_kv, d)
    qs, ks, vs = torch.split(qkv, [n_q * d, n_kv * d, n_kv * d], dim=-1)
    qr, kr = apply_rotary_pos_emb(qs.reshape(B, S, n_q, d).transpose(1, 2), ks.reshape(B, S, n_kv, d).transpose(1, 2),
                                  cos, sin)
    assert torch.equal(q, qr) and torch.equal(k, kr)
    assert torch.equal(v, vs.reshape(B, S, n_kv, d).transpose(1, 2))


def test_rope_split_strided_rows_and_2d_tables():
    """qkv rows inside a wider buffer (row stride > width) and cos / sin given as (S, d)."""
    B, S, n_q, n_kv, d = 2, 6, 8, 2, 128
    qkv, cos, sin = make_rope_case(B, S, n_q, n_kv, d, torch.bfloat16, seed=11)
    W = qkv.shape[-1]
    wide = torch.zeros(B, S, W + 64, dtype=qkv.dtype, device="cuda")
    wide[..., :W] = qkv.cuda()
    q, k, v = qkv_rope_split(wide[..., :W], cos[0].cuda(), sin[0].cuda(), n_q, n_kv, d)
    rq, rk, rv = rope_split(qkv, cos, sin, n_q, n_kv, d)
    assert torch.equal(q.cpu(), rq) and torch.equal(k.cpu(), rk) and torch.equal(v.cpu(), rv)


def test_rope_split_argument_errors():
    qkv = torch.zeros(1, 2, 6 * 64, dtype=torch.bfloat16, device="cuda")
    cs = torch.zeros(1, 2, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        qkv_rope_split(qkv, cs, cs, 4, 2, 48)                 # width is not (4 + 4) * 48
    with pytest.raises(TypeError):
        qkv_rope_split(qkv, cs.float(), cs, 2, 2)             # cos in another dtype
    with pytest.raises(ValueError):
        qkv_rope_split(qkv, cs[:, :1], cs[:, :1], 2, 2)       # cos for another sequence length


# ---------------------------------------------------------------- the rotary split fused into the op
from oracle import forward, make_case, parity_metrics, within_bars  # noqa: E402
from triton_fused_rmsnorm_qkv import fused_add_rmsnorm_matmul, fused_add_rmsnorm_qkv_rope  # noqa: E402

FUSED_CASES = [  # B, S, H, n_q, n_kv, d, cos batch rows
    (1, 1, 4096, 32, 8, 128, 1),    # Llama-3-8B decode, M = 1
    (16, 1, 4096, 32, 8, 128, 16),  # M = 16, a position per sequence
    (4, 4, 4096, 32, 8, 128, 1),    # M = 16 as 4 x 4
    (64, 1, 4096, 32, 8, 128, 64),  # M = 64: the projection and the split run as two launches
    (3, 2, 1024, 8, 2, 64, 3),      # head_dim 64: two heads per 128-row tile
    (2, 5, 3584, 28, 4, 128, 1),    # Qwen2-7B heads, M = 10
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("res", [True, False], ids=["res", "nores"])
@pytest.mark.parametrize("B,S,H,n_q,n_kv,d,cb", FUSED_CASES,
                         ids=[f"B{c[0]}_S{c[1]}_H{c[2]}_d{c[5]}" for c in FUSED_CASES])
def test_fused_qkv_rope_matches_the_two_launches(B, S, H, n_q, n_kv, d, cb, dtype, res):
    """fused_add_rmsnorm_qkv_rope is bit-identical to the fused projection followed by the
    rotary split (and so to oracle/rope.py on that projection), and its projection meets the
    parity bars against the CPU oracle."""
    M, N = B * S, (n_q + 2 * n_kv) * d
    xc, rc_, gc, wc = make_case(M, H, N, dtype, seed=300 + M + d, has_residual=res)
    _, cos, sin = make_rope_case(B, S, n_q, n_kv, d, dtype, seed=5, cos_batch=cb)
    x = xc.cuda().view(B, S, H)
    r = rc_.cuda().view(B, S, H) if res else None
    g, w, cs, sn = gc.cuda(), wc.cuda(), cos.cuda(), sin.cuda()
    q, k, v, hidden = fused_add_rmsnorm_qkv_rope(x, r, g, w, cs, sn, n_q, n_kv, d, 1e-5)
    out, hid2 = fused_add_rmsnorm_matmul(x, r, g, w, 1e-5)
    rq, rk, rv = qkv_rope_split(out, cs, sn, n_q, n_kv, d)
    torch.cuda.synchronize()
    assert q.shape == (B, n_q, S, d) and k.shape == v.shape == (B, n_kv, S, d)
    assert torch.equal(q, rq) and torch.equal(k, rk) and torch.equal(v, rv)
    assert torch.equal(hidden, hid2)
    oq, ok_, ov = rope_split(out.cpu(), cos, sin, n_q, n_kv, d)   # the oracle's rotary split
    assert torch.equal(q.cpu(), oq) and torch.equal(k.cpu(), ok_) and torch.equal(v.cpu(), ov)
    ref_out, ref_hidden = forward(xc, rc_, gc, wc, 1e-5)
    m = parity_metrics(out.reshape(M, N).cpu(), ref_out)
    assert within_bars(m), m
    assert torch.equal(hidden.reshape(M, H).cpu(), ref_hidden)
