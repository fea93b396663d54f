"""The keyword-only ``out=`` / ``residual_out=`` destinations of the public calls: the
results written into caller-owned tensors (here views into one buffer, as a caller that
moves a step's results with one copy would hold them) equal the allocating calls' bit for
bit, and a destination of the wrong shape, dtype or layout is rejected before any launch."""
from __future__ import annotations

import pytest
import torch

from oracle import make_case
from triton_fused_rmsnorm_qkv import fused_add_rmsnorm_matmul, fused_rmsnorm_residual_matmul

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,H,N", [(1, 4096, 6144), (16, 4096, 6144), (64, 1024, 1536), (300, 1024, 1280)])
def test_out_views_match_allocating_calls(M, H, N):
    xc, rc_, gc, wc = make_case(M, H, N, torch.bfloat16, seed=5)
    x, r, g, w = (t.cuda() for t in (xc, rc_, gc, wc))
    x3, r3 = x.view(1, M, H), r.view(1, M, H)
    ref_out, ref_hid = fused_add_rmsnorm_matmul(x3, r3, g, w, 1e-5)
    buf = torch.full((M * N + M * H,), float("nan"), dtype=torch.bfloat16, device="cuda")
    out_v, hid_v = buf[:M * N].view(1, M, N), buf[M * N:].view(1, M, H)
    out, hid = fused_add_rmsnorm_matmul(x3, r3, g, w, 1e-5, out=out_v, residual_out=hid_v)
    torch.cuda.synchronize()
    assert out.data_ptr() == out_v.data_ptr() and hid.data_ptr() == hid_v.data_ptr()
    assert torch.equal(out, ref_out) and torch.equal(hid, ref_hid)
    out2 = torch.empty(1, M, N, dtype=torch.bfloat16, device="cuda")
    res = fused_rmsnorm_residual_matmul(x3, r3, g, w, 1e-5, out=out2)
    torch.cuda.synchronize()
    assert res.data_ptr() == out2.data_ptr() and torch.equal(out2, ref_out)


def test_bad_out_is_rejected():
    M, H, N = 4, 1024, 1536
    xc, rc_, gc, wc = make_case(M, H, N, torch.bfloat16, seed=6)
    x, r, g, w = xc.cuda().view(1, M, H), rc_.cuda().view(1, M, H), gc.cuda(), wc.cuda()
    for bad in (torch.empty(1, M, N + 1, dtype=torch.bfloat16, device="cuda"),
                torch.empty(1, M, N, dtype=torch.float16, device="cuda"),
                torch.empty(1, N, M, dtype=torch.bfloat16, device="cuda").transpose(1, 2)):
        with pytest.raises(ValueError):
            fused_rmsnorm_residual_matmul(x, r, g, w, 1e-5, out=bad)
