"""The grid decode schedule: the fused decode kernel without clusters.

Every CTA forms the whole activation rows and their RMS itself, the K split of each tile
group runs on independent CTAs, and the CTA that arrives last on the group's counter sums
the partial tiles in rank order through a zero-filled workspace.  Checked against the
CPU oracle (restated baseline.py) with the benchmark bars -- Q/K/V max-abs error <= 2e-2
(1 ulp of the reference above |x| = 4 for bf16) and relative L2 error <= 5e-3, the
updated residual bit-exact -- and for what is particular to it: repeated launches give
identical bits and leave the arrival counters at zero, the automatic choice (taken at M = 1
for the Qwen2-7B shape, not for Llama-3-8B or above two rows), ragged K and N, row-strided
inputs.
"""
from __future__ import annotations

import pytest
import torch

from oracle import faithful_rounding_metrics, forward, make_case, parity_metrics, rms_normalize, within_bars
from triton_fused_rmsnorm_qkv import _lib, device_status, fused_add_rmsnorm_matmul, get_autotune_best_config
from triton_fused_rmsnorm_qkv import kernel as fk

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 5e-3


def check(out, hidden, x, r, g, w, eps):
    ref_out, ref_hidden = forward(x, r, g, w, eps)
    m = parity_metrics(out, ref_out)
    assert within_bars(m, MAX_ABS, REL_L2), m
    exact = torch.nn.functional.linear(rms_normalize(ref_hidden, g, eps).float(), w.float())
    f = faithful_rounding_metrics(out, exact)
    assert f["n_bad"] == 0, f
    assert torch.equal(hidden, ref_hidden), "updated residual is not bit-exact"
    return m


def run_grid(M, H, N, dtype=torch.bfloat16, seed=0, res=True, eps=1e-5, schedule="grid"):
    x, r, g, w = make_case(M, H, N, dtype, seed, res)
    out, hidden = fused_add_rmsnorm_matmul(x.cuda()[None], r.cuda()[None] if r is not None else None, g.cuda(),
                                           w.cuda(), eps, schedule=schedule)
    torch.cuda.synchronize()
    m = check(out[0].cpu(), hidden[0].cpu(), x, r, g, w, eps)
    assert device_status() == 0
    print(f"grid M={M} H={H} N={N} {dtype}: {m} {_lib.query_schedule(M, H, N, _lib.BF16, _lib.SCHED_GRID)}")
    return out[0].cpu(), hidden[0].cpu()


def counters_zero() -> bool:
    """Every grid workspace's arrival counters (its first 4096 bytes) are zero."""
    torch.cuda.synchronize()
    return all(int(buf[:4096].count_nonzero()) == 0 for buf in fk._grid_ws.values())


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
def test_llama3_8b_rows(M, dtype):
    run_grid(M, 4096, 6144, dtype, seed=700 + M)


@pytest.mark.parametrize("H,N", [(3584, 4608), (8192, 10240), (4096, 28672), (4096, 3072), (8192, 1280)],
                         ids=["qwen2", "llama70b", "gate_up", "tp2", "70b_tp8"])
@pytest.mark.parametrize("M", [1, 4])
def test_model_shapes(M, H, N):
    """Shapes whose best grid configuration takes 1, 4 or 5 tiles of 128 rows per CTA."""
    run_grid(M, H, N, seed=710 + M + N % 97)


@pytest.mark.parametrize("H,N", [(4104, 6144), (4096, 6000), (256, 512), (1032, 392)],
                         ids=["ragged_k", "ragged_n", "small", "ragged_both"])
@pytest.mark.parametrize("res", [False, True], ids=["R0", "R1"])
def test_ragged_shapes(H, N, res):
    """K not a multiple of 64 (the slice of the last CTA runs past the row), N not a
    multiple of 128 (the last tile group is partly outside the weight), no residual."""
    run_grid(3, H, N, seed=720 + H + N, res=res)


def test_repeated_launches_are_identical_and_reset_counters():
    """Five launches on the same inputs: identical bits (the rank-order sum does not depend
    on which CTA arrives last), and the arrival counters are back at zero after each."""
    M, H, N = 2, 4096, 6144
    x, r, g, w = make_case(M, H, N, torch.bfloat16, 731, True)
    xd, rd, gd, wd = x.cuda()[None], r.cuda()[None], g.cuda(), w.cuda()
    first = hid = None
    for _ in range(5):
        out, hidden = fused_add_rmsnorm_matmul(xd, rd, gd, wd, 1e-5, schedule="grid")
        assert counters_zero()
        if first is None:
            first, hid = out.clone(), hidden.clone()
        assert torch.equal(out, first) and torch.equal(hidden, hid)
    check(first[0].cpu(), hid[0].cpu(), x, r, g, w, 1e-5)
    ref, _ = fused_add_rmsnorm_matmul(xd, rd, gd, wd, 1e-5, schedule="decode")
    m = parity_metrics(first[0].cpu(), ref[0].cpu())
    assert within_bars(m, MAX_ABS, REL_L2), m


def test_alternating_shapes_share_one_workspace():
    """Different shapes on one stream reuse (and grow) the same zero-filled workspace."""
    for M, H, N in [(1, 4096, 6144), (4, 8192, 10240), (2, 4096, 6144), (8, 3584, 4608), (1, 4096, 6144)]:
        run_grid(M, H, N, seed=740 + M)
        assert counters_zero()


def test_row_strided_inputs():
    """x, residual and the outputs as rows of wider buffers (row strides != H)."""
    M, H, N = 4, 4096, 6144
    x, r, g, w = make_case(M, H, N, torch.bfloat16, 750, True)
    xb = torch.zeros(M, H + 64, dtype=x.dtype, device="cuda")
    rb = torch.zeros(M, H + 128, dtype=x.dtype, device="cuda")
    ob = torch.full((M, N + 64), 7.0, dtype=x.dtype, device="cuda")
    hb = torch.full((M, H + 64), 7.0, dtype=x.dtype, device="cuda")
    xb[:, :H] = x.cuda()
    rb[:, :H] = r.cuda()
    gd, wd = g.cuda(), w.cuda()
    stream = fk._current_stream(0)
    ws_bytes = _lib.workspace_bytes(M, H, N, _lib.BF16, _lib.SCHED_GRID)
    ws = fk._grid_workspace(0, stream, ws_bytes, torch.device("cuda", 0))
    rc = _lib.launch(xb.data_ptr(), rb.data_ptr(), gd.data_ptr(), _lib.BF16, wd.data_ptr(), ob.data_ptr(),
                     hb.data_ptr(), M, H, N, H + 64, H + 128, H, N + 64, H + 64, 1e-5, _lib.BF16, _lib.SCHED_GRID, 0,
                     ws.data_ptr(), ws_bytes, stream)
    _lib.check(rc)
    torch.cuda.synchronize()
    check(ob[:, :N].cpu(), hb[:, :H].cpu(), x, r, g, w, 1e-5)
    assert torch.all(ob[:, N:] == 7.0) and torch.all(hb[:, H:] == 7.0), "wrote outside the rows"
    assert counters_zero()


def test_automatic_choice():
    """On a full B200 (148 SMs) the model shapes keep the cluster kernel at one and two rows:
    the grid variant's 14 k-blocks per CTA on 144 CTAs against 20 on the cluster kernel's 108
    (Qwen2-7B) is not the 0.6 the rule asks for, nor is Llama-3-8B's 22 against 26; and every
    shape above two rows keeps it as well."""
    run_grid(1, 3584, 4608, seed=760, schedule=None)
    run_grid(1, 4096, 6144, seed=761, schedule=None)
    qwen, llama = get_autotune_best_config(1, 3584), get_autotune_best_config(1, 4096)
    print(qwen, llama)
    if torch.cuda.get_device_properties(0).multi_processor_count >= 148:
        assert qwen["schedule"] == "decode"
        assert llama["schedule"] == "decode"
    run_grid(4, 3584, 4608, seed=762, schedule=None)
    assert get_autotune_best_config(4, 3584)["schedule"] == "decode"


def test_grid_under_graph_capture():
    """The grid schedule inside CUDA graph captures: each capture keeps its own zero-filled
    counters (zeroed by its own replays), so two graphs captured on the same stream, replayed
    in reverse order, and an eager call afterwards all match the oracle and leave their
    counters at zero."""
    M, H, N, eps = 1, 3584, 4608, 1e-6
    cases = [make_case(M, H, N, torch.bfloat16, seed=900 + i) for i in range(3)]
    dev = [tuple(t.cuda() for t in c) for c in cases]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graphs, outs = [], []
    with torch.cuda.stream(side):
        for i in range(2):
            x, r, g, w = dev[i]
            fused_add_rmsnorm_matmul(x[None], r[None], g, w, eps, schedule="grid")  # warm-up outside the capture
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=side):
                outs.append(fused_add_rmsnorm_matmul(x[None], r[None], g, w, eps, schedule="grid"))
            graphs.append(gr)
    torch.cuda.synchronize()
    for i in (1, 0):
        for o in outs[i]:
            o.zero_()
        graphs[i].replay()
        torch.cuda.synchronize()
        check(outs[i][0][0].cpu(), outs[i][1][0].cpu(), *cases[i], eps)
    x, r, g, w = dev[2]
    out, hidden = fused_add_rmsnorm_matmul(x[None], r[None], g, w, eps, schedule="grid")
    torch.cuda.synchronize()
    check(out[0].cpu(), hidden[0].cpu(), *cases[2], eps)
    assert counters_zero()
    assert all(int(buf[:4096].count_nonzero()) == 0 for buf in fk._grid_ws_capture.values())
    assert device_status() == 0
    del graphs
