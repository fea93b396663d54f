"""Head-sharded (column-parallel) layout: shard the packed weight by attention heads,
run the op per rank, all-gather and reassemble [Q | K | V].  Rehearsed on the CPU with
2 gloo ranks, the per-rank op being the oracle (the GPU run uses the CUDA kernels and
NCCL, bench.py --gpus N)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import forward, make_case
from triton_fused_rmsnorm_qkv.sharding import HeadLayout, assemble, gather_qkv, shard_qkv_weight, shard_rows


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_rows_partition_the_weight():
    lay = HeadLayout(32, 8, 128)
    for world in (1, 2, 4, 8):
        rows = torch.cat([shard_rows(lay, r, world) for r in range(world)])
        assert sorted(rows.tolist()) == list(range(lay.n_out))
        assert all(len(shard_rows(lay, r, world)) == lay.n_out // world for r in range(world))


def test_assemble_inverts_sharding():
    lay = HeadLayout(4, 2, 8)
    full = torch.arange(3 * lay.n_out, dtype=torch.float32).reshape(3, lay.n_out)
    for world in (1, 2):
        parts = [full[:, shard_rows(lay, r, world)] for r in range(world)]
        assert torch.equal(assemble(parts, lay), full)


def test_bad_head_split_is_rejected():
    with pytest.raises(ValueError):
        HeadLayout(32, 8, 128).local(3)


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lay = HeadLayout(4, 2, 64)  # H = 256, N = 512 (the CPU-ref config's heads)
        x, r, g, w = make_case(4, 256, lay.n_out, torch.float32, seed=1)
        w_local = shard_qkv_weight(w, lay, rank, world)
        out_local, hidden = forward(x, r, g, w_local, 1e-5)
        full = gather_qkv(out_local, lay)
        if rank == 0:
            ref, ref_hidden = forward(x, r, g, w, 1e-5)
            result_q.put((float((full - ref).abs().max()), bool(torch.equal(hidden, ref_hidden))))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_gather_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(rk, 2, port, q)) for rk in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    max_diff, hidden_equal = q.get(timeout=10)
    assert max_diff < 1e-5 and hidden_equal
