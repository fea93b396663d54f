"""Head-sharded (Megatron column-parallel) layout of the packed QKV projection.

The reference is single-GPU (README.md:27); this module adds the partitioning the
multi-GPU configs use.  Rank p of P owns query heads [p*n_q/P, (p+1)*n_q/P) and
key/value heads [p*n_kv/P, (p+1)*n_kv/P) of the packed weight
``[Wq (n_q*d rows); Wk (n_kv*d); Wv (n_kv*d)]`` (integration/llama3_patch.py:111-127).
Its local weight is the contiguous ``[Wq_p; Wk_p; Wv_p]`` with N/P rows, so the fused
op runs unchanged on each rank with replicated x / residual / gain and produces a
head-sharded ``[q_p | k_p | v_p]`` output.  There is no exchange step in the op
itself; ``gather_qkv`` (an all-gather) reassembles the global ``[Q | K | V]`` only to
verify a sharded run against the unsharded one.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadLayout:
    n_q: int      # query heads
    n_kv: int     # key/value heads
    d: int        # head dimension

    @property
    def h_q(self) -> int:
        return self.n_q * self.d

    @property
    def h_kv(self) -> int:
        return self.n_kv * self.d

    @property
    def n_out(self) -> int:
        return self.h_q + 2 * self.h_kv

    def check(self, world: int) -> None:
        if self.n_q % world or self.n_kv % world:
            raise ValueError(f"{self.n_q} q / {self.n_kv} kv heads do not split over {world} ranks")

    def local(self, world: int) -> "HeadLayout":
        self.check(world)
        return HeadLayout(self.n_q // world, self.n_kv // world, self.d)


def shard_rows(layout: HeadLayout, rank: int, world: int) -> torch.Tensor:
    """Row indices of the global packed weight owned by ``rank`` (in local order)."""
    loc = layout.local(world)
    q0 = rank * loc.h_q
    k0 = layout.h_q + rank * loc.h_kv
    v0 = layout.h_q + layout.h_kv + rank * loc.h_kv
    return torch.cat([torch.arange(q0, q0 + loc.h_q), torch.arange(k0, k0 + loc.h_kv),
                      torch.arange(v0, v0 + loc.h_kv)])


def shard_qkv_weight(weight: torch.Tensor, layout: HeadLayout, rank: int, world: int) -> torch.Tensor:
    """Contiguous local weight ``[Wq_p; Wk_p; Wv_p]`` of shape (N / world, H)."""
    if weight.shape[0] != layout.n_out:
        raise ValueError(f"weight has {weight.shape[0]} rows, layout needs {layout.n_out}")
    idx = shard_rows(layout, rank, world).to(weight.device)
    return weight.index_select(0, idx).contiguous()


def assemble(parts: list[torch.Tensor], layout: HeadLayout) -> torch.Tensor:
    """Global ``[Q | K | V]`` (..., N) from the per-rank ``[q_p | k_p | v_p]`` outputs."""
    world = len(parts)
    loc = layout.local(world)
    qs = [p[..., :loc.h_q] for p in parts]
    ks = [p[..., loc.h_q:loc.h_q + loc.h_kv] for p in parts]
    vs = [p[..., loc.h_q + loc.h_kv:] for p in parts]
    return torch.cat(qs + ks + vs, dim=-1)


def gather_qkv(local_out: torch.Tensor, layout: HeadLayout, group=None) -> torch.Tensor:
    """All-gather the head-sharded outputs of every rank and reassemble [Q | K | V].

    Uses ``torch.distributed.all_gather`` (NCCL over NVLink on GPUs, gloo on CPU).
    Verification only: the fused op itself needs no communication.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    parts = [torch.empty_like(local_out) for _ in range(world)]
    dist.all_gather(parts, local_out.contiguous(), group=group)
    return assemble(parts, layout)
