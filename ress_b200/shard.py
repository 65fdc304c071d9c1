"""Splitting one sparse global-attention layer across the GPUs of a node.

Every stage of the layer is independent per attention head except the HeSS
budget (budget/_proportional.py:149-215), which re-allocates the baseline
counts of all heads of a q-block column.  Heads are therefore split evenly
across ranks, and the only exchange is an all-gather of the (B, H/N, nq)
int32 baselines before ``ress_hess_adjust``, which then runs redundantly on
every rank over all heads (it is tiny).  The gather uses the list form of
``all_gather`` so the same code runs on NCCL and on gloo (CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .layer import HeadShard


def head_range(n_heads: int, world: int, rank: int):
    if n_heads % world:
        raise ValueError(f"{n_heads} heads do not split evenly over {world} ranks")
    hl = n_heads // world
    return rank * hl, hl


def make_gather(world: int, group=None):
    """base (B, H_local, nq) int32 -> (B, world * H_local, nq), rank order."""
    def gather(base: torch.Tensor) -> torch.Tensor:
        parts = [torch.empty_like(base) for _ in range(world)]
        dist.all_gather(parts, base.contiguous(), group=group)
        return torch.cat(parts, dim=1)
    return gather


def make_head_shard(n_heads: int, world: int, rank: int, group=None) -> HeadShard:
    h0, _ = head_range(n_heads, world, rank)
    return HeadShard(h0=h0, h_total=n_heads, gather=make_gather(world, group))
