"""Sequence sharding across GPUs (one process per GPU) and the output gather.

Sequences (and the masked variants of a mutational scan) are independent forwards, so a batch is
split into contiguous per-rank blocks whose estimated cost is balanced; every rank holds a full
weight replica and the only collective is the gather of the per-sequence outputs. The cost model
counts the projection FLOPs (linear in L) and the attention FLOPs (quadratic in L) of one forward.
"""
from __future__ import annotations

import numpy as np


def forward_cost(length: int, dim: int, hidden_dim: int) -> float:
    """Algorithmic FLOPs of one sequence per layer: projections 2L(4d^2 + 2dF) + attention 4L^2 d."""
    return 2.0 * length * (4 * dim * dim + 2 * dim * hidden_dim) + 4.0 * length * length * dim


def partition(lengths, world: int, dim: int = 1280, hidden_dim: int = 5120) -> list[range]:
    """Contiguous blocks [start, end) of sequence indices, one per rank, with balanced cost.

    Greedy over the prefix sums: rank r ends its block where the cumulative cost first reaches
    (r + 1) / world of the total. Blocks may be empty when there are fewer sequences than ranks.
    """
    lengths = list(lengths)
    if world <= 0:
        raise ValueError("world must be positive")
    cost = np.array([forward_cost(L, dim, hidden_dim) for L in lengths], dtype=np.float64)
    csum = np.concatenate([[0.0], np.cumsum(cost)])
    total = csum[-1]
    bounds = [0]
    for r in range(1, world):
        target = total * r / world
        # first index whose prefix cost reaches the target, never moving backwards
        idx = int(np.searchsorted(csum, target, side="left"))
        idx = min(max(idx, bounds[-1]), len(lengths))
        bounds.append(idx)
    bounds.append(len(lengths))
    return [range(bounds[r], bounds[r + 1]) for r in range(world)]


def gather_rows(local, group=None, dst_all: bool = True):
    """All-gathers a per-rank [n_local, ...] tensor of variable n_local; returns the concatenation
    in rank order (on every rank). Works with NCCL (CUDA tensors) and gloo (CPU tensors)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    n = torch.tensor([local.shape[0]], dtype=torch.int64, device=local.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]
    mx = max(sizes)
    pad = torch.zeros((mx,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], dim=0)
