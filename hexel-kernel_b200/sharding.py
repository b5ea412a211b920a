"""Multi-GPU partitioning of the rasteriser workloads (one process per GPU).

* 3D multi-view: views are dealt round-robin (rank g renders the views
  v = g (mod world)), or by measured cost (balance_views); surfels are
  replicated and each rank sums its views' per-surfel gradients into one
  flat buffer, all-reduced once per step.
* 2D Image-GS: horizontal stripes of 16-pixel tile rows, rank g renders
  rows [tiles_y g / world, tiles_y (g+1) / world); Gaussians are replicated
  and their gradients all-reduced.

Nothing here touches another GPU's memory: the only exchange is the NCCL (or
gloo) all-reduce of the gradient buffer.
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch


def view_split(num_views: int, world: int, rank: int) -> List[int]:
    """Views of `rank`: v = rank, rank + world, ..."""
    return [v for v in range(num_views) if v % world == rank]


def balance_views(costs: Sequence[float], world: int) -> List[List[int]]:
    """Views dealt to `world` ranks by cost, longest first, each to the rank
    with the least cost so far (ties: lower rank; equal costs: lower view
    index first).  Deterministic, so every rank computes the same split from
    the same cost vector.  Returns each rank's views in ascending order."""
    order = sorted(range(len(costs)), key=lambda v: (-float(costs[v]), v))
    loads = [0.0] * world
    out: List[List[int]] = [[] for _ in range(world)]
    for v in order:
        r = min(range(world), key=lambda i: (loads[i], i))
        out[r].append(v)
        loads[r] += float(costs[v])
    return [sorted(x) for x in out]


def stripe_rows(tiles_y: int, world: int, rank: int) -> Optional[Tuple[int, int]]:
    """Tile rows [r0, r1) of `rank`'s stripe, or None for a single rank."""
    if world == 1:
        return None
    return (tiles_y * rank // world, tiles_y * (rank + 1) // world)


class GradBuffer:
    """One flat float32 buffer holding a gradient per parameter (views of
    the parameters' shapes, each starting on a 16-byte boundary) and a loss
    slot: zeroed with one fill and all-reduced in place."""

    def __init__(self, shapes: Sequence[Sequence[int]], device):
        sizes = [int(torch.Size(s).numel()) for s in shapes]
        padded = [(n + 3) // 4 * 4 for n in sizes]
        self.flat = torch.zeros(sum(padded) + 4, dtype=torch.float32, device=device)
        self.views, o = [], 0
        for s, n, pn in zip(shapes, sizes, padded):
            self.views.append(self.flat[o:o + n].view(*s))
            o += pn
        self.loss = self.flat[o:o + 1]

    def zero_(self) -> None:
        self.flat.zero_()

    def all_reduce_(self, world: int) -> None:
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(self.flat)
