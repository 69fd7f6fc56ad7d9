"""Multi-GPU partitioning of one grouped convolution.

Outputs shard exactly like inputs, so the only split needed is of the work:
no collective is on the data path.  A rank's share is a list of units; each
unit is a sub-problem the unchanged C ABI can run as one call on pointer
offsets into the full tensors:

  * by batch (N >= world size): images [n0, n1) of every channel - the
    sub-tensors x[n0:n1], y[n0:n1] are contiguous, weights are whole;
  * by group block (N < world size): one image, channels [c0, c1) made of
    whole groups - x[n, c0:c1], y[n, c0:c1] and w[c0:c1] are contiguous.

``units_for_rank`` balances units so ranks differ by at most one image (batch)
or one group block.  ``max_over_ranks`` is the timing reduction: the job
takes as long as its slowest rank.
"""
from __future__ import annotations

import dataclasses
import math

from .api import Shape


@dataclasses.dataclass(frozen=True)
class Unit:
    n0: int
    n1: int
    c0: int
    c1: int

    def shape(self, full: Shape) -> Shape:
        c = self.c1 - self.c0
        return dataclasses.replace(full, n=self.n1 - self.n0, cin=c, cout=c,
                                   groups=c // (full.cin // full.groups))

    def offsets(self, full: Shape):
        """Element offsets of this unit's x, w, y inside the full tensors."""
        _, c, ho, wo = full.output
        hw = full.h * full.w
        x = (self.n0 * full.cin + self.c0) * hw
        y = (self.n0 * c + self.c0) * ho * wo
        w = self.c0 * (full.cin // full.groups) * full.r * full.s
        return x, w, y

    def images(self):
        return self.n1 - self.n0


def _split(total, parts, index):
    """Contiguous [lo, hi) of `total` items for part `index` of `parts`."""
    base, extra = divmod(total, parts)
    lo = index * base + min(index, extra)
    return lo, lo + base + (1 if index < extra else 0)


def units_for_rank(shape: Shape, world: int, rank: int) -> list[Unit]:
    if not (shape.cin == shape.cout):
        raise ValueError('group-block sharding needs Cin == Cout')
    if world < 1 or not 0 <= rank < world:
        raise ValueError('bad world size or rank')
    if shape.n >= world:
        n0, n1 = _split(shape.n, world, rank)
        return [Unit(n0, n1, 0, shape.cin)]
    # Fewer images than ranks: split each image into group blocks so that
    # there are at least `world` units, then hand contiguous runs of units out.
    cpg = shape.cin // shape.groups
    blocks = min(shape.groups, math.ceil(world / shape.n))
    while shape.groups % blocks:
        blocks += 1
    per = shape.groups // blocks
    all_units = [Unit(n, n + 1, b * per * cpg, (b + 1) * per * cpg)
                 for n in range(shape.n) for b in range(blocks)]
    lo, hi = _split(len(all_units), world, rank)
    return all_units[lo:hi]


def max_over_ranks(value: float, group=None) -> float:
    """All ranks receive the maximum of `value` (a duration) across ranks."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    backend = dist.get_backend(group)
    device = f'cuda:{torch.cuda.current_device()}' if backend == 'nccl' else 'cpu'
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def sum_over_ranks(value: float, group=None) -> float:
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    backend = dist.get_backend(group)
    device = f'cuda:{torch.cuda.current_device()}' if backend == 'nccl' else 'cpu'
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return float(t.item())
