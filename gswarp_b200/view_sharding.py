"""Multi-view data parallelism for the 3DGS training step.

Views are independent, so they shard across ranks (one process per GPU,
``torch.distributed`` over NCCL): every rank holds a full replica of the
Gaussians, renders its own contiguous block of views, accumulates every
view's per-Gaussian gradients into one contiguous fp32 buffer and then takes
part in ONE all-reduce (sum) of that buffer -- the only exchange of the step.
The buffer is laid out in SoA blocks ``[means | scales | rotations |
opacities | SH]`` (59 floats per Gaussian at SH degree 3), so each parameter's
``.grad`` is a contiguous view into it and autograd accumulates in place.
Screen-space (means2D) gradients and radii stay rank-local.

The per-view work is a callable, so the host logic (sharding, accumulation,
all-reduce, max-over-ranks timing, failure propagation) is exercised on CPU
with gloo ranks in the tests, and on GPUs with the native rasterizer.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch


def shard_views(num_views: int, world: int, rank: int) -> range:
    """Contiguous block of view indices owned by ``rank`` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} for world size {world}")
    base, extra = divmod(num_views, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


class GradientBuffer:
    """One flat fp32 buffer whose SoA blocks are the parameters' ``.grad``."""

    def __init__(self, params: Sequence[torch.Tensor]):
        if not params:
            raise ValueError("no parameters")
        dev = params[0].device
        total = sum(p.numel() for p in params)
        self.flat = torch.zeros(total, dtype=torch.float32, device=dev)
        self.params = list(params)
        self.views = []
        off = 0
        for p in self.params:
            n = p.numel()
            self.views.append(self.flat[off:off + n].view_as(p))
            off += n
        self.attach()

    def attach(self) -> None:
        for p, v in zip(self.params, self.views):
            p.grad = v

    def zero_(self) -> None:
        self.flat.zero_()
        self.attach()

    def detach(self) -> None:
        """Unset every parameter's ``.grad``: the next backward stores its
        gradients as fresh tensors instead of adding them into the buffer."""
        for p in self.params:
            p.grad = None

    def take(self) -> None:
        """After one backward since :meth:`detach`: copy each parameter's
        ``.grad`` into its block (zero for a parameter that received none) and
        attach the blocks again.  The buffer then holds that backward's
        gradients -- one copy, where zeroing the buffer and accumulating into
        it reads and writes it twice more."""
        for p, v in zip(self.params, self.views):
            if p.grad is None:
                v.zero_()
            elif p.grad.data_ptr() != v.data_ptr():
                v.copy_(p.grad)
        self.attach()

    def all_reduce(self, group=None) -> None:
        if torch.distributed.is_available() and torch.distributed.is_initialized():
            if torch.distributed.get_world_size(group) > 1:
                torch.distributed.all_reduce(self.flat, group=group)

    @property
    def floats_per_item(self) -> int:
        n = self.params[0].shape[0]
        return self.flat.numel() // n if n else 0


@dataclass
class StepResult:
    losses: list
    views: int


class ViewShardedStep:
    """One data-parallel training step over this rank's views.

    ``view_fn(view_index) -> loss`` runs forward, builds the loss and returns
    it; ``step`` calls ``backward`` on each loss (gradients land in the flat
    buffer) and finishes with the all-reduce."""

    def __init__(self, params: Sequence[torch.Tensor], view_indices: Sequence[int],
                 view_fn: Callable[[int], torch.Tensor], group=None):
        self.grads = GradientBuffer(params)
        self.view_indices = list(view_indices)
        self.view_fn = view_fn
        self.group = group

    def step(self) -> StepResult:
        losses = []
        if not self.view_indices:
            self.grads.zero_()
        for n, i in enumerate(self.view_indices):
            loss = self.view_fn(i)
            if n == 0:
                # the first view's gradients are copied into the buffer rather
                # than added to a zero-filled one
                self.grads.detach()
                try:
                    loss.backward()
                finally:
                    self.grads.take()
            else:
                loss.backward()
            losses.append(loss.detach())
        self.grads.all_reduce(self.group)
        return StepResult(losses=losses, views=len(self.view_indices))


def max_over_ranks(value: float, device=None, group=None) -> float:
    """Max of a per-rank scalar (e.g. elapsed milliseconds) across ranks."""
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return float(value)
    if torch.distributed.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
    return float(t.item())
