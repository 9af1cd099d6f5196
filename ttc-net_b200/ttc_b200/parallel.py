"""Batch-sharded data parallelism for TTCLayer (one process per GPU).

TTC rows never interact (every (row, head) LQR problem is independent,
ttc/layers/ttc_layer.py:104-150), so the batch splits across ranks with no traffic inside
the solve.  The only exchange is one all-reduce (SUM) of the parameter gradients after
backward, which makes the per-rank gradients equal to those of the whole global batch.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_rows(x: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """Contiguous, even split of `x` along `dim`; rank r gets block r."""
    n = x.shape[dim]
    if n % world:
        raise ValueError(f"batch dim {n} is not divisible by world size {world}")
    step = n // world
    return x.narrow(dim, rank * step, step)


def allreduce_grads(module: torch.nn.Module, group=None) -> None:
    """Sum the parameter gradients over all ranks in one flat bucket (a single collective).
    Parameters without a gradient take part as zeros so every rank issues the same call."""
    params = [p for p in module.parameters() if p.requires_grad]
    if not params:
        return
    flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1)
                      for p in params])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    off = 0
    for p in params:
        n = p.numel()
        g = flat[off:off + n].view_as(p)
        if p.grad is None:
            p.grad = g.clone()
        else:
            p.grad.copy_(g)
        off += n


class OverlappedGradAllReduce:
    """All-reduce (SUM) of each parameter's gradient started as soon as that gradient is
    final, so the collectives overlap the rest of the backward (for TTCLayer: out_proj's and
    the bases' gradients go out while the prologue and in_proj backward still run).

    ``arm()`` before the backward that completes the gradients (the last micro-batch of
    ``TTCLayer.forward_backward``), ``wait()`` after it.  Every rank arms and waits at the same
    points; the hooks fire in the autograd order of the same graph, so all ranks issue the same
    collectives in the same order.  A parameter the backward leaves without a gradient is
    all-reduced as zeros in ``wait()``, after the others, so that every rank still issues it."""

    def __init__(self, module: torch.nn.Module, group=None):
        self.params = [p for p in module.parameters() if p.requires_grad]
        self.group = group
        self.handles = []
        self.works = []
        self.done = set()

    def _hook(self, p):
        self.done.add(id(p))
        self.works.append(dist.all_reduce(p.grad, op=dist.ReduceOp.SUM, group=self.group, async_op=True))

    def arm(self) -> None:
        self.works, self.done = [], set()
        self.handles = [p.register_post_accumulate_grad_hook(self._hook) for p in self.params]

    def wait(self) -> None:
        for h in self.handles:
            h.remove()
        self.handles = []
        for p in self.params:
            if id(p) not in self.done:
                if p.grad is None:
                    p.grad = torch.zeros_like(p)
                self.works.append(dist.all_reduce(p.grad, op=dist.ReduceOp.SUM, group=self.group,
                                                  async_op=True))
        for w in self.works:
            w.wait()
        self.works = []
