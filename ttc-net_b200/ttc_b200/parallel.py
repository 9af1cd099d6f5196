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
