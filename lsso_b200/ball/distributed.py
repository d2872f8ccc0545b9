"""Data-parallel gradient reduction for the LSSO layer (one process per GPU).

Samples are independent, so the batch shards over ranks and the forward needs
no collective.  After the backward, every rank holds the parameter gradients
of its shard; ``allreduce_gradients`` packs them into one flat FP32 buffer,
runs a single ``all_reduce`` (NCCL over NVLink on B200 ranks, gloo on CPU) and
writes the average back, matching DDP's mean over ranks.
"""

from __future__ import annotations

from typing import Iterable

import torch
import torch.distributed as dist


def allreduce_gradients(parameters: Iterable[torch.nn.Parameter], *, group=None,
                        buffer: torch.Tensor | None = None, average: bool = True) -> torch.Tensor | None:
    """Average ``p.grad`` of ``parameters`` over the process group in one collective.

    Parameters without a gradient contribute zeros (and receive the average
    of the others).  Returns the flat buffer used (pass it back in to reuse).
    """
    params = [p for p in parameters]
    if not dist.is_available() or not dist.is_initialized():
        return buffer
    world = dist.get_world_size(group)
    if world == 1 or not params:
        return buffer
    device = params[0].device
    total = sum(p.numel() for p in params)
    if buffer is None or buffer.numel() != total or buffer.device != device:
        buffer = torch.empty(total, dtype=torch.float32, device=device)
    # One gather kernel into the flat buffer, one collective, one scatter kernel
    # back (multi-tensor copy), instead of a copy launch per parameter each way.
    grads = [p.grad.reshape(-1) if p.grad is not None else torch.zeros(p.numel(), device=device,
                                                                       dtype=torch.float32) for p in params]
    torch.cat([g.to(torch.float32) for g in grads], out=buffer)
    dist.all_reduce(buffer, op=dist.ReduceOp.SUM, group=group)
    if average:
        buffer.div_(world)
    views = list(buffer.split([p.numel() for p in params]))
    missing = [i for i, p in enumerate(params) if p.grad is None]
    for i in missing:
        params[i].grad = views[i].view_as(params[i]).to(params[i].dtype).clone()
    present = [i for i, p in enumerate(params) if p.grad is not None and i not in missing]
    if present:
        torch._foreach_copy_([params[i].grad for i in present],
                             [views[i].view_as(params[i]).to(params[i].grad.dtype) for i in present])
    return buffer


__all__ = ["allreduce_gradients"]
