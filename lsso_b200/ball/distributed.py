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
    offset = 0
    for p in params:
        n = p.numel()
        view = buffer[offset:offset + n]
        if p.grad is None:
            view.zero_()
        else:
            view.copy_(p.grad.reshape(-1))
        offset += n
    dist.all_reduce(buffer, op=dist.ReduceOp.SUM, group=group)
    if average:
        buffer.div_(world)
    offset = 0
    for p in params:
        n = p.numel()
        flat = buffer[offset:offset + n].view_as(p)
        if p.grad is None:
            p.grad = flat.to(p.dtype).clone()
        else:
            p.grad.copy_(flat)
        offset += n
    return buffer


__all__ = ["allreduce_gradients"]
