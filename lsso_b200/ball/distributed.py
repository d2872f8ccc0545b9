"""Data-parallel gradient reduction for the LSSO layer (one process per GPU).

Samples are independent, so the batch shards over ranks and the forward needs
no collective.  After the backward, every rank holds the parameter gradients
of its shard, and their average over ranks (DDP's mean) is what every rank
applies.  Two ways to get it:

* ``allreduce_gradients``: after the backward, pack every gradient into one
  flat FP32 buffer, one ``all_reduce`` (NCCL over NVLink on B200 ranks, gloo
  on CPU), write the average back.  Simple; the exchange follows the backward.
* ``GradientExchange``: every gradient has a slot in a persistent flat
  buffer, grouped into buckets in the order the backward produces them
  (``layer_buckets``: the output projection and the mixer's compact
  parameters, then the input projection).  The projection weight gradients
  are written by the library straight into their slots, and a bucket's
  ``all_reduce`` is launched on a side stream the moment it is complete --
  from inside the input projection's backward, before its input-gradient
  GEMM -- so the exchange runs under the rest of the backward.  ``finish()``
  joins the side stream and points each ``p.grad`` at its averaged slot.

  With ``transport="peer"`` (the default for CUDA ranks on one host, through
  ``"auto"``) the flat buffer is the library's IPC-shared exchange region and
  each complete bucket is averaged by the library's one-shot all-reduce
  kernel (on the side stream, under the rest of the backward), which reads
  every rank's part of the buffer over NVLink and writes the average on
  every rank, in place of NCCL.  Buckets go out in bucket order on every
  rank whatever order they complete in, so the ranks' exchanges pair up.
"""

from __future__ import annotations

from typing import Iterable

import torch
import torch.distributed as dist

from . import peer, projection


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


def layer_buckets(layer) -> list[list[torch.nn.Parameter]]:
    """Buckets of an ``LSSO`` layer's parameters in the order its backward
    finishes them: output projection + compact parameters, then the input
    projection."""
    first = [layer.w_o.weight, layer.w_o.bias, layer.core_base_raw, layer.core_drive_weight, layer.eta_raw]
    last = [layer.w_bc.weight, layer.w_bc.bias]
    return [[p for p in first if p is not None], [p for p in last if p is not None]]


class GradientExchange:
    """Gradient average over the process group, overlapped with the backward.

    ``buckets``: lists of parameters, each list complete at one point of the
    backward (``layer_buckets(layer)``, or the concatenation of several
    layers' buckets).  Usage per step: clear the gradients (``p.grad = None``,
    as ``optimizer.zero_grad()`` does), run the backward, call ``finish()``.
    Works under CUDA-graph capture (the collectives are recorded with the
    step).  With one rank it only points ``p.grad`` at the flat buffer.
    """

    def __init__(self, buckets: list[list[torch.nn.Parameter]], *, group=None, average: bool = True,
                 overlap: bool = True, transport: str = "auto") -> None:
        self.buckets = [list(b) for b in buckets if b]
        params = [p for b in self.buckets for p in b]
        if not params:
            raise ValueError("GradientExchange needs at least one parameter")
        if transport not in ("auto", "peer", "nccl"):
            raise ValueError(f"transport must be 'auto', 'peer' or 'nccl', got {transport!r}")
        self.group = group
        self.average = average
        # overlap=False: every bucket goes out in finish(), after the backward, in one collective
        # on the current stream (no side stream competing with the backward's kernels for SMs)
        self.overlap = overlap
        device = params[0].device
        # each bucket starts at a multiple of four values (16 bytes: the peer
        # exchange reads and writes whole float4 columns of a bucket)
        sizes = [sum(p.numel() for p in b) for b in self.buckets]
        self.bucket_start = []
        total = 0
        for size in sizes:
            self.bucket_start.append(total)
            total += (size + 3) // 4 * 4
        # transport: "peer" sums the ranks' buffers with the library's exchange kernel over peer
        # memory, one launch per bucket; "nccl" uses the process group's all_reduce; "auto"
        # takes "peer" when every rank can map the others' memory.
        self.peers = None
        if transport != "nccl" and self._world() > 1:
            if device.type != "cuda":
                if transport == "peer":
                    raise ValueError("transport='peer' needs CUDA parameters")
            else:
                try:
                    self.peers = peer.PeerGroup(total, device, group=group)
                except peer.PeerUnavailable:
                    if transport == "peer":
                        raise
        self.transport = "peer" if self.peers is not None else ("nccl" if self._world() > 1 else "none")
        if self.peers is not None:
            self.flat = self.peers.values
            self.flat.zero_()
            self.averaged = torch.empty_like(self.flat)
        else:
            self.flat = torch.zeros(total, dtype=torch.float32, device=device)
            self.averaged = self.flat
        self.slot = {}
        self.result = {}
        self.bucket_of = {}
        for k, bucket in enumerate(self.buckets):
            offset = self.bucket_start[k]
            for p in bucket:
                if p.dtype != torch.float32:
                    raise TypeError("GradientExchange keeps FP32 gradients; got a parameter of " + str(p.dtype))
                self.slot[p] = self.flat.narrow(0, offset, p.numel()).view_as(p)
                self.result[p] = self.averaged.narrow(0, offset, p.numel()).view_as(p)
                self.bucket_of[p] = k
                offset += p.numel()
        self.bucket_size = sizes
        self.bucket_flat = [self.flat.narrow(0, s, n) for s, n in zip(self.bucket_start, sizes)]
        self.bucket_out = [self.averaged.narrow(0, s, n) for s, n in zip(self.bucket_start, sizes)]
        self.stream = torch.cuda.Stream(device) if device.type == "cuda" else None
        self._ready = [set() for _ in self.buckets]
        self._launched = [False] * len(self.buckets)
        self._next = 0  # buckets [0, _next) are launched; launches go in bucket order
        self._side_used = False
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_accumulated) for p in params]
        for p in params:  # the projections write their weight and bias gradients straight into these
            projection.register_gradient_slot(p, self.slot[p], self._on_written)

    # ------------------------------------------------------------------ internals
    def _world(self) -> int:
        if not dist.is_available() or not dist.is_initialized():
            return 1
        return dist.get_world_size(self.group)

    def _mark(self, p: torch.nn.Parameter) -> None:
        k = self.bucket_of[p]
        self._ready[k].add(p)
        if not self.overlap:
            return
        # every complete bucket from the next unlaunched one on, in order (the same on all ranks)
        while self._next < len(self.buckets) and len(self._ready[self._next]) == len(self.buckets[self._next]):
            self._launch(self._next)

    def _on_written(self, p: torch.nn.Parameter) -> None:
        """The library wrote p's gradient of this backward into its slot."""
        self._mark(p)

    def _on_accumulated(self, p: torch.nn.Parameter) -> None:
        if p in self._ready[self.bucket_of[p]]:
            return
        slot = self.slot[p]
        if p.grad is not None and p.grad.data_ptr() != slot.data_ptr():
            slot.copy_(p.grad)
        self._mark(p)

    def _launch(self, k: int) -> None:
        self._launched[k] = True
        self._next = k + 1
        world = self._world()
        if world == 1:
            return
        buf = self.bucket_flat[k]
        if self.peers is not None:
            # the library's exchange kernel for this bucket's part of every rank's region
            current = torch.cuda.current_stream(buf.device)
            self.stream.wait_stream(current)
            self._side_used = True
            with torch.cuda.stream(self.stream):
                self.peers.reduce(self.bucket_out[k], 1.0 / self.peers.world if self.average else 1.0,
                                  first=self.bucket_start[k], count=self.bucket_size[k])
            return
        if self.stream is None:
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group)
            if self.average:
                buf.div_(world)
            return
        current = torch.cuda.current_stream(buf.device)
        self.stream.wait_stream(current)
        self._side_used = True
        with torch.cuda.stream(self.stream):
            op = dist.ReduceOp.AVG if self.average else dist.ReduceOp.SUM
            dist.all_reduce(buf, op=op, group=self.group)

    # ------------------------------------------------------------------ API
    def finish(self) -> None:
        """Complete the exchange of this backward: launch what is left (a
        parameter that got no gradient contributes zeros), make the current
        stream wait for the collectives, and set every ``p.grad`` to its
        averaged slot."""
        for k, bucket in enumerate(self.buckets):
            if self._launched[k]:
                continue
            for p in bucket:
                if p not in self._ready[k]:
                    self.slot[p].zero_()
            if self.overlap:
                self._launch(k)
        if not self.overlap and self.peers is not None:
            self.peers.reduce(self.averaged, 1.0 / self.peers.world if self.average else 1.0)
        elif not self.overlap and self._world() > 1:
            if self.stream is None:
                dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group)
                if self.average:
                    self.flat.div_(self._world())
            else:
                op = dist.ReduceOp.AVG if self.average else dist.ReduceOp.SUM
                dist.all_reduce(self.flat, op=op, group=self.group)
        if self._side_used:
            torch.cuda.current_stream(self.flat.device).wait_stream(self.stream)
        for bucket in self.buckets:
            for p in bucket:
                p.grad = self.result[p]
        self._ready = [set() for _ in self.buckets]
        self._launched = [False] * len(self.buckets)
        self._next = 0
        self._side_used = False

    def close(self) -> None:
        """Remove the hooks and the library's gradient slots of these parameters."""
        for h in self._hooks:
            h.remove()
        for p in self.slot:
            projection.register_gradient_slot(p, None, None)
        self._hooks = []
        if self.peers is not None:
            self.peers.close()


__all__ = ["GradientExchange", "allreduce_gradients", "layer_buckets"]
