"""Two NCCL ranks (launched by tests/test_exchange_gpu.py): GradientExchange
against allreduce_gradients' single collective, eagerly and as CUDA-graph
replays holding the exchange, for both transports: NCCL collectives
overlapped with the backward, and the library's peer-memory kernel, per
bucket under the backward and in one launch after it (whose averages must
also be bit-identical on the two ranks)."""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    rank = dist.get_rank()
    from lsso import LSSO, LSSOConfig
    from lsso.ball import cuda
    from lsso_b200.ball.distributed import GradientExchange, allreduce_gradients, layer_buckets

    cuda.load(device=local)
    torch.manual_seed(0)
    layer = LSSO(LSSOConfig(256, 8, 32, bias=True)).to(device)
    params = list(layer.parameters())
    x = torch.randn(2, 1500, 256, generator=torch.Generator().manual_seed(10 + rank)).half().to(device)

    def step():
        for q in params:
            q.grad = None
        with torch.autocast("cuda", dtype=torch.float16, cache_enabled=False):
            y = layer(x, implementation="cuda")
        y.float().square().mean().backward()

    step()
    allreduce_gradients(params)
    reference = [q.grad.clone() for q in params]

    ok = True
    rel = lambda u, v: float((u - v).norm() / v.norm().clamp_min(1e-30))  # noqa: E731
    for transport, overlap in (("nccl", True), ("peer", True), ("peer", False)):
        exchange = GradientExchange(layer_buckets(layer), transport=transport, overlap=overlap)
        ok &= exchange.transport == transport
        for _ in range(2):
            step()
            exchange.finish()
            errors = [rel(q.grad, g) for q, g in zip(params, reference)]
            ok &= max(errors) < 1e-6
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            step()
            exchange.finish()
        torch.cuda.current_stream(device).wait_stream(side)
        for q in params:
            q.grad = None
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
            exchange.finish()
        for _ in range(3):
            exchange.flat.zero_()
            graph.replay()
        torch.cuda.synchronize()
        errors = [rel(q.grad, g) for q, g in zip(params, reference)]
        if rank == 0:
            print(f"{transport} (overlap={overlap}): graph replay errors vs one-collective average:",
                  " ".join(f"{e:.1e}" for e in errors))
        ok &= max(errors) < 1e-6
        if transport == "peer":
            # every rank sums in rank order: the averages agree bit for bit
            mine = torch.cat([q.grad.reshape(-1) for q in params])
            both = [torch.empty_like(mine) for _ in range(dist.get_world_size())]
            dist.all_gather(both, mine)
            ok &= all(torch.equal(both[0], b) for b in both)
            from lsso_b200.ball import _native
            ok &= _native.device_status(reset=True) == 0
        del graph
        exchange.close()
    flag = torch.tensor([1 if ok else 0], device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0 and flag.item():
        print("exchange ok")
    return 0 if flag.item() else 1


if __name__ == "__main__":
    raise SystemExit(main())
